/*
 * C restatement of the hot-path oracle — TEST / BASELINE INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline and
 * reference arm load this library; the product path never does.
 *
 * Same formulas as oracle/expressions.py, i.e. the reference's numpy oracle
 * (tools/expressions_open.py:27-104, float64 intermediates cast to float32)
 * and its GELU formula (tests/test_gelu.py:51-66), split over POSIX threads
 * so the CPU baseline can use every host core (oc_set_threads).  It is
 * checked against the numpy oracle by tests/test_oracle_c.py.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdint.h>
#include <stdlib.h>
#include <unistd.h>

static int g_threads = 0;

int oc_default_threads(void) {
  cpu_set_t set;
  if (sched_getaffinity(0, sizeof(set), &set) == 0) return CPU_COUNT(&set);
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

void oc_set_threads(int n) { g_threads = n; }
int oc_threads(void) { return g_threads > 0 ? g_threads : oc_default_threads(); }

typedef void (*range_fn)(void *ctx, int64_t begin, int64_t end);
struct task { range_fn fn; void *ctx; int64_t begin, end; };

static void *run_task(void *arg) {
  struct task *t = (struct task *)arg;
  t->fn(t->ctx, t->begin, t->end);
  return NULL;
}

/* Runs fn over [0, n) in oc_threads() contiguous chunks (serially below min_items). */
static void parallel_for_min(int64_t n, int64_t min_items, range_fn fn, void *ctx) {
  int t = oc_threads();
  if (t > 256) t = 256;
  if (n < min_items || t <= 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t ids[256];
  struct task tasks[256];
  const int64_t chunk = (n + t - 1) / t;
  int started = 0;
  for (int i = 0; i < t; ++i) {
    int64_t b = i * chunk, e = b + chunk < n ? b + chunk : n;
    if (b >= e) break;
    tasks[i] = (struct task){fn, ctx, b, e};
    if (pthread_create(&ids[i], NULL, run_task, &tasks[i]) != 0) {
      run_task(&tasks[i]);
      ids[i] = 0;
    }
    started = i + 1;
  }
  for (int i = 0; i < started; ++i)
    if (ids[i]) pthread_join(ids[i], NULL);
}

static void parallel_for(int64_t n, range_fn fn, void *ctx) { parallel_for_min(n, 4096, fn, ctx); }

struct ew { const float *x0, *x1; float *out; float a, b; int mode; };

static void ew_range(void *p, int64_t b, int64_t e) {
  const struct ew *c = (const struct ew *)p;
  for (int64_t i = b; i < e; ++i) {
    const float v = c->x0[i];
    switch (c->mode) {
      case 0: c->out[i] = v + c->x1[i]; break;
      case 1: { volatile float prod = v * c->a; c->out[i] = prod + c->b; break; }
      case 2: c->out[i] = (v > 0.0f ? v : 0.0f) * c->x1[i]; break;
      case 3: {
        const float scaled = v / 1.4142135623730951f;
        const float gate = (float)erf((double)scaled);
        c->out[i] = (0.5f * v) * (1.0f + gate);
        break;
      }
      default: {
        const float cube = (v * v) * v;
        const float scaled = 0.7978845608028654f * (v + 0.044715f * cube);
        const float gate = (float)tanh((double)scaled);
        c->out[i] = (0.5f * v) * (1.0f + gate);
      }
    }
  }
}

void oc_add(const float *x0, const float *x1, float *out, int64_t n) {
  struct ew c = {x0, x1, out, 0, 0, 0};
  parallel_for(n, ew_range, &c);
}
void oc_axpb(float a, float b, const float *x, float *out, int64_t n) {
  struct ew c = {x, NULL, out, a, b, 1};
  parallel_for(n, ew_range, &c);
}
void oc_relumul(const float *x, const float *y, float *out, int64_t n) {
  struct ew c = {x, y, out, 0, 0, 2};
  parallel_for(n, ew_range, &c);
}
void oc_gelu(int tanh_form, const float *x, float *out, int64_t n) {
  struct ew c = {x, NULL, out, 0, 0, tanh_form ? 4 : 3};
  parallel_for(n, ew_range, &c);
}

struct sum_ctx { const float *x; double part[256]; int64_t chunk; };
static void sum_range(void *p, int64_t b, int64_t e) {
  struct sum_ctx *c = (struct sum_ctx *)p;
  double s = 0.0;
  for (int64_t i = b; i < e; ++i) s += (double)c->x[i];
  c->part[c->chunk ? b / c->chunk : 0] = s;
}
double oc_sum(const float *x, int64_t n) {
  struct sum_ctx c;
  int t = oc_threads();
  if (t > 256) t = 256;
  for (int i = 0; i < 256; ++i) c.part[i] = 0.0;
  c.x = x;
  c.chunk = (n < 4096 || t <= 1) ? 0 : (n + t - 1) / t;
  parallel_for(n, sum_range, &c);
  double s = 0.0;
  for (int i = 0; i < 256; ++i) s += c.part[i];
  return s;
}

struct rows { const float *x, *w; float *out; int64_t cols; double eps, count; int mode; };
static void row_range(void *p, int64_t b, int64_t e) {
  const struct rows *c = (const struct rows *)p;
  const int64_t cols = c->cols;
  for (int64_t r = b; r < e; ++r) {
    const float *xr = c->x + r * cols;
    float *o = c->out + r * cols;
    if (c->mode == 0) {
      double s = 0.0;
      for (int64_t j = 0; j < cols; ++j) s += (double)xr[j];
      c->out[r] = (float)s;
    } else if (c->mode == 2) {
      double m = -INFINITY, s = 0.0;
      for (int64_t j = 0; j < cols; ++j) m = xr[j] > m ? xr[j] : m;
      for (int64_t j = 0; j < cols; ++j) s += exp((double)xr[j] - m);
      for (int64_t j = 0; j < cols; ++j) o[j] = (float)(exp((double)xr[j] - m) / s);
    } else {
      double ss = 0.0;
      for (int64_t j = 0; j < cols; ++j) ss += (double)xr[j] * (double)xr[j];
      if (c->mode == 1) {
        const double inv = 1.0 / sqrt(ss / c->count + c->eps);
        for (int64_t j = 0; j < cols; ++j) o[j] = (float)((double)xr[j] * inv * (double)c->w[j]);
      } else {
        const double inv = 1.0 / sqrt(ss);
        for (int64_t j = 0; j < cols; ++j) o[j] = (float)((double)xr[j] * inv);
      }
    }
  }
}
static void rows_run(struct rows *c, int64_t rows) { parallel_for_min(rows, 2, row_range, c); }
void oc_rowsum(const float *x, float *out, int64_t rows, int64_t cols) {
  struct rows c = {x, NULL, out, cols, 0, 0, 0};
  rows_run(&c, rows);
}
void oc_rmsnorm(const float *x, const float *w, float *out, int64_t rows, int64_t cols, double eps,
                double count) {
  struct rows c = {x, w, out, cols, eps, count, 1};
  rows_run(&c, rows);
}
void oc_softmax(const float *x, float *out, int64_t rows, int64_t cols) {
  struct rows c = {x, NULL, out, cols, 0, 0, 2};
  rows_run(&c, rows);
}
void oc_l2norm(const float *x, float *out, int64_t rows, int64_t cols) {
  struct rows c = {x, NULL, out, cols, 0, 0, 3};
  rows_run(&c, rows);
}
