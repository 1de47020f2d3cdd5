// FP32 attention, O = epilogue(softmax(score(Q Kt)) V), the reference's scalar
// attention class.
//
// Replaces the per-output online-softmax kernels Emmy schedules for FP32
// attention (problems/a01_attention, problems/a02_attention_128,
// examples/phase9/generated/phase9_gelu_attention): every thread of those
// kernels walks all keys for its (query row, value column) pairs, recomputing
// each q.kt dot product, with exp(x) = ex2.approx(x * log2 e)
// (ptx_backend.py:1062-1068), reciprocal = 1 / x correctly rounded
// (ptx_backend.py:1047-1048) and the coupled (max, sum, acc) accumulators of
// the IR (running max seeded with -1e30).
//
// Here one CTA of 256 threads owns 128 query rows of one (batch, head): Q is
// staged once in shared memory (transposed), then per 64-key block Kt and V
// are staged (cp.async into two buffers: the next block's copies are in
// flight while this one is computed), each thread computes an 8 x 4 block of
// scores with FFMA (two Q and one Kt 16-byte shared loads per 32 FMAs), the
// row max and sum are combined across the 16 threads sharing a row by
// shuffles, P goes through shared memory and each thread accumulates an 8 x 4
// (head size <= 64) or 8 x 8 (<= 128) block of O in registers.  The score is
// dot * c, dot * (1/c) or dot / c for the 1-element scale buffer c, matching
// the three forms the IR can take.  Head sizes above 128 take a direct kernel
// with one thread per output element.
#include "common.cuh"
#include "epilogue.cuh"

namespace lc {
namespace {

constexpr int RPT = 8;         // query rows per thread (a thread computes RPT x 4 scores)
constexpr int BQ = 16 * RPT;   // query rows per CTA
constexpr int BKV = 64;
constexpr int kThreads = 256;
constexpr int kMaxTiled = 128;
constexpr int QS = BQ + 4;  // padded row of the transposed Q tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMaxIdentity = -1e30f;  // the IR's identity of `maximum`

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// exp as the reference lowers it
__device__ __forceinline__ float exp_ref(float x) { return ex2_approx(__fmul_rn(x, kLog2e)); }

// 4-byte asynchronous copy global -> shared; an invalid element is zero-filled
// (no bytes are read from `src`, which stays a valid address)
__device__ __forceinline__ void cp_async4(float *dst, const float *src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ float apply_scale(float dot, float c, float rc, int mode) {
  if (mode == LC_SCALE_MUL) return __fmul_rn(dot, c);
  if (mode == LC_SCALE_MUL_RECIP) return __fmul_rn(dot, rc);
  return __fdiv_rn(dot, c);
}

template <int DVH, int EPI, bool COMP = false>
__global__ void __launch_bounds__(kThreads) attention_f32_kernel(
    const float *__restrict__ q, const float *__restrict__ kt, const float *__restrict__ v,
    float *__restrict__ o, int s_q, int s_kv, int d, int dv, const float *__restrict__ scale,
    int scale_mode) {
  constexpr int DVW = 64 * DVH;  // value columns staged per key
  extern __shared__ float4 smem4[];
  float *Qs = reinterpret_cast<float *>(smem4);  // [d][QS]   Q transposed
  float *Kbuf = Qs + d * QS;                      // 2 x [d][BKV]  Kt blocks (double-buffered)
  float *Vbuf = Kbuf + 2 * d * BKV;               // 2 x [BKV][DVW]
  float *Ps = Vbuf + 2 * BKV * DVW;               // [BKV][BQ]  P transposed

  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int bh = blockIdx.y;
  const int q0 = blockIdx.x * BQ;
  const float *qb = q + (int64_t)bh * s_q * d;
  const float *kb = kt + (int64_t)bh * d * s_kv;
  const float *vb = v + (int64_t)bh * s_kv * dv;
  const float c = scale[0];
  const float rc = __frcp_rn(c);

  for (int idx = t; idx < BQ * d; idx += kThreads) {
    const int row = idx / d, dd = idx - row * d;
    Qs[dd * QS + row] = q0 + row < s_q ? qb[(int64_t)(q0 + row) * d + dd] : 0.f;
  }

  float m[RPT], l[RPT], acc[RPT][4 * DVH];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    m[i] = kMaxIdentity;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4 * DVH; ++j) acc[i][j] = 0.f;
  }

  // Kt / V of the block starting at key k into buffer b, asynchronously (the
  // next block's copies overlap this block's arithmetic)
  auto stage = [&](int k, int b) {
    float *ks = Kbuf + b * d * BKV;
    float *vs = Vbuf + b * BKV * DVW;
    for (int idx = t; idx < d * BKV; idx += kThreads) {
      const int dd = idx / BKV, key = idx - dd * BKV;
      const bool ok = k + key < s_kv;
      cp_async4(ks + idx, ok ? kb + (int64_t)dd * s_kv + k + key : kb, ok);
    }
    for (int idx = t; idx < BKV * DVW; idx += kThreads) {
      const int key = idx / DVW, col = idx - key * DVW;
      const bool ok = k + key < s_kv && col < dv;
      cp_async4(vs + idx, ok ? vb + (int64_t)(k + key) * dv + col : vb, ok);
    }
  };
  stage(0, 0);
  cp_async_commit();
  int buf = 0;
  for (int k0 = 0; k0 < s_kv; k0 += BKV, buf ^= 1) {
    if (k0 + BKV < s_kv) stage(k0 + BKV, buf ^ 1);  // that buffer's last readers passed the barrier below
    cp_async_commit();
    cp_async_wait_1();  // this block's copies (all groups but the newest) have landed
    __syncthreads();
    const float *Ks = Kbuf + buf * d * BKV;
    const float *Vs = Vbuf + buf * BKV * DVW;

    float s[RPT][4], s_low[COMP ? RPT : 1][COMP ? 4 : 1];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    if constexpr (COMP) {
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s_low[i][j] = 0.f;
    }
    for (int dd = 0; dd < d; ++dd) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&Qs[dd * QS + ty * RPT]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&Qs[dd * QS + ty * RPT + 4]);
      const float4 b = *reinterpret_cast<const float4 *>(&Ks[dd * BKV + tx * 4]);
      const float av[RPT] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
      if constexpr (COMP) {
        // the score dot as a Dot2 pair, in the IR's operand order kt * q
#pragma unroll
        for (int i = 0; i < RPT; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) dot2_step(s[i][j], s_low[i][j], bv[j], av[i]);
      } else {
#pragma unroll
        for (int i = 0; i < RPT; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) s[i][j] = fmaf(av[i], bv[j], s[i][j]);
      }
    }
    if constexpr (COMP) {
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = dot2_value(s[i][j], s_low[i][j]);
    }

#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x = apply_scale(s[i][j], c, rc, scale_mode);
        s[i][j] = k0 + tx * 4 + j < s_kv ? x : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m[i], mx);
      const float alpha = exp_ref(__fsub_rn(m[i], m_new));
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = exp_ref(__fsub_rn(s[i][j], m_new));
        sum = __fadd_rn(sum, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
      l[i] = __fadd_rn(__fmul_rn(l[i], alpha), sum);
      m[i] = m_new;
#pragma unroll
      for (int j = 0; j < 4 * DVH; ++j) acc[i][j] = __fmul_rn(acc[i][j], alpha);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 *dst = reinterpret_cast<float4 *>(&Ps[(tx * 4 + j) * BQ + ty * RPT]);
      dst[0] = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
      dst[1] = make_float4(s[4][j], s[5][j], s[6][j], s[7][j]);
    }
    __syncthreads();

    const int keys = s_kv - k0 < BKV ? s_kv - k0 : BKV;
    for (int key = 0; key < keys; ++key) {
      const float4 p0 = *reinterpret_cast<const float4 *>(&Ps[key * BQ + ty * RPT]);
      const float4 p1 = *reinterpret_cast<const float4 *>(&Ps[key * BQ + ty * RPT + 4]);
      const float pv[RPT] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int h = 0; h < DVH; ++h) {
        const float4 w = *reinterpret_cast<const float4 *>(&Vs[key * DVW + h * 64 + tx * 4]);
        const float wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < RPT; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][h * 4 + j] = fmaf(pv[i], wv[j], acc[i][h * 4 + j]);
      }
    }
    __syncthreads();  // every thread is done with this block's Kt, V and P before they are reused
  }

  float *ob = o + (int64_t)bh * s_q * dv;
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = q0 + ty * RPT + i;
    if (row >= s_q) continue;
    const float inv = __frcp_rn(l[i]);
#pragma unroll
    for (int h = 0; h < DVH; ++h)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = h * 64 + tx * 4 + j;
        if (col < dv) ob[(int64_t)row * dv + col] = apply_epilogue<EPI>(__fmul_rn(acc[i][h * 4 + j], inv));
      }
  }
}

// Any head size: one thread per output element, online softmax over the keys
// in order, the arithmetic of the tiled kernel.
template <int EPI, bool COMP = false>
__global__ void __launch_bounds__(256) attention_f32_direct_kernel(
    const float *__restrict__ q, const float *__restrict__ kt, const float *__restrict__ v,
    float *__restrict__ o, int64_t bh, int s_q, int s_kv, int d, int dv,
    const float *__restrict__ scale, int scale_mode) {
  const int64_t total = bh * s_q * dv;
  const float c = scale[0];
  const float rc = __frcp_rn(c);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int col = (int)(e % dv);
    const int64_t r = e / dv;
    const int row = (int)(r % s_q);
    const int64_t b = r / s_q;
    const float *qr = q + (b * s_q + row) * d;
    const float *kb = kt + b * d * s_kv;
    const float *vb = v + b * s_kv * dv;
    float m = kMaxIdentity, l = 0.f, acc = 0.f;
    for (int key = 0; key < s_kv; ++key) {
      float dot = 0.f, dot_low = 0.f;
      if constexpr (COMP) {
        for (int dd = 0; dd < d; ++dd) dot2_step(dot, dot_low, kb[(int64_t)dd * s_kv + key], qr[dd]);
        dot = dot2_value(dot, dot_low);
      } else {
        for (int dd = 0; dd < d; ++dd) dot = fmaf(qr[dd], kb[(int64_t)dd * s_kv + key], dot);
      }
      const float x = apply_scale(dot, c, rc, scale_mode);
      const float m_new = fmaxf(m, x);
      const float alpha = exp_ref(__fsub_rn(m, m_new));
      const float p = exp_ref(__fsub_rn(x, m_new));
      l = __fadd_rn(__fmul_rn(l, alpha), p);
      acc = __fadd_rn(__fmul_rn(acc, alpha), __fmul_rn(vb[(int64_t)key * dv + col], p));
      m = m_new;
    }
    o[e] = apply_epilogue<EPI>(__fmul_rn(acc, __frcp_rn(l)));
  }
}

// The fragment attention tile (examples/phase9/fragments/fragment_attention_tile_f16):
// Q, Kt and V are read as f16 (round to nearest), S = Q Kt accumulates their
// exact products in f32, each row is normalised before the PV product
// (max, exp(s - max) = ex2.approx((s - max) log2 e), row sum, correctly rounded
// division) and the weights are rounded to f16 — the reference's
// FragmentRowReduce / FragmentApply / FragmentRepack chain
// (ptx_tensor.py:459-618) — and O = P V accumulates in f32.  One warp per
// query row: lanes stride over keys for the statistics and over output columns
// for O; the row's f16 weights live in shared memory.
constexpr int kTileWarps = 4;
constexpr int kTileMaxKeys = 4096;

__device__ __forceinline__ float f16r(float x) { return __half2float(__float2half_rn(x)); }

__global__ void __launch_bounds__(32 * kTileWarps) attention_tile_f16q_kernel(
    const float *__restrict__ q, const float *__restrict__ kt, const float *__restrict__ v,
    float *__restrict__ o, int s_q, int s_kv, int d, int dv) {
  __shared__ __half pw[kTileWarps][kTileMaxKeys];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kTileWarps + warp;
  const int64_t bh = blockIdx.y;
  if (row >= s_q) return;
  const float *qr = q + (bh * s_q + row) * d;
  const float *kb = kt + bh * d * s_kv;
  const float *vb = v + bh * s_kv * dv;
  auto score = [&](int key) {
    float acc = 0.f;
    for (int dd = 0; dd < d; ++dd) acc = fmaf(f16r(qr[dd]), f16r(kb[(int64_t)dd * s_kv + key]), acc);
    return acc;
  };
  float mx = -INFINITY;
  for (int key = lane; key < s_kv; key += 32) mx = fmaxf(mx, score(key));
  mx = warp_max(mx);
  float sum = 0.f;
  for (int key = lane; key < s_kv; key += 32) sum += exp_ref(__fsub_rn(score(key), mx));
  sum = warp_sum(sum);
  for (int key = lane; key < s_kv; key += 32)
    pw[warp][key] = __float2half_rn(__fdiv_rn(exp_ref(__fsub_rn(score(key), mx)), sum));
  __syncwarp();
  float *orow = o + (bh * s_q + row) * dv;
  for (int c = lane; c < dv; c += 32) {
    float acc = 0.f;
    for (int key = 0; key < s_kv; ++key)
      acc = fmaf(__half2float(pw[warp][key]), f16r(vb[(int64_t)key * dv + c]), acc);
    orow[c] = acc;
  }
}

size_t tiled_smem(int d, int dvh) {
  return (size_t)(d * QS + 2 * d * BKV + 2 * BKV * 64 * dvh + BKV * BQ) * sizeof(float);
}

template <int DVH, int EPI, bool COMP>
int launch_tiled(const float *q, const float *kt, const float *v, float *o, int64_t bh, int s_q,
                 int s_kv, int d, int dv, const float *scale, int mode, cudaStream_t s) {
  auto kernel = attention_f32_kernel<DVH, EPI, COMP>;
  const size_t smem = tiled_smem(d, DVH);
  if (smem > 48 * 1024) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)tiled_smem(kMaxTiled, DVH)),
                            "attention smem attribute"))
      return rc;
  }
  dim3 grid((s_q + BQ - 1) / BQ, (unsigned)bh);
  kernel<<<grid, kThreads, smem, s>>>(q, kt, v, o, s_q, s_kv, d, dv, scale, mode);
  return check_launch("lc_attention_f32");
}

template <int EPI, bool COMP>
int launch(const float *q, const float *kt, const float *v, float *o, int64_t bh, int s_q,
           int s_kv, int d, int dv, const float *scale, int mode, cudaStream_t s) {
  if (d <= kMaxTiled && dv <= kMaxTiled) {
    if (dv <= 64) return launch_tiled<1, EPI, COMP>(q, kt, v, o, bh, s_q, s_kv, d, dv, scale, mode, s);
    return launch_tiled<2, EPI, COMP>(q, kt, v, o, bh, s_q, s_kv, d, dv, scale, mode, s);
  }
  const int64_t total = bh * s_q * dv;
  const int64_t blocks = (total + 255) / 256;
  const int64_t cap = 16LL * sm_count();
  attention_f32_direct_kernel<EPI, COMP><<<(int)(blocks < cap ? blocks : cap), 256, 0, s>>>(
      q, kt, v, o, bh, s_q, s_kv, d, dv, scale, mode);
  return check_launch("lc_attention_f32 (direct)");
}

}  // namespace
}  // namespace lc

namespace {
int attention_f32_entry(bool comp, int scale_mode, int epilogue, const void *scale, const void *q,
                        const void *kt, const void *v, void *o, int64_t bh, int64_t s_q, int64_t s_kv,
                        int64_t d, int64_t dv, void *stream) {
  using namespace lc;
  if (scale_mode != LC_SCALE_MUL && scale_mode != LC_SCALE_MUL_RECIP && scale_mode != LC_SCALE_DIV)
    return fail(LC_ERR_INVALID, "lc_attention_f32: unknown scale mode %d", scale_mode);
  if (epilogue < LC_EPI_NONE || epilogue > LC_EPI_GELU_TANH)
    return fail(LC_ERR_INVALID, "lc_attention_f32: unknown epilogue %d", epilogue);
  if (bh < 0 || s_q < 0 || s_kv < 0 || d < 0 || dv < 0)
    return fail(LC_ERR_INVALID, "lc_attention_f32: negative shape");
  if (bh > 65535 || s_q > 0x7fffffff || s_kv > 0x7fffffff || d > 0x7fffffff || dv > 0x7fffffff)
    return fail(LC_ERR_UNSUPPORTED, "lc_attention_f32: shape beyond the supported range");
  if (bh == 0 || s_q == 0 || dv == 0) return LC_OK;
  // empty operands may be null: Q when d = 0, V when s_kv = 0, Kt when either is
  if (!o || !scale || (d > 0 && !q) || (s_kv > 0 && !v) || (d > 0 && s_kv > 0 && !kt))
    return fail(LC_ERR_INVALID, "lc_attention_f32: null buffer");
  auto *qf = static_cast<const float *>(q);
  auto *kf = static_cast<const float *>(kt);
  auto *vf = static_cast<const float *>(v);
  auto *of = static_cast<float *>(o);
  auto *sc = static_cast<const float *>(scale);
  cudaStream_t s = as_stream(stream);
#define LC_ATT(E)                                                                                   \
  if (epilogue == E)                                                                                \
    return comp ? launch<E, true>(qf, kf, vf, of, bh, (int)s_q, (int)s_kv, (int)d, (int)dv, sc, scale_mode, s) \
                : launch<E, false>(qf, kf, vf, of, bh, (int)s_q, (int)s_kv, (int)d, (int)dv, sc, scale_mode, s);
  LC_ATT(LC_EPI_NONE) LC_ATT(LC_EPI_GELU_ERF) LC_ATT(LC_EPI_GELU_TANH)
#undef LC_ATT
  return fail(LC_ERR_INVALID, "lc_attention_f32: bad epilogue");
}
}  // namespace

extern "C" int lc_attention_f32(int scale_mode, int epilogue, const void *scale, const void *q,
                                const void *kt, const void *v, void *o, int64_t bh, int64_t s_q,
                                int64_t s_kv, int64_t d, int64_t dv, void *stream) {
  return attention_f32_entry(false, scale_mode, epilogue, scale, q, kt, v, o, bh, s_q, s_kv, d, dv, stream);
}

extern "C" int lc_attention_f32_dot2(int scale_mode, int epilogue, const void *scale, const void *q,
                                     const void *kt, const void *v, void *o, int64_t bh, int64_t s_q,
                                     int64_t s_kv, int64_t d, int64_t dv, void *stream) {
  return attention_f32_entry(true, scale_mode, epilogue, scale, q, kt, v, o, bh, s_q, s_kv, d, dv, stream);
}

extern "C" int lc_attention_tile_f16q(const void *q, const void *kt, const void *v, void *o,
                                      int64_t bh, int64_t s_q, int64_t s_kv, int64_t d, int64_t dv,
                                      void *stream) {
  using namespace lc;
  if (bh < 0 || s_q < 0 || s_kv < 0 || d < 0 || dv < 0)
    return fail(LC_ERR_INVALID, "lc_attention_tile_f16q: negative shape");
  if (s_kv > kTileMaxKeys || bh > 65535 || s_q > 0x7fffffff || d > 0x7fffffff || dv > 0x7fffffff)
    return fail(LC_ERR_UNSUPPORTED, "lc_attention_tile_f16q: more than %d keys or too large", kTileMaxKeys);
  if (bh == 0 || s_q == 0 || dv == 0) return LC_OK;
  if (s_kv == 0) return fail(LC_ERR_INVALID, "lc_attention_tile_f16q: softmax over zero keys");
  if (!o || !v || (d > 0 && (!q || !kt))) return fail(LC_ERR_INVALID, "lc_attention_tile_f16q: null buffer");
  dim3 grid((unsigned)((s_q + kTileWarps - 1) / kTileWarps), (unsigned)bh);
  attention_tile_f16q_kernel<<<grid, 32 * kTileWarps, 0, as_stream(stream)>>>(
      static_cast<const float *>(q), static_cast<const float *>(kt), static_cast<const float *>(v),
      static_cast<float *>(o), (int)s_q, (int)s_kv, (int)d, (int)dv);
  return check_launch("lc_attention_tile_f16q");
}
