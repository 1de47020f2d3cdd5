// Row operations on X[rows, cols] f32: row sum, RMSNorm, softmax, L2 norm,
// and row dot products sum_c Y[r,c] * f(X[r,c]) with f the identity or GELU.
//
// The reference lowers r04/f01/f02/f03 to one 128-thread CTA per row with a
// strided first pass (sum, sum of squares or the coupled online-softmax
// (max, sum) state, ptx_backend.py:1443-1447, 1496-1554), a warp butterfly
// and shared tree (:1668-1744), and — for the fused ops — a second strided
// pass that re-reads the row from global memory to write the output.
//
// Here one CTA owns one row at a time and holds the whole row in registers
// (V float4 per thread, V in {1,2,4,8}, so rows of up to 32,768 columns), so
// X is read from HBM exactly once and the output written once: 128-bit
// streaming loads, block reductions in registers/shared memory, 128-bit
// evict-first stores.  Row sums use an error-free compensated fp32 sum per
// thread and an f64 block combine; the norms accumulate squares in fp32 per
// thread and combine in f64; softmax takes the block max, keeps exp(x - max)
// in registers and scales by the reciprocal of the block sum.  The epilogue
// arithmetic follows the IR's own order (f01: w * (x * 1/sqrt(eps + ss/count)),
// f03: x * 1/sqrt(ss), f02: 1/sum * exp(x - max)) with correctly rounded
// sqrt and reciprocal (ptx_backend.py:1047-1050 div.rn / sqrt.rn).
// Row dot products (phase9_gelu_row_dot: acc += g * gelu(x)) round each
// product once and sum like the row sum.
// Rows that are not 16-byte aligned, not a multiple of 4 wide or wider than
// 32,768 take a scalar kernel that streams the row from global (L2) per pass.
#include "common.cuh"
#include "epilogue.cuh"

namespace lc {
namespace {

enum RowOp { kRowSum = 0, kRmsNorm = 1, kSoftmax = 2, kL2 = 3, kRowDot = 4, kRowDotGeluErf = 5,
             kRowDotGeluTanh = 6 };

constexpr bool is_dot(int op) { return op >= kRowDot; }

// y * f(x) of the row dot products, rounded once
template <int OP>
__device__ __forceinline__ float dot_factor(float x) {
  if constexpr (OP == kRowDotGeluErf) return gelu_erf(x);
  else if constexpr (OP == kRowDotGeluTanh) return gelu_tanh(x);
  else return x;
}
// Adds the term y * f(x) to a compensated row sum: the rounded product by
// TwoSum and its rounding residual (by FMA) into the correction, as the
// reference's Dot2 accumulation of this product keeps it (ptx_backend.py:571-593).
template <int OP>
__device__ __forceinline__ void add_dot_term(CompSum &acc, float x, float y) {
  const float fx = dot_factor<OP>(x);
  const float p = __fmul_rn(y, fx);
  acc.add(p);
  acc.c = __fadd_rn(acc.c, __fmaf_rn(y, fx, -p));
}

struct RowArgs {
  const float *x;
  const float *w;  // RMSNorm weight, or Y of the row dot products
  const float *count;
  const float *eps;
  float *out;
  int64_t rows;
  int64_t cols;
};

__device__ __forceinline__ float norm_scale(int op, double ss, const float *count,
                                            const float *eps) {
  const float acc = (float)ss;
  if (op == kL2) return __frcp_rn(__fsqrt_rn(acc));
  const float inv_count = __frcp_rn(__ldg(count));
  const float mean = __fmul_rn(acc, inv_count);
  return __frcp_rn(__fsqrt_rn(__fadd_rn(__ldg(eps), mean)));
}

template <int OP, int V>
__global__ void __launch_bounds__(1024) row_vec_kernel(RowArgs args) {
  __shared__ double dscratch[32];
  __shared__ float fscratch[32];
  pdl_wait();     // the rows may be the previous kernel's output
  pdl_trigger();
  const int64_t c4 = args.cols >> 2;
  const int T = blockDim.x;
  for (int64_t row = blockIdx.x; row < args.rows; row += gridDim.x) {
    const float4 *xr = reinterpret_cast<const float4 *>(args.x + row * args.cols);
    float4 v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int64_t idx = threadIdx.x + (int64_t)j * T;
      if (idx < c4) v[j] = ld_stream(xr + idx);
      else v[j] = OP == kSoftmax ? make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if constexpr (OP == kRowSum) {
      CompSum acc;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        acc.add(v[j].x);
        acc.add(v[j].y);
        acc.add(v[j].z);
        acc.add(v[j].w);
      }
      const double total = block_sum<double>(acc.value(), dscratch);
      if (threadIdx.x == 0) args.out[row] = (float)total;
    } else if constexpr (is_dot(OP)) {
      const float4 *yr = reinterpret_cast<const float4 *>(args.w + row * args.cols);
      CompSum acc;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int64_t idx = threadIdx.x + (int64_t)j * T;
        if (idx < c4) {
          const float4 y = ld_stream(yr + idx);
          add_dot_term<OP>(acc, v[j].x, y.x);
          add_dot_term<OP>(acc, v[j].y, y.y);
          add_dot_term<OP>(acc, v[j].z, y.z);
          add_dot_term<OP>(acc, v[j].w, y.w);
        }
      }
      const double total = block_sum<double>(acc.value(), dscratch);
      if (threadIdx.x == 0) args.out[row] = (float)total;
    } else if constexpr (OP == kSoftmax) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < V; ++j) m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
      m = block_max(m, fscratch);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int64_t idx = threadIdx.x + (int64_t)j * T;
        if (idx < c4) {
          v[j].x = expf(__fsub_rn(v[j].x, m));
          v[j].y = expf(__fsub_rn(v[j].y, m));
          v[j].z = expf(__fsub_rn(v[j].z, m));
          v[j].w = expf(__fsub_rn(v[j].w, m));
          s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
      }
      const float r = __frcp_rn(block_sum<float>(s, fscratch));
      float4 *orow = reinterpret_cast<float4 *>(args.out + row * args.cols);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int64_t idx = threadIdx.x + (int64_t)j * T;
        if (idx < c4)
          st_stream(orow + idx, make_float4(__fmul_rn(r, v[j].x), __fmul_rn(r, v[j].y),
                                            __fmul_rn(r, v[j].z), __fmul_rn(r, v[j].w)));
      }
    } else {  // RMSNorm and L2: sum of squares, then scale
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        ss = fmaf(v[j].x, v[j].x, ss);
        ss = fmaf(v[j].y, v[j].y, ss);
        ss = fmaf(v[j].z, v[j].z, ss);
        ss = fmaf(v[j].w, v[j].w, ss);
      }
      const double total = block_sum<double>((double)ss, dscratch);
      const float scale = norm_scale(OP, total, args.count, args.eps);
      float4 *orow = reinterpret_cast<float4 *>(args.out + row * args.cols);
      const float4 *wv = reinterpret_cast<const float4 *>(args.w);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int64_t idx = threadIdx.x + (int64_t)j * T;
        if (idx < c4) {
          float4 y = make_float4(__fmul_rn(v[j].x, scale), __fmul_rn(v[j].y, scale),
                                 __fmul_rn(v[j].z, scale), __fmul_rn(v[j].w, scale));
          if constexpr (OP == kRmsNorm) {
            const float4 g = __ldg(wv + idx);
            y = make_float4(__fmul_rn(g.x, y.x), __fmul_rn(g.y, y.y), __fmul_rn(g.z, y.z),
                            __fmul_rn(g.w, y.w));
          }
          st_stream(orow + idx, y);
        }
      }
    }
  }
}

// Scalar fallback: any width and alignment; passes re-read the row from global.
template <int OP>
__global__ void __launch_bounds__(256) row_scalar_kernel(RowArgs args) {
  pdl_wait();
  pdl_trigger();
  __shared__ double dscratch[32];
  __shared__ float fscratch[32];
  for (int64_t row = blockIdx.x; row < args.rows; row += gridDim.x) {
    const float *xr = args.x + row * args.cols;
    float *orow = args.out + row * args.cols;
    if constexpr (OP == kRowSum) {
      CompSum acc;
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x) acc.add(xr[c]);
      const double total = block_sum<double>(acc.value(), dscratch);
      if (threadIdx.x == 0) args.out[row] = (float)total;
    } else if constexpr (is_dot(OP)) {
      const float *yr = args.w + row * args.cols;
      CompSum acc;
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x) add_dot_term<OP>(acc, xr[c], yr[c]);
      const double total = block_sum<double>(acc.value(), dscratch);
      if (threadIdx.x == 0) args.out[row] = (float)total;
    } else if constexpr (OP == kSoftmax) {
      float m = -INFINITY;
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x) m = fmaxf(m, xr[c]);
      m = block_max(m, fscratch);
      float s = 0.f;
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x) s += expf(__fsub_rn(xr[c], m));
      const float r = __frcp_rn(block_sum<float>(s, fscratch));
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x)
        orow[c] = __fmul_rn(r, expf(__fsub_rn(xr[c], m)));
    } else {
      float ss = 0.f;
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x) ss = fmaf(xr[c], xr[c], ss);
      const double total = block_sum<double>((double)ss, dscratch);
      const float scale = norm_scale(OP, total, args.count, args.eps);
      for (int64_t c = threadIdx.x; c < args.cols; c += blockDim.x) {
        float y = __fmul_rn(xr[c], scale);
        if constexpr (OP == kRmsNorm) y = __fmul_rn(__ldg(args.w + c), y);
        orow[c] = y;
      }
    }
  }
}

template <int OP>
int launch_rows(const char *name, const RowArgs &a, void *stream) {
  if (!a.x || !a.out) return fail(LC_ERR_INVALID, "%s: null buffer", name);
  if (OP == kRmsNorm && (!a.w || !a.count || !a.eps))
    return fail(LC_ERR_INVALID, "%s: null weight, count or eps", name);
  if (is_dot(OP) && !a.w) return fail(LC_ERR_INVALID, "%s: null y", name);
  if (a.rows < 0 || a.cols < 0) return fail(LC_ERR_INVALID, "%s: negative shape", name);
  if (a.rows == 0) return LC_OK;
  if (a.cols == 0) {
    if (OP == kRowSum || is_dot(OP)) return check_cuda(cudaMemsetAsync(a.out, 0, a.rows * sizeof(float),
                                                         as_stream(stream)), name);
    return LC_OK;
  }
  cudaStream_t s = as_stream(stream);
  const int64_t grid = a.rows < 0x7fffffff ? a.rows : 0x7fffffff;
  const int64_t c4 = a.cols >> 2;
  const bool vec = (a.cols & 3) == 0 && aligned(a.x, 16) && aligned(a.out, 16) &&
                   ((OP != kRmsNorm && !is_dot(OP)) || aligned(a.w, 16)) && c4 <= 8 * 1024;
  if (!vec) {
    if (cudaError_t e = launch_pdl(row_scalar_kernel<OP>, dim3((unsigned)grid), dim3(256), 0, s, a))
      return check_cuda(e, name);
    return check_launch(name);
  }
  // the most float4 per thread (up to 8) that leaves at least 128 threads per
  // row: 4096 columns take 128-thread CTAs, 16 resident per SM (3-4% faster
  // than 256 threads at 4096-16384 rows, one wave for 2048-row shards)
  int v = 8;
  while (v > 1 && (c4 + v - 1) / v < 128) v >>= 1;
  int threads = (int)((c4 + v - 1) / v);
  threads = (threads + 31) & ~31;
  if (threads > 1024) threads = 1024;
  auto kernel = v == 1 ? row_vec_kernel<OP, 1> : v == 2 ? row_vec_kernel<OP, 2>
               : v == 4 ? row_vec_kernel<OP, 4> : row_vec_kernel<OP, 8>;
  if (cudaError_t e = launch_pdl(kernel, dim3((unsigned)grid), dim3(threads), 0, s, a)) return check_cuda(e, name);
  return check_launch(name);
}

}  // namespace
}  // namespace lc

extern "C" int lc_rowsum_f32(const float *x, float *out, int64_t rows, int64_t cols,
                             void *stream) {
  lc::RowArgs a{x, nullptr, nullptr, nullptr, out, rows, cols};
  return lc::launch_rows<lc::kRowSum>("lc_rowsum_f32", a, stream);
}

extern "C" int lc_rmsnorm_f32(const float *count, const float *eps, const float *x,
                              const float *w, float *out, int64_t rows, int64_t cols,
                              void *stream) {
  lc::RowArgs a{x, w, count, eps, out, rows, cols};
  return lc::launch_rows<lc::kRmsNorm>("lc_rmsnorm_f32", a, stream);
}

extern "C" int lc_softmax_f32(const float *x, float *out, int64_t rows, int64_t cols,
                              void *stream) {
  lc::RowArgs a{x, nullptr, nullptr, nullptr, out, rows, cols};
  return lc::launch_rows<lc::kSoftmax>("lc_softmax_f32", a, stream);
}

extern "C" int lc_l2norm_f32(const float *x, float *out, int64_t rows, int64_t cols,
                             void *stream) {
  lc::RowArgs a{x, nullptr, nullptr, nullptr, out, rows, cols};
  return lc::launch_rows<lc::kL2>("lc_l2norm_f32", a, stream);
}

extern "C" int lc_rowdot_f32(int activation, const float *x, const float *y, float *out,
                             int64_t rows, int64_t cols, void *stream) {
  lc::RowArgs a{x, y, nullptr, nullptr, out, rows, cols};
  if (activation == LC_EPI_NONE) return lc::launch_rows<lc::kRowDot>("lc_rowdot_f32", a, stream);
  if (activation == LC_EPI_GELU_ERF)
    return lc::launch_rows<lc::kRowDotGeluErf>("lc_rowdot_f32", a, stream);
  if (activation == LC_EPI_GELU_TANH)
    return lc::launch_rows<lc::kRowDotGeluTanh>("lc_rowdot_f32", a, stream);
  return lc::fail(LC_ERR_INVALID, "lc_rowdot_f32: unknown activation %d", activation);
}
