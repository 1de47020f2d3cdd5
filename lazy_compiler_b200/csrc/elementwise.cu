// Pointwise kernels: add, scale-shift, relu*mul and GELU (erf / tanh).
//
// Replaces the reference's pointwise lowering (ptx_backend.py:1409-1427 Load /
// Write, :1574-1642 tile, :894-1177 operation): one Tile cell per thread with
// per-element scalar ld.global and a v2/v4 store, grid = ceil(cells/256).
// Here every pointwise op is one HBM pass with 128-bit streaming loads
// (ld.global.nc.L1::no_allocate) and evict-first 128-bit stores, four vectors
// in flight per thread, one 4096-element tile per 256-thread CTA.  The arithmetic uses the
// reference's explicit-rounding form (mul.rn / add.rn, no FMA contraction,
// ptx_backend.py:777-781) so add, scale-shift and relu*mul are bit-identical
// to numpy float32.  GELU follows ptx_backend.py:1122-1140:
// gelu = (0.5x)(1 + erf(x/sqrt2)), gelu_tanh = (0.5x)(1 + tanh(sqrt(2/pi)(x + 0.044715 x^3)))
// with CUDA's erff / tanhf; f16/bf16 storage computes in f32 and rounds once.
#include "common.cuh"
#include "epilogue.cuh"

namespace lc {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

struct AddOp {
  static constexpr int kInputs = 2;
  __device__ void load() {}
  __device__ float operator()(float a, float b) const { return __fadd_rn(a, b); }
};

struct AxpbOp {  // b + a * x, with a and b read from device scalars
  static constexpr int kInputs = 1;
  const float *pa, *pb;
  float a, b;
  __device__ void load() {
    a = __ldg(pa);
    b = __ldg(pb);
  }
  __device__ float operator()(float x, float) const { return __fadd_rn(b, __fmul_rn(a, x)); }
};

struct ReluMulOp {  // y * relu(x); argument order (x, y)
  static constexpr int kInputs = 2;
  __device__ void load() {}
  __device__ float operator()(float x, float y) const { return __fmul_rn(y, fmaxf(x, 0.0f)); }
};


template <int TANH>
struct GeluFixedOp {
  static constexpr int kInputs = 1;
  __device__ void load() {}
  __device__ float operator()(float x, float) const { return TANH ? gelu_tanh(x) : gelu_erf(x); }
};

template <class Op>
__device__ __forceinline__ float4 apply4(const float4 &a, const float4 &b, const Op &op) {
  return make_float4(op(a.x, b.x), op(a.y, b.y), op(a.z, b.z), op(a.w, b.w));
}

// f32, 16-byte aligned x0/x1/out.  The n % 4 tail is done by CTA 0.
template <class Op>
__global__ void __launch_bounds__(kThreads) ew_f32_vec(const float *__restrict__ x0,
                                                       const float *__restrict__ x1,
                                                       float *__restrict__ out, int64_t n, Op op) {
  op.load();
  const int64_t nvec = n >> 2;
  const float4 *a = reinterpret_cast<const float4 *>(x0);
  const float4 *b = reinterpret_cast<const float4 *>(x1);
  float4 *o = reinterpret_cast<float4 *>(out);
  const int64_t tile = (int64_t)kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * tile; base < nvec; base += (int64_t)gridDim.x * tile) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kThreads + threadIdx.x;
      if (i < nvec) {
        va[u] = ld_stream(a + i);
        if constexpr (Op::kInputs == 2) vb[u] = ld_stream(b + i);
        else vb[u] = va[u];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kThreads + threadIdx.x;
      if (i < nvec) st_stream(o + i, apply4(va[u], vb[u], op));
    }
  }
  if (blockIdx.x == 0) {
    const int64_t i = (nvec << 2) + threadIdx.x;
    if (i < n) out[i] = op(x0[i], Op::kInputs == 2 ? x1[i] : 0.0f);
  }
}

// Any alignment: one element per thread per step.
template <class Op>
__global__ void __launch_bounds__(kThreads) ew_f32_scalar(const float *__restrict__ x0,
                                                          const float *__restrict__ x1,
                                                          float *__restrict__ out, int64_t n,
                                                          Op op) {
  op.load();
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    out[i] = op(x0[i], Op::kInputs == 2 ? x1[i] : 0.0f);
}

// GELU on 16-bit storage: eight elements per 16-byte vector.
template <class T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <class T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <class T, int TANH>
__global__ void __launch_bounds__(kThreads) gelu16_vec(const T *__restrict__ x,
                                                       T *__restrict__ out, int64_t n) {
  GeluFixedOp<TANH> op;
  const int64_t nvec = n >> 3;
  const uint4 *xv = reinterpret_cast<const uint4 *>(x);
  uint4 *ov = reinterpret_cast<uint4 *>(out);
  const int64_t tile = (int64_t)kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * tile; base < nvec; base += (int64_t)gridDim.x * tile) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kThreads + threadIdx.x;
      if (i < nvec) v[u] = ld_stream_u4(xv + i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kThreads + threadIdx.x;
      if (i < nvec) {
        T *e = reinterpret_cast<T *>(&v[u]);
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = from_f<T>(op(to_f<T>(e[j]), 0.0f));
        st_stream_u4(ov + i, v[u]);
      }
    }
  }
  if (blockIdx.x == 0) {
    const int64_t i = (nvec << 3) + threadIdx.x;
    if (i < n) out[i] = from_f<T>(op(to_f<T>(x[i]), 0.0f));
  }
}

template <class T, int TANH>
__global__ void __launch_bounds__(kThreads) gelu16_scalar(const T *__restrict__ x,
                                                          T *__restrict__ out, int64_t n) {
  GeluFixedOp<TANH> op;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    out[i] = from_f<T>(op(to_f<T>(x[i]), 0.0f));
}

// One tile of work per CTA (no persistent cap): measured on B200, a grid that
// covers the array outright keeps more loads in flight than a grid-stride loop
// over 8 CTAs per SM (6.8-7.0 vs 5.4-6.5 TB/s on 2^28 elements).  The loop in
// the kernels only strides when n exceeds what one launch grid can cover.
int grid_for(int64_t work_items, int64_t per_block) {
  constexpr int64_t kMaxGrid = 0x7fffffff;
  int64_t blocks = (work_items + per_block - 1) / per_block;
  if (blocks < 1) blocks = 1;
  return (int)(blocks < kMaxGrid ? blocks : kMaxGrid);
}

template <class Op>
int launch_f32(const char *name, const float *x0, const float *x1, float *out, int64_t n,
               void *stream, Op op) {
  if (n < 0) return fail(LC_ERR_INVALID, "%s: negative length %lld", name, (long long)n);
  if (n == 0) return LC_OK;  // nothing to touch; empty buffers may be null
  if (!x0 || !out || (Op::kInputs == 2 && !x1))
    return fail(LC_ERR_INVALID, "%s: null buffer", name);
  cudaStream_t s = as_stream(stream);
  const bool vec = aligned(x0, 16) && aligned(out, 16) && (Op::kInputs == 1 || aligned(x1, 16));
  if (vec) {
    const int grid = grid_for(n >> 2, (int64_t)kThreads * kUnroll);
    ew_f32_vec<Op><<<grid, kThreads, 0, s>>>(x0, x1, out, n, op);
  } else {
    const int grid = grid_for(n, kThreads);
    ew_f32_scalar<Op><<<grid, kThreads, 0, s>>>(x0, x1, out, n, op);
  }
  return check_launch(name);
}

template <class T>
int launch_gelu16(int tanh_form, const void *x, void *out, int64_t n, cudaStream_t s) {
  const T *xi = static_cast<const T *>(x);
  T *o = static_cast<T *>(out);
  if (aligned(x, 16) && aligned(out, 16)) {
    const int grid = grid_for(n >> 3, (int64_t)kThreads * kUnroll);
    if (tanh_form) gelu16_vec<T, 1><<<grid, kThreads, 0, s>>>(xi, o, n);
    else gelu16_vec<T, 0><<<grid, kThreads, 0, s>>>(xi, o, n);
  } else {
    const int grid = grid_for(n, kThreads);
    if (tanh_form) gelu16_scalar<T, 1><<<grid, kThreads, 0, s>>>(xi, o, n);
    else gelu16_scalar<T, 0><<<grid, kThreads, 0, s>>>(xi, o, n);
  }
  return check_launch("lc_gelu");
}

}  // namespace
}  // namespace lc

extern "C" int lc_add_f32(const float *x0, const float *x1, float *out, int64_t n,
                          void *stream) {
  return lc::launch_f32("lc_add_f32", x0, x1, out, n, stream, lc::AddOp{});
}

extern "C" int lc_axpb_f32(const float *a, const float *b, const float *x, float *out,
                           int64_t n, void *stream) {
  if (n > 0 && (!a || !b)) return lc::fail(LC_ERR_INVALID, "lc_axpb_f32: null scalar");
  lc::AxpbOp op{a, b, 0.0f, 0.0f};
  return lc::launch_f32("lc_axpb_f32", x, nullptr, out, n, stream, op);
}

extern "C" int lc_relumul_f32(const float *x, const float *y, float *out, int64_t n,
                              void *stream) {
  return lc::launch_f32("lc_relumul_f32", x, y, out, n, stream, lc::ReluMulOp{});
}

extern "C" int lc_gelu(int dtype, int approximate, const void *x, void *out, int64_t n,
                       void *stream) {
  if (approximate != 0 && approximate != 1)
    return lc::fail(LC_ERR_INVALID, "lc_gelu: approximate must be 0 (erf) or 1 (tanh)");
  if (n < 0) return lc::fail(LC_ERR_INVALID, "lc_gelu: negative length");
  if (n == 0) return LC_OK;
  if (!x || !out) return lc::fail(LC_ERR_INVALID, "lc_gelu: null buffer");
  switch (dtype) {
    case LC_F32: {
      if (approximate)
        return lc::launch_f32("lc_gelu", static_cast<const float *>(x), nullptr,
                              static_cast<float *>(out), n, stream, lc::GeluFixedOp<1>{});
      return lc::launch_f32("lc_gelu", static_cast<const float *>(x), nullptr,
                            static_cast<float *>(out), n, stream, lc::GeluFixedOp<0>{});
    }
    case LC_F16:
      return lc::launch_gelu16<__half>(approximate, x, out, n, lc::as_stream(stream));
    case LC_BF16:
      return lc::launch_gelu16<__nv_bfloat16>(approximate, x, out, n, lc::as_stream(stream));
    default:
      return lc::fail(LC_ERR_INVALID, "lc_gelu: unknown dtype %d", dtype);
  }
}
