// Pointwise math shared by the elementwise kernels and the GEMM epilogue.
//
// GELU follows the reference's lowering (ptx_backend.py:1122-1140):
//   gelu      = (0.5 x)(1 + erf(x / sqrt 2))
//   gelu_tanh = (0.5 x)(1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
// with explicitly rounded f32 products and sums (no FMA contraction) and
// CUDA's erff / tanhf for the transcendental.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "lazyb200.h"

namespace lc {

__device__ __forceinline__ float gelu_erf(float x) {
  const float gate = erff(__fmul_rn(x, 0.70710678118654752440f));
  return __fmul_rn(__fadd_rn(1.0f, gate), __fmul_rn(0.5f, x));
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float cube = __fmul_rn(x, __fmul_rn(x, x));
  const float inner =
      __fmul_rn(0.79788456080286535588f, __fadd_rn(x, __fmul_rn(0.044715f, cube)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

template <int EPI>
__device__ __forceinline__ float apply_epilogue(float v) {
  if constexpr (EPI == LC_EPI_GELU_ERF) return gelu_erf(v);
  else if constexpr (EPI == LC_EPI_GELU_TANH) return gelu_tanh(v);
  else return v;
}

template <int OUT>
struct OutType;
template <>
struct OutType<LC_F32> { using type = float; };
template <>
struct OutType<LC_F16> { using type = __half; };
template <>
struct OutType<LC_BF16> { using type = __nv_bfloat16; };

template <class T>
__device__ __forceinline__ T to_out(float v);
template <>
__device__ __forceinline__ float to_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float in_to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float in_to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float in_to_float(float v) { return v; }

}  // namespace lc
