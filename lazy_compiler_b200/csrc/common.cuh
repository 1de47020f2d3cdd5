// Shared helpers of liblazyb200.so: status/error reporting, device facts,
// streaming memory access and block reductions.  sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <utility>
#include <stdint.h>

#include "lazyb200.h"

namespace lc {

// Records a formatted message for lc_last_error() on this thread and returns code.
int fail(int code, const char *fmt, ...);
// Maps a pending launch error (cudaGetLastError) to LC_ERR_CUDA, else LC_OK.
int check_launch(const char *what);
// Maps a CUDA status to LC_ERR_CUDA with a message, else LC_OK.
int check_cuda(cudaError_t err, const char *what);
// Number of SMs of the current device (cached per device).
int sm_count();

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned(const void *p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

// Library-owned reduction workspace, one per (device, stream); created once
// under a mutex.  `partials` holds kMaxPartials doubles, `counter` one
// zero-initialised unsigned int that the last block of a reduction resets.
struct ReduceWorkspace {
  double *partials;
  unsigned int *counter;
};
constexpr int kMaxPartials = 4096;
int reduce_workspace(cudaStream_t stream, ReduceWorkspace *out);

// GEMM paths shared between the 16-bit (gemm.cu) and f32 (gemm_f32.cu) entry
// points.  gemm_path16/32 return 2 (tcgen05 on SM pairs), 1 (tcgen05 on one
// SM) or 0 (SIMT); gemm_tc_launch runs the tcgen05 kernel on 16-bit operands.
int gemm_path16(int b_layout, const void *a, const void *b, int64_t m, int64_t n, int64_t k);
// gemm_path16 from the operands' 16-byte alignment instead of their addresses
int gemm_path16_shape(int b_layout, bool a_aligned, bool b_aligned, int64_t m, int64_t n, int64_t k);
int gemm_path32(int b_layout, const void *a, const void *b, int64_t m, int64_t n, int64_t k);
// any_k_order: the caller lets the 2-SM kernel walk K in either direction per
// tile (a plain 16-bit product); callers whose K order carries the rounding
// order (the f32 split's small-products-first operands) keep it false.
int gemm_tc_launch(bool bf16, bool b_mn, int out, int epi, const void *a, const void *b,
                   const float *bias, void *c, int m, int n, int k, cudaStream_t s, bool pair,
                   bool any_k_order = false);
int gemm_f32(int out, int b_layout, int epi, const void *a, const void *b, const float *bias,
             void *c, int m, int n, int k, cudaStream_t s);
int gemm_f32_dot2(int b_layout, int epi, const float *a, const float *b, const float *bias, float *c,
                  int m, int n, int k, cudaStream_t s);
// lc_gemm_mixed after argument checks (gemm_mixed.cu)
int gemm_mixed(int mma_type, int a_type, int b_type, int c_type, int b_layout, int epilogue,
               int flags, const void *a, const void *b, const float *bias, void *c, int m, int n,
               int k, cudaStream_t s);

// Library-owned scratch of at least `bytes`, one per (device, stream, slot),
// grown (never shrunk) on demand with cudaMalloc.  Growing synchronises the
// device, so it must not happen inside stream capture.
int scratch_buffer(cudaStream_t stream, int slot, size_t bytes, void **out);

// Per-device error word that kernels with bounded waits write when a wait
// gives up (zero-initialised; read and cleared by lc_device_status).
int device_error_word(int **out);

// ---------------------------------------------------------------- device side

// 128-bit streaming load that bypasses L1 allocation (read-only data).
// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the previous kernel on its stream is still draining: pdl_wait blocks
// until that kernel has completed and its writes are visible (a no-op when the
// previous work was not a PDL launch), and pdl_trigger lets the next such
// kernel on the stream be scheduled as soon as resources free up.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ float4 ld_stream(const float4 *p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// 128-bit store with the evict-first (streaming) policy.
__device__ __forceinline__ void st_stream(float4 *p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_stream_u4(void *p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Error-free transformation (Knuth TwoSum): s + e == a + b exactly.
struct CompSum {
  float s = 0.f, c = 0.f;
  __device__ __forceinline__ void add(float x) {
    float t = __fadd_rn(s, x);
    float bp = __fsub_rn(t, s);
    float e = __fadd_rn(__fsub_rn(s, __fsub_rn(t, bp)), __fsub_rn(x, bp));
    s = t;
    c = __fadd_rn(c, e);
  }
  __device__ __forceinline__ double value() const { return (double)s + (double)c; }
};

// One step of the compensated dot product Dot2 (Ogita, Rump and Oishi 2005,
// "Accurate Sum and Dot Product", Algorithm 5.3): hi + lo += a * b, where the
// product's rounding residual (by FMA) and the addition's rounding error
// (TwoSum) accumulate in lo.  Every operation is explicitly rounded, in the
// order the reference's compensated accumulation uses (ptx_backend.py:571-593).
__device__ __forceinline__ void dot2_step(float &hi, float &lo, float a, float b) {
  const float p = __fmul_rn(a, b);
  const float r = __fmaf_rn(a, b, -p);
  const float t = __fadd_rn(hi, p);
  const float d = __fsub_rn(t, hi);
  const float e = __fadd_rn(__fsub_rn(hi, __fsub_rn(t, d)), __fsub_rn(p, d));
  lo = __fadd_rn(lo, __fadd_rn(e, r));
  hi = t;
}
// The value of a Dot2 state: the correction counts while hi is finite
// (ptx_backend.py:539-552).
__device__ __forceinline__ float dot2_value(float hi, float lo) {
  return __fadd_rn(hi, fabsf(hi) < INFINITY ? lo : 0.f);
}

template <class T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; every thread receives the total.  `scratch` holds >= 32 T.
// The combination order is fixed, so results are deterministic.
template <class T>
__device__ __forceinline__ T block_sum(T v, T *scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // scratch may still be read by a previous call
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  T t = lane < nwarps ? scratch[lane] : T(0);
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float *scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? scratch[lane] : -INFINITY;
  return warp_max(t);
}

}  // namespace lc
