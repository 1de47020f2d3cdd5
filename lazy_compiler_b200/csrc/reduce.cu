// Whole-array FP32 sum and mean.
//
// The reference lowers r01/r02/r03 to ONE CTA of 128 threads
// (problems/r02_big_sum/meta.json grid [1,1,1]): a strided fp32 accumulate
// (ptx_backend.py:1496-1554 loop), a shfl.sync.bfly butterfly (:1668-1703
// shuffle) and a 4-slot shared tree (:1705-1744 tree); r03 divides by the
// count buffer.  At 2^24 elements that is 131,072 dependent loads per thread
// on one of 148 SMs.
//
// Here one launch covers the whole array: a grid of up to 2 CTAs x 512
// threads per SM strides over the array with 128-bit streaming loads, each
// thread keeps an error-free compensated fp32 sum (TwoSum), the block tree
// combines in f64 and writes one f64 partial per CTA, and the last CTA to
// finish (atomic ticket after a fence) adds the partials in a fixed order and
// writes the fp32 result.  The order of every addition is fixed by the grid,
// so the result is deterministic; the f64 combine makes it the correctly
// rounded fp32 value of the exact sum in all but tie cases.
#include <mutex>

#include "common.cuh"

namespace lc {
namespace {

constexpr int kThreads = 512;
constexpr int kBlocksPerSm = 2;
constexpr int kUnroll = 4;

__device__ __forceinline__ void accumulate(CompSum &acc, const float *__restrict__ x, int64_t n) {
  const int64_t nvec = n >> 2;
  const float4 *xv = reinterpret_cast<const float4 *>(x);
  const int64_t tile = (int64_t)kThreads * kUnroll;
  for (int64_t base = (int64_t)blockIdx.x * tile; base < nvec; base += (int64_t)gridDim.x * tile) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * kThreads + threadIdx.x;
      v[u] = i < nvec ? ld_stream(xv + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      acc.add(v[u].x);
      acc.add(v[u].y);
      acc.add(v[u].z);
      acc.add(v[u].w);
    }
  }
  if (blockIdx.x == 0) {
    const int64_t i = (nvec << 2) + threadIdx.x;
    if (i < n) acc.add(x[i]);
  }
}

__device__ __forceinline__ void accumulate_scalar(CompSum &acc, const float *__restrict__ x,
                                                  int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kThreads)
    acc.add(x[i]);
}

// mode 0: out = sum; mode 1: out = sum / count[0]; mode 2: partial_out = sum (f64)
template <bool VEC>
__global__ void __launch_bounds__(kThreads, kBlocksPerSm) sum_kernel(const float *__restrict__ x, int64_t n,
                                                       double *__restrict__ partials,
                                                       unsigned int *__restrict__ counter,
                                                       int mode, const float *__restrict__ count,
                                                       float *__restrict__ out,
                                                       double *__restrict__ partial_out) {
  __shared__ double scratch[32];
  __shared__ bool is_last;
  CompSum acc;
  if (VEC) accumulate(acc, x, n);
  else accumulate_scalar(acc, x, n);
  const double block_total = block_sum<double>(acc.value(), scratch);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = block_total;
    __threadfence();
    const unsigned int ticket = atomicAdd(counter, 1u);
    is_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  double t = 0.0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += kThreads) t += __ldcg(partials + i);
  const double total = block_sum<double>(t, scratch);
  if (threadIdx.x == 0) {
    if (mode == 0) out[0] = (float)total;
    else if (mode == 1) out[0] = (float)(total / (double)__ldg(count));
    else partial_out[0] = total;
    *counter = 0u;  // ready for the next launch on this workspace
  }
}

__global__ void finalize_kernel(const double *__restrict__ total, const float *__restrict__ count,
                                float *__restrict__ out) {
  const double t = *total;
  out[0] = count ? (float)(t / (double)*count) : (float)t;
}

int launch_sum(const char *name, const float *x, int64_t n, int mode, const float *count,
               float *out, double *partial_out, void *stream) {
  if (n < 0 || (!x && n > 0)) return fail(LC_ERR_INVALID, "%s: null input or negative length", name);
  if (mode < 2 && !out) return fail(LC_ERR_INVALID, "%s: null output", name);
  if (mode == 1 && !count) return fail(LC_ERR_INVALID, "%s: null count", name);
  if (mode == 2 && !partial_out) return fail(LC_ERR_INVALID, "%s: null partial", name);
  cudaStream_t s = as_stream(stream);
  ReduceWorkspace ws;
  if (int rc = reduce_workspace(s, &ws)) return rc;
  const bool vec = aligned(x, 16);
  const int64_t per_block = vec ? (int64_t)kThreads * kUnroll * 4 : (int64_t)kThreads;
  int64_t blocks = (n + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * kBlocksPerSm;
  if (blocks > cap) blocks = cap;
  if (blocks > kMaxPartials) blocks = kMaxPartials;
  if (blocks < 1) blocks = 1;
  if (vec)
    sum_kernel<true><<<(int)blocks, kThreads, 0, s>>>(x, n, ws.partials, ws.counter, mode, count,
                                                      out, partial_out);
  else
    sum_kernel<false><<<(int)blocks, kThreads, 0, s>>>(x, n, ws.partials, ws.counter, mode, count,
                                                       out, partial_out);
  return check_launch(name);
}

}  // namespace
}  // namespace lc

// ---------------------------------------------------------------- no-allocation variant
//
// lc_sum_f32 keeps its per-CTA partials in a workspace the library creates
// with cudaMalloc on the first call per (device, stream).  Some callers cannot
// let a library allocate: applications whose device memory is entirely owned
// by their own allocator (a framework's caching pool, or a service that
// reserves the GPU's memory at start-up), and launch paths that must not pay
// cudaMalloc's implicit device-wide synchronisation.  lc_sum_f32_noalloc runs
// the same kernel with its scratch in this fixed-size device array instead.
// Every device on which the library's module has been loaded holds the array
// (LC_SUM_NOALLOC_SCRATCH_BYTES) until the process exits; all calls share it,
// so calls that overlap on the GPU (different streams, or other threads) race
// on it.  The array bounds the number of CTAs (one f64 partial each), not n.
namespace {
static __device__ __align__(256) unsigned char
    g_sum_noalloc_scratch[LC_SUM_NOALLOC_MAX_BLOCKS * sizeof(double) + 256];

std::mutex g_noalloc_mutex;
unsigned char *g_noalloc_address[64] = {nullptr};

// Device address of g_sum_noalloc_scratch on the current device.  Host code
// only sees a host-side stand-in under that name, so the address is looked up
// once per device (with that device current) and cached for the life of the
// process; a device reset would invalidate it, and the library must not
// outlive one.  The lookup also loads the module on the device under lazy
// loading, so the first call per device must precede any stream capture.
int noalloc_scratch(unsigned char **out) {
  int dev = 0;
  if (int rc = lc::check_cuda(cudaGetDevice(&dev), "lc_sum_f32_noalloc: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64)
    return lc::fail(LC_ERR_UNSUPPORTED, "lc_sum_f32_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_address[dev]) {
    void *ptr = nullptr;
    if (int rc = lc::check_cuda(cudaGetSymbolAddress(&ptr, g_sum_noalloc_scratch),
                                "lc_sum_f32_noalloc: cudaGetSymbolAddress"))
      return rc;
    g_noalloc_address[dev] = static_cast<unsigned char *>(ptr);
  }
  *out = g_noalloc_address[dev];
  return LC_OK;
}
}  // namespace

extern "C" int lc_sum_f32_noalloc(const float *x, float *out, int64_t n, void *stream) {
  using namespace lc;
  if (n < 0 || (!x && n > 0) || !out)
    return fail(LC_ERR_INVALID, "lc_sum_f32_noalloc: null buffer or negative length");
  if (n > LC_SUM_NOALLOC_MAX_N)
    return fail(LC_ERR_UNSUPPORTED,
                "lc_sum_f32_noalloc: n = %lld exceeds the maximum of %lld elements; use lc_sum_f32",
                (long long)n, (long long)LC_SUM_NOALLOC_MAX_N);
  unsigned char *scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  double *partials = reinterpret_cast<double *>(scratch);
  unsigned int *counter =
      reinterpret_cast<unsigned int *>(scratch + LC_SUM_NOALLOC_MAX_BLOCKS * sizeof(double));
  cudaStream_t s = as_stream(stream);
  const bool vec = aligned(x, 16);
  const int64_t per_block = vec ? (int64_t)kThreads * kUnroll * 4 : (int64_t)kThreads;
  int64_t blocks = (n + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * kBlocksPerSm;
  if (blocks > cap) blocks = cap;
  // grid-stride and int64-indexed: a grid clamped to the array's partials covers any n
  if (blocks > LC_SUM_NOALLOC_MAX_BLOCKS) blocks = LC_SUM_NOALLOC_MAX_BLOCKS;
  if (blocks < 1) blocks = 1;
  // the CTA ticket counter must start at zero; the array keeps the last call's contents
  if (int rc = check_cuda(cudaMemsetAsync(counter, 0, sizeof(unsigned int), s),
                          "lc_sum_f32_noalloc: clear counter"))
    return rc;
  if (vec)
    sum_kernel<true><<<(int)blocks, kThreads, 0, s>>>(x, n, partials, counter, 0, nullptr, out,
                                                      nullptr);
  else
    sum_kernel<false><<<(int)blocks, kThreads, 0, s>>>(x, n, partials, counter, 0, nullptr, out,
                                                       nullptr);
  return check_launch("lc_sum_f32_noalloc");
}

extern "C" int lc_sum_f32(const float *x, float *out, int64_t n, void *stream) {
  return lc::launch_sum("lc_sum_f32", x, n, 0, nullptr, out, nullptr, stream);
}

extern "C" int lc_mean_f32(const float *x, const float *count, float *out, int64_t n,
                           void *stream) {
  return lc::launch_sum("lc_mean_f32", x, n, 1, count, out, nullptr, stream);
}

extern "C" int lc_sum_partial_f32(const float *x, int64_t n, double *partial, void *stream) {
  return lc::launch_sum("lc_sum_partial_f32", x, n, 2, nullptr, nullptr, partial, stream);
}

extern "C" int lc_sum_finalize(const double *total, const float *count, float *out,
                               void *stream) {
  if (!total || !out) return lc::fail(LC_ERR_INVALID, "lc_sum_finalize: null buffer");
  lc::finalize_kernel<<<1, 1, 0, lc::as_stream(stream)>>>(total, count, out);
  return lc::check_launch("lc_sum_finalize");
}
