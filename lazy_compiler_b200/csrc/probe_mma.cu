// Diagnostic: throughput of back-to-back tcgen05.mma streams (no reference
// counterpart).  One CTA per SM; one thread issues `groups` groups of 8
// M128 x N128 x K16 kind::f16 MMAs into TMEM accumulators, with no waits
// between groups and one commit at the end (bounded wait).  Operands are
// zeroed shared memory / tensor memory.  Variants:
//   0  SS: A and B from shared memory, B K-major
//   1  TS: A from tensor memory, B MN-major (the attention PV form)
//   2  SS with B MN-major
//   3  variant 0 and variant 1 alternating every 2 groups
//   4  variant 0 and variant 2 alternating every 2 groups
//   5  variant 0 with one accumulator for every group
//   6  variant 1 with the accumulator alternating between two TMEM regions per group
//   7  variant 2 with the accumulator alternating per group
//   8  TS with B K-major, one accumulator
//   9  TS with B K-major, accumulator alternating per group
// Variants 0, 6, 7, 9 alternate accumulators; 1, 2, 5, 8 chain every group
// into one.  Used to measure what each MMA form and each switch costs.
#include "common.cuh"
#include "sm100.cuh"

namespace lc {
namespace {

using namespace sm100;

constexpr int kProbeSmem = 120 * 1024;  // > half the SM's shared memory: one CTA per SM

template <int VARIANT>
__global__ void __launch_bounds__(128, 1) mma_probe_kernel(int groups, int *err) {
  constexpr int variant = VARIANT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 96 * 1024 / 4; i += blockDim.x) reinterpret_cast<uint32_t *>(smem)[i] = 0;
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  {  // zero the TMEM A operand region of the TS form (columns 256..319), each warp its lane quarter
    uint32_t z[16] = {0};
    for (int c = 0; c < 64; c += 16) tmem_st16(tmem + ((uint32_t)(warp * 32) << 16) + 256 + c, z);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc_k = idesc_f16(false, false, false, 128, 128);
    constexpr uint32_t idesc_mn = idesc_f16(false, false, true, 128, 128);
    const uint32_t a = smem_u32(smem), b = smem_u32(smem + 32768), v = smem_u32(smem + 65536);
    for (int g = 0; g < groups; ++g) {
      // form: 0 SS/K, 1 TS/MN, 2 SS/MN, 3 TS/K; the accumulator is column 0 or
      // 384, alternating with 128 per group when `alt`
      constexpr bool alt = variant == 0 || variant == 6 || variant == 7 || variant == 9;
      constexpr int fixed_form = variant == 5 ? 0 : variant == 6 ? 1 : variant == 7 ? 2
                               : (variant == 8 || variant == 9) ? 3 : variant;
      constexpr bool mixed = variant == 3 || variant == 4;
      if (mixed && ((g >> 1) & 1)) {
        // second form of the alternating variants, accumulator at column 384
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if constexpr (variant == 3)
            mma_f16_tmem_a(tmem + 384, tmem + 256 + k * 8, smem_desc_sw128(v + k * 2048, 16384, 1024),
                           idesc_mn, 1);
          else
            mma_f16(tmem + 384, smem_desc_sw128(a + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
                    smem_desc_sw128(v + k * 2048, 16384, 1024), idesc_mn, 1);
        }
        continue;
      }
      constexpr int form = mixed ? 0 : fixed_form;
      constexpr uint32_t d_base = form == 0 ? 0u : 384u;
      const uint32_t d = alt && (g & 1) ? 128u : d_base;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
        if constexpr (form == 0)
          mma_f16(tmem + d, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(b + off, 16, 1024),
                  idesc_k, 1);
        else if constexpr (form == 1)
          mma_f16_tmem_a(tmem + d, tmem + 256 + k * 8, smem_desc_sw128(v + k * 2048, 16384, 1024),
                         idesc_mn, 1);
        else if constexpr (form == 2)
          mma_f16(tmem + d, smem_desc_sw128(a + off, 16, 1024),
                  smem_desc_sw128(v + k * 2048, 16384, 1024), idesc_mn, 1);
        else
          mma_f16_tmem_a(tmem + d, tmem + 256 + k * 8, smem_desc_sw128(b + off, 16, 1024), idesc_k, 1);
      }
    }
    mma_commit(&done);
    if (!mbar_wait(&done, 0, &abort_flag)) atomicCAS(err, 0, kErrTimeoutMma);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace
}  // namespace lc

extern "C" int lc_probe_mma(int variant, int groups, void *stream) {
  using namespace lc;
  if (variant < 0 || variant > 9 || groups < 1 || groups > (1 << 16))
    return fail(LC_ERR_INVALID, "lc_probe_mma: bad variant or group count");
  int *err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  void (*kernels[10])(int, int *) = {mma_probe_kernel<0>, mma_probe_kernel<1>, mma_probe_kernel<2>,
                                     mma_probe_kernel<3>, mma_probe_kernel<4>, mma_probe_kernel<5>,
                                     mma_probe_kernel<6>, mma_probe_kernel<7>, mma_probe_kernel<8>,
                                     mma_probe_kernel<9>};
  auto kernel = kernels[variant];
  if (int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kProbeSmem),
                          "probe smem attribute"))
    return rc;
  kernel<<<sm_count(), 128, kProbeSmem, as_stream(stream)>>>(groups, err);
  return check_launch("lc_probe_mma");
}
