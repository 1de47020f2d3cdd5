// Failure-detection self-test: a bounded mbarrier wait that is made to run out.
//
// The kernel initialises an mbarrier that expects one arrival and waits on it
// through the same bounded-wait routine the GEMM and attention kernels use,
// but nothing ever arrives.  The wait gives up after `limit_ns`, writes the
// device error word and returns, so the host sees LC_ERR_TIMEOUT from
// lc_device_status and the CUDA context stays usable.  No trap, no fault.
#include "common.cuh"
#include "sm100.cuh"

namespace {

__global__ void bounded_wait_selftest_kernel(int *err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    lc::sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    lc::sm100::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!lc::sm100::mbar_wait_limit(&bar, 0, &abort_flag, limit_ns))
      atomicCAS(err, 0, lc::sm100::kErrTimeoutSelftest);
  }
}

}  // namespace

extern "C" int lc_selftest_bounded_wait(int64_t limit_ns, void *stream) {
  if (limit_ns <= 0 || limit_ns > 2000000000ll)
    return lc::fail(LC_ERR_INVALID, "lc_selftest_bounded_wait: limit must be in (0, 2 s]");
  int *err = nullptr;
  if (int rc = lc::device_error_word(&err)) return rc;
  bounded_wait_selftest_kernel<<<1, 32, 0, lc::as_stream(stream)>>>(err, (uint64_t)limit_ns);
  return lc::check_launch("lc_selftest_bounded_wait");
}
