// placeholder until the tcgen05 GEMM lands
#include "common.cuh"
extern "C" int lc_gemm(int, int, int, int, const void *, const void *, void *, int64_t, int64_t,
                       int64_t, void *) {
  return lc::fail(LC_ERR_UNSUPPORTED, "lc_gemm: not built yet");
}
extern "C" int lc_sdpa_f16(const void *, const void *, const void *, void *, int64_t, int64_t,
                           int64_t, int64_t, float, void *) {
  return lc::fail(LC_ERR_UNSUPPORTED, "lc_sdpa_f16: not built yet");
}
