// Fused scaled-dot-product attention (tcgen05) — entry point placeholder.
#include "common.cuh"
extern "C" int lc_sdpa_f16(const void *, const void *, const void *, void *, int64_t, int64_t,
                           int64_t, int64_t, float, void *) {
  return lc::fail(LC_ERR_UNSUPPORTED, "lc_sdpa_f16: not available in this build");
}
