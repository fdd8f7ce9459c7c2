// placeholder replaced by the tcgen05 forward kernel
#include "common.cuh"
#include "watchdog.cuh"
KRSI_DEFINE_WATCHDOG(attn_fwd)
extern "C" int krsi_relpos_attn_fwd(const void*, int64_t, const float*, void*, float*, float*, int64_t, int64_t,
                                    int64_t, int64_t, float, int, cudaStream_t) {
  return KRSI_ERR_UNSUPPORTED;
}
