// placeholder replaced by the tcgen05 backward kernel
#include "common.cuh"
#include "watchdog.cuh"
KRSI_DEFINE_WATCHDOG(attn_bwd)
extern "C" int krsi_relpos_attn_bwd_workspace_size(int64_t, int64_t, int64_t, int64_t, size_t* b) {
  *b = 0;
  return KRSI_ERR_UNSUPPORTED;
}
extern "C" int krsi_relpos_attn_bwd(const void*, const void*, int64_t, const float*, const float*, const float*,
                                    void*, int64_t, float*, void*, size_t, int64_t, int64_t, int64_t, int64_t, float,
                                    int, cudaStream_t) {
  return KRSI_ERR_UNSUPPORTED;
}
