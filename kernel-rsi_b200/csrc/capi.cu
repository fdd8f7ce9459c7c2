// capi.cu - library-wide entry points of the C ABI: error text, version, and the device
// watchdog word that bounded waits inside the attention kernels write when they give up.
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "watchdog.cuh"

namespace {
thread_local char g_cuda_error_text[160] = "";
}

void krsi_set_last_cuda_error(cudaError_t e) {
  snprintf(g_cuda_error_text, sizeof(g_cuda_error_text), "CUDA error %d (%s): %s", (int)e,
           cudaGetErrorName(e), cudaGetErrorString(e));
}

extern "C" const char* krsi_error_string(int status) {
  switch (status) {
    case KRSI_OK: return "ok";
    case KRSI_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, size, stride or dtype)";
    case KRSI_ERR_UNSUPPORTED: return "unsupported shape or dtype for the B200 kernels";
    case KRSI_ERR_MISALIGNED: return "pointer or stride alignment not met (16-byte TMA/vector access)";
    case KRSI_ERR_WORKSPACE: return "workspace missing or smaller than the *_workspace_size() query";
    case KRSI_ERR_CUDA: return g_cuda_error_text[0] ? g_cuda_error_text : "CUDA call failed";
    case KRSI_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait gave up (pipeline stalled)";
    default: return "unknown krsi status";
  }
}

extern "C" int krsi_abi_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" int krsi_device_status(int* status_out, int clear) {
  KRSI_CHECK_ARG(status_out);
  unsigned word = 0;
  KRSI_CUDA_TRY(cudaDeviceSynchronize());
  KRSI_CUDA_TRY(krsi::watchdog_read(&word, clear != 0));
  *status_out = word == 0 ? 0 : (int)(KRSI_ERR_DEVICE_TIMEOUT | ((word & 0xff) << 8));
  return KRSI_OK;
}
