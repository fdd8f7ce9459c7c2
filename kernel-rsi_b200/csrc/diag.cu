// diag.cu - diagnostic entry points (include/krsi_b200_diag.h): a self-test of the bounded-wait
// watchdog that the attention kernels rely on, and an evaluator of their FMA-pipe exp2.
#include "../../include/krsi_b200_diag.h"
#include "common.cuh"
#include "sm100.cuh"
#include "watchdog.cuh"

KRSI_DEFINE_WATCHDOG(diag)

namespace krsi {
namespace {

__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  const int64_t i = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const bool two = i + 1 < n;
  float y0, y1;
  sm100::exp2_poly3_x2(x[i], two ? x[i + 1] : 0.f, y0, y1);
  y[i] = y0;
  if (two) y[i + 1] = y1;
}

// The same protocol as the attention kernels' failure path, on barriers that never complete:
// a role waits with a spin limit, raises the CTA's abort flag and records its role when it gives
// up; the other roles leave their own waits through the abort flag; the TMEM owner frees its
// columns before the CTA returns.  Decisions are warp-uniform (__all_sync), as TMEM ops are
// warp-collective.
__global__ void __launch_bounds__(64) watchdog_selftest_kernel(uint32_t spin_limit, int* flags) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x / 32;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bars[0], 1);
    sm100::mbar_init(&bars[1], 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 0) sm100::tmem_alloc(&tmem_base, 32);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) {
    const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait_bounded(&bars[0], 0, abort_flag, spin_limit));
    if (!ok) {
      *abort_flag = 1;
      if (threadIdx.x == 0) {
        watchdog_fire(kWdTest);
        flags[0] = 1;
      }
    }
  } else {
    // A limit far above warp 0's, so that only warp 0's wait runs out; this warp leaves through
    // the abort flag (or, were that flag never raised, through its own limit).
    const uint32_t own_limit = spin_limit > (1u << 20) ? spin_limit : spin_limit * 64u + 4096u;
    const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait_bounded(&bars[1], 0, abort_flag, own_limit));
    if (threadIdx.x == 32) flags[1] = (!ok && *abort_flag) ? 1 : 0;
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, 32);
    sm100::tmem_relinquish();
  }
}

}  // namespace
}  // namespace krsi

using namespace krsi;

extern "C" int krsi_diag_watchdog_selftest(uint32_t spin_limit, int* flags, cudaStream_t stream) {
  KRSI_CHECK_ARG(flags && spin_limit > 0);
  KRSI_CUDA_TRY(cudaMemsetAsync(flags, 0, 2 * sizeof(int), stream));
  watchdog_selftest_kernel<<<1, 64, 0, stream>>>(spin_limit, flags);
  KRSI_LAUNCH_CHECK();
  return KRSI_OK;
}

extern "C" int krsi_diag_exp2_poly(const float* x, float* y, int64_t n, cudaStream_t stream) {
  KRSI_CHECK_ARG(n >= 0);
  if (n == 0) return KRSI_OK;
  KRSI_CHECK_ARG(x && y);
  const int64_t pairs = (n + 1) / 2;
  exp2_poly_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, stream>>>(x, y, n);
  KRSI_LAUNCH_CHECK();
  return KRSI_OK;
}
