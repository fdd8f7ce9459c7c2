/*
 * krsi_b200_diag.h - diagnostic entry points of libkrsi_b200.so.
 *
 * These are not part of the reference's interface (kernel-rsi has no native code and no device
 * watchdog); they exist so that tests can check two pieces of the kernels directly on a GPU:
 *   - the bounded-wait watchdog (every mbarrier wait in the attention kernels gives up after a
 *     spin limit, records its role in a device word and lets the kernel return), and
 *   - the FMA-pipe exp2 the attention forward uses for a share of its exponentials.
 * Same conventions as krsi_b200.h: device pointers, asynchronous on `stream`, status return.
 */
#ifndef KRSI_B200_DIAG_H
#define KRSI_B200_DIAG_H

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Launches one CTA whose warp 0 holds 32 TMEM columns and waits, with `spin_limit` polls, on an
 * mbarrier that nothing completes, while warp 1 waits on a second such barrier and only watches
 * the CTA's abort flag.  When warp 0's wait gives up it raises the abort flag, records the
 * self-test role (0x7f) in the device watchdog word read by krsi_device_status(), frees its TMEM
 * and returns; warp 1 sees the flag and returns too.  flags[0] = 1 if warp 0's wait gave up,
 * flags[1] = 1 if warp 1 left through the abort flag (device int[2]).
 * No counterpart in the reference. */
int krsi_diag_watchdog_selftest(uint32_t spin_limit, int* flags, cudaStream_t stream);

/* y[i] = 2^x[i] computed by the attention kernels' FMA-pipe exp2 (Cody-Waite reduction and a
 * degree-3 polynomial; valid for x < 128, inputs below -125 give about 2^-125).
 * x, y: device float[n].  No counterpart in the reference. */
int krsi_diag_exp2_poly(const float* x, float* y, int64_t n, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KRSI_B200_DIAG_H */
