// watchdog.cuh - bounded device-side waits.  A wait that exceeds its spin limit records
// the waiting role in a per-translation-unit device word, marks its CTA as failed and
// lets the kernel wind down (no trap, no endless loop); the host reads the word through
// krsi_device_status().
#pragma once
#include <cuda_runtime.h>

namespace krsi {

// Role codes stored in the low byte of the watchdog word.
enum WatchdogRole : unsigned {
  kWdNone = 0,
  kWdFwdLoad = 1,     // attention forward: TMA producer waiting for a free stage
  kWdFwdMma = 2,      // attention forward: MMA issuer waiting for data / P
  kWdFwdSoftmax = 3,  // attention forward: softmax waiting for S
  kWdFwdEpilogue = 4,
  kWdBwdLoad = 9,
  kWdBwdMma = 10,
  kWdBwdCompute = 11,
  kWdBwdDq = 12,
  kWdGemmLoad = 17,   // fused projection GEMM: TMA producer waiting for a free stage
  kWdGemmMma = 18,    // fused projection GEMM: MMA issuer waiting for data / a free accumulator
  kWdGemmEpilogue = 19,
  kWdTest = 0x7f      // the self-test kernel's deliberately unsatisfied wait
};

// Spin limit for one mbarrier wait.  Each try_wait blocks for a hardware-defined
// interval before returning false, so this bound is several seconds of wall time:
// far above any legitimate stall, far below a process timeout.
constexpr unsigned kSpinLimit = 1u << 22;

// Host readers of each translation unit's watchdog word (OR-ed by watchdog_read).
cudaError_t watchdog_read_attn_fwd(unsigned* word, bool clear);
cudaError_t watchdog_read_attn_bwd(unsigned* word, bool clear);
cudaError_t watchdog_read_diag(unsigned* word, bool clear);
cudaError_t watchdog_read_gemm(unsigned* word, bool clear);

inline cudaError_t watchdog_read(unsigned* word, bool clear) {
  unsigned a = 0, b = 0, c = 0, d = 0;
  cudaError_t e = watchdog_read_attn_fwd(&a, clear);
  if (e != cudaSuccess) return e;
  e = watchdog_read_attn_bwd(&b, clear);
  if (e != cudaSuccess) return e;
  e = watchdog_read_diag(&c, clear);
  if (e != cudaSuccess) return e;
  e = watchdog_read_gemm(&d, clear);
  *word = a | b | c | d;
  return e;
}

}  // namespace krsi

// Defines the device word and its host reader inside one translation unit.
#define KRSI_DEFINE_WATCHDOG(TAG)                                                    \
  namespace krsi {                                                                   \
  static __device__ unsigned g_watchdog_word;                                        \
  cudaError_t watchdog_read_##TAG(unsigned* word, bool clear) {                      \
    cudaError_t e = cudaMemcpyFromSymbol(word, g_watchdog_word, sizeof(unsigned));   \
    if (e == cudaSuccess && clear) {                                                 \
      const unsigned zero = 0;                                                       \
      e = cudaMemcpyToSymbol(g_watchdog_word, &zero, sizeof(unsigned));              \
    }                                                                                \
    return e;                                                                        \
  }                                                                                  \
  __device__ __forceinline__ void watchdog_fire(unsigned role) {                     \
    atomicCAS(&g_watchdog_word, 0u, role); /* first failure wins */                  \
  }                                                                                  \
  }
