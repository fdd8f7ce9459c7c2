// common.cuh - shared host/device helpers for the krsi_b200 kernels: status codes,
// element conversion with explicit rounding points, vectorised IO and reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <utility>

#include "../../include/krsi_b200.h"

#define KRSI_CHECK_ARG(cond)                    \
  do {                                          \
    if (!(cond)) return KRSI_ERR_INVALID_ARGUMENT; \
  } while (0)

#define KRSI_CUDA_TRY(expr)                     \
  do {                                          \
    cudaError_t e_ = (expr);                    \
    if (e_ != cudaSuccess) {                    \
      krsi_set_last_cuda_error(e_);             \
      return KRSI_ERR_CUDA;                     \
    }                                           \
  } while (0)

// Records the last CUDA error seen by an entry point (text retrievable through
// krsi_error_string(KRSI_ERR_CUDA)).
void krsi_set_last_cuda_error(cudaError_t e);

// Launch check: a failed launch is reported as KRSI_ERR_CUDA.
#define KRSI_LAUNCH_CHECK() KRSI_CUDA_TRY(cudaGetLastError())

namespace krsi {

constexpr int kNumSMsB200 = 148;

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of this library is launched with programmatic stream serialisation, so the next
// kernel in the stream is launched (and its CTAs placed on SMs as ours finish) while ours still
// runs, instead of after a launch gap.  The rule that keeps this safe: every kernel calls
// pdl_wait() before its first global-memory access, in every thread, unconditionally: it returns
// once the preceding kernel in the stream has completed and its writes are visible (at once if that
// kernel was launched normally and has finished), so a chain of such kernels stays in stream order.
// pdl_launch_dependents() right after it lets the next kernel launch early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_launch_dependents();
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int device_sm_count() {
  int dev = 0, sms = kNumSMsB200;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : kNumSMsB200;
}

// ---------------------------------------------------------------- element types
// Tag types so that kernels are templated on storage type and know their rounding.
template <int DT> struct Elem;
template <> struct Elem<KRSI_F32> {
  using T = float;
  static __device__ __forceinline__ float load(T v) { return v; }
  static __device__ __forceinline__ T store(float v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }  // no-op rounding
};
template <> struct Elem<KRSI_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T store(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct Elem<KRSI_F16> {
  using T = __half;
  static __device__ __forceinline__ float load(T v) { return __half2float(v); }
  static __device__ __forceinline__ T store(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};

// Type promotion of two storage types (as torch/Triton promote a product of two tensors).
// f32 wins over everything; bf16 and f16 mixed promote to f32.
template <int A, int B> struct Promote { static constexpr int value = KRSI_F32; };
template <int A> struct Promote<A, A> { static constexpr int value = A; };

// ---------------------------------------------------------------- 16-byte vectors
// A 16-byte aligned packet of `sizeof(uint4)/sizeof(T)` elements, loaded/stored as one
// 128-bit transaction.
template <typename T>
struct alignas(16) Vec16 {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T>
__device__ __forceinline__ Vec16<T> ldg16(const T* p) {
  Vec16<T> r;
  *reinterpret_cast<uint4*>(&r) = __ldg(reinterpret_cast<const uint4*>(p));
  return r;
}
// Streaming load (data read once): do not keep it in L1.
template <typename T>
__device__ __forceinline__ Vec16<T> ldg16_stream(const T* p) {
  Vec16<T> r;
  uint4 u;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(p));
  *reinterpret_cast<uint4*>(&r) = u;
  return r;
}
template <typename T>
__device__ __forceinline__ void stg16(T* p, const Vec16<T>& r) {
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(&r);
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x == NT threads (multiple of 32); `red` holds NT/32 floats.
// Every thread gets the total; the summation order is fixed (deterministic).
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if constexpr (NT == 32) {
    return v;
  } else {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();  // `red` may still be read by a previous call
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) t += red[i];
    return t;
  }
}

// Fast exp2 on the SFU (ex2.approx, flush-to-zero), the operation Triton's tl.exp2 lowers to.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Reciprocal on the SFU.
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace krsi
