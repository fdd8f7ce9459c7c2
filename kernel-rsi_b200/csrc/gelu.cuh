// gelu.cuh - the GEGLU element arithmetic shared by the standalone GEGLU kernels (geglu.cu) and the
// GEGLU epilogues of the fused GEMMs (linear_geglu.cu: the gate|value projection's forward, the down
// projection's input gradient), so all of them round at the same points and produce identical bits
// from identical inputs.
//
// Semantics follow library/geglu.py of kernel-rsi:
//   gelu parts (geglu.py:20-24): z = sqrt(2/pi)*(a + 0.044715 a^3);
//                                  t = tanh(z) = 1 - 2/(exp(2z)+1);  gel = 0.5 a (1+t)
//   forward  (geglu.py:27-35): out = gel.to(dtype) * b          (product rounded to dtype)
//   backward (geglu.py:38-52): db = g * gel.to(dtype)           (rounded to dtype)
//                                dgel = (g*b) rounded to dtype, then fp32
//                                da = dgel * (0.5(1+t) + 0.5 a (1-t^2) sqrt(2/pi)(1+3*0.044715 a^2))
//   with a = u[:, :F] (gate), b = u[:, F:] (value); du = [da | db].
#pragma once
#include "common.cuh"

namespace krsi {
namespace gelu {

constexpr float kSqrt2OverPi = 0.7978845608028654f;
constexpr float kGeluC = 0.044715f;
constexpr float kLog2e = 1.4426950408889634f;

struct GeluParts {
  float t, gel;
};

__device__ __forceinline__ GeluParts gelu_parts(float a) {
  const float z = kSqrt2OverPi * (a + kGeluC * a * a * a);
  // exp(2z) and the reciprocal on the SFU (the reference's tl.exp and approximate division);
  // 1 - 2/(e+1) saturates to +-1 for large |z| (e = inf or 0).
  const float e = ex2_approx(2.0f * kLog2e * z);
  const float t = fmaf(-2.0f, rcp_approx(e + 1.0f), 1.0f);
  return {t, 0.5f * a * (1.0f + t)};
}

template <int DT>
__device__ __forceinline__ float geglu_out(float a, float b) {
  using E = Elem<DT>;
  return E::round(E::round(gelu_parts(a).gel) * b);
}

// d(gate) from the gate value a, its tanh t and the rounded dgel = (g * b).to(dtype).
__device__ __forceinline__ float geglu_dgate(float a, float t, float dgel) {
  const float dz = kSqrt2OverPi * (1.0f + 3.0f * kGeluC * a * a);
  return dgel * (0.5f * (1.0f + t) + 0.5f * a * (1.0f - t * t) * dz);
}

template <int DT>
__device__ __forceinline__ void geglu_grad(float a, float b, float g, float* da, float* db) {
  using E = Elem<DT>;
  const GeluParts p = gelu_parts(a);
  *db = E::round(g * E::round(p.gel));
  *da = geglu_dgate(a, p.t, E::round(g * b));
}

}  // namespace gelu
}  // namespace krsi
