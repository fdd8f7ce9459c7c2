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
#include "sm100.cuh"

namespace krsi {
namespace gelu {

constexpr float kSqrt2OverPi = 0.7978845608028654f;
constexpr float kGeluC = 0.044715f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kExp2Scale = 2.0f * kLog2e * kSqrt2OverPi;   // exp(2z) = 2^(kExp2Scale * (a + c a^3))
constexpr float kDz3 = 3.0f * kGeluC * kSqrt2OverPi;        // dz/da = sqrt(2/pi) + kDz3 a^2

// Every operation below is an explicit IEEE round-to-nearest one (no contraction left to the
// compiler), so the paired forms, which issue the same operations two lanes at a time on the FMA
// pipe's f32x2 instructions, give the same bits as the scalar forms.

struct GeluParts {
  float t, gel;
};

// t = tanh(z) = 1 - 2/(exp(2z)+1) with exp(2z) on the SFU (the reference's tl.exp) and the reciprocal
// on the SFU (its approximate division); it saturates to +-1 for large |z| (exp = inf or 0).
// gel = 0.5 a (1 + t).
__device__ __forceinline__ GeluParts gelu_parts(float a) {
  const float a2 = __fmul_rn(a, a);
  const float inner = __fmaf_rn(__fmul_rn(kGeluC, a2), a, a);   // a + c a^3
  const float e = ex2_approx(__fmul_rn(kExp2Scale, inner));
  const float t = __fmaf_rn(-2.0f, rcp_approx(__fadd_rn(e, 1.0f)), 1.0f);
  const float h = __fmul_rn(0.5f, a);
  return {t, __fmaf_rn(h, t, h)};
}

// d(gate) from the gate value a, its tanh t and the rounded dgel = (g * b).to(dtype):
// dgel * (0.5 (1 + t) + 0.5 a (1 - t^2) dz/da).
__device__ __forceinline__ float geglu_dgate(float a, float t, float dgel) {
  const float dz = __fmaf_rn(__fmul_rn(a, a), kDz3, kSqrt2OverPi);
  const float omt = __fmaf_rn(-t, t, 1.0f);
  const float x = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, a), omt), dz);
  return __fmul_rn(dgel, __fadd_rn(__fmaf_rn(0.5f, t, 0.5f), x));
}

template <int DT>
__device__ __forceinline__ float geglu_out(float a, float b) {
  using E = Elem<DT>;
  return E::round(__fmul_rn(E::round(gelu_parts(a).gel), b));
}

template <int DT>
__device__ __forceinline__ void geglu_grad(float a, float b, float g, float* da, float* db) {
  using E = Elem<DT>;
  const GeluParts p = gelu_parts(a);
  *db = E::round(__fmul_rn(g, E::round(p.gel)));
  *da = geglu_dgate(a, p.t, E::round(__fmul_rn(g, b)));
}

// ---------------------------------------------------------------- paired forms (two lanes per register)
using sm100::f2_add;
using sm100::f2_fma;
using sm100::f2_mul;
using sm100::f2_pack;
using sm100::f2_unpack;

__device__ __forceinline__ uint64_t f2c(float c) { return f2_pack(c, c); }

struct GeluParts2 {
  uint64_t t, gel;
};

__device__ __forceinline__ GeluParts2 gelu_parts2(uint64_t a) {
  const uint64_t a2 = f2_mul(a, a);
  const uint64_t inner = f2_fma(f2_mul(f2c(kGeluC), a2), a, a);
  float x0, x1;
  f2_unpack(f2_mul(f2c(kExp2Scale), inner), x0, x1);
  float y0, y1;
  f2_unpack(f2_add(f2_pack(ex2_approx(x0), ex2_approx(x1)), f2c(1.0f)), y0, y1);
  const uint64_t t = f2_fma(f2c(-2.0f), f2_pack(rcp_approx(y0), rcp_approx(y1)), f2c(1.0f));
  const uint64_t h = f2_mul(f2c(0.5f), a);
  return {t, f2_fma(h, t, h)};
}

__device__ __forceinline__ uint64_t geglu_dgate2(uint64_t a, uint64_t t, uint64_t dgel) {
  const uint64_t dz = f2_fma(f2_mul(a, a), f2c(kDz3), f2c(kSqrt2OverPi));
  const uint64_t omt = f2_fma(t ^ 0x8000000080000000ull, t, f2c(1.0f));   // -t * t + 1
  const uint64_t x = f2_mul(f2_mul(f2_mul(f2c(0.5f), a), omt), dz);
  return f2_mul(dgel, f2_add(f2_fma(f2c(0.5f), t, f2c(0.5f)), x));
}


// Two 16-bit values in one 32-bit word (low half first): one cvt.rn.*x2 rounds a pair, and the
// rounded values come back to fp32 with integer ops, so the epilogue's conversions take half the
// conversion-pipe slots of per-element rounding, with the same round-to-nearest-even result.
template <bool F16> struct Pair;
template <> struct Pair<false> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return sm100::pack_bf16x2(lo, hi); }
  static __device__ __forceinline__ float lo(uint32_t v) { return __uint_as_float(v << 16); }
  static __device__ __forceinline__ float hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
};
template <> struct Pair<true> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return sm100::pack_f16x2(lo, hi); }
  static __device__ __forceinline__ float lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)v)); }
  static __device__ __forceinline__ float hi(uint32_t v) {
    return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
  }
};
// A rounded 16-bit pair as two fp32 lanes of one f32x2 register, and back (rounding both lanes).
template <bool F16>
__device__ __forceinline__ uint64_t widen(uint32_t v) { return f2_pack(Pair<F16>::lo(v), Pair<F16>::hi(v)); }
template <bool F16>
__device__ __forceinline__ uint32_t narrow(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  return Pair<F16>::pack(lo, hi);
}

}  // namespace gelu
}  // namespace krsi
