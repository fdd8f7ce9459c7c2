// geglu.cu - GEGLU (gelu-tanh gate) forward/backward for B200: 128-bit coalesced
// elementwise kernels over the merged [gate | value] GEMM output.
//
// The element arithmetic (rounding points of library/geglu.py:20-52) is in gelu.cuh.
// One work item is a 16-byte packet (8 bf16/f16 or 4 fp32) of one row: two packet loads
// from u (gate and value halves) per output packet.  A scalar variant covers F that is not
// a multiple of the packet width or unaligned buffers.
#include "common.cuh"
#include "gelu.cuh"

namespace krsi {
namespace {

using gelu::geglu_grad;
using gelu::geglu_out;

// A 16-byte packet of 16-bit elements as four pairs: gelu.cuh's paired forms (two lanes per f32x2
// instruction, each pair rounded by one cvt.rn.*x2), the same bits as geglu_out / geglu_grad.
template <int DT> struct Is16 { static constexpr bool value = DT != KRSI_F32; };

template <int DT>
__device__ __forceinline__ uint4 geglu_out_packet(uint4 a, uint4 b) {
  constexpr bool F16 = DT == KRSI_F16;
  auto one = [](uint32_t a2, uint32_t b2) {
    const uint32_t gel = gelu::narrow<F16>(gelu::gelu_parts2(gelu::widen<F16>(a2)).gel);
    return gelu::narrow<F16>(sm100::f2_mul(gelu::widen<F16>(gel), gelu::widen<F16>(b2)));
  };
  return make_uint4(one(a.x, b.x), one(a.y, b.y), one(a.z, b.z), one(a.w, b.w));
}

template <int DT>
__device__ __forceinline__ void geglu_grad_packet(uint4 a, uint4 b, uint4 g, uint4* da, uint4* db) {
  constexpr bool F16 = DT == KRSI_F16;
  auto one = [](uint32_t a2, uint32_t b2, uint32_t g2w, uint32_t* da2, uint32_t* db2) {
    const uint64_t g2 = gelu::widen<F16>(g2w), aa = gelu::widen<F16>(a2);
    const gelu::GeluParts2 pp = gelu::gelu_parts2(aa);
    *db2 = gelu::narrow<F16>(sm100::f2_mul(g2, gelu::widen<F16>(gelu::narrow<F16>(pp.gel))));
    const uint64_t dgel = gelu::widen<F16>(gelu::narrow<F16>(sm100::f2_mul(g2, gelu::widen<F16>(b2))));
    *da2 = gelu::narrow<F16>(gelu::geglu_dgate2(aa, pp.t, dgel));
  };
  one(a.x, b.x, g.x, &da->x, &db->x);
  one(a.y, b.y, g.y, &da->y, &db->y);
  one(a.z, b.z, g.z, &da->z, &db->z);
  one(a.w, b.w, g.w, &da->w, &db->w);
}

// Vector path: items = rows * FV packets, FV = F / VEC.  Grid-stride over items, two
// independent items per iteration so each thread keeps four 16-byte loads in flight.
template <int DT>
__global__ void __launch_bounds__(256)
geglu_fwd_vec(const typename Elem<DT>::T* __restrict__ u, typename Elem<DT>::T* __restrict__ out,
              uint32_t items, uint32_t FV) {
  pdl_enter();
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VEC = Vec16<T>::N;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < items; i0 += 2 * stride) {
    const uint32_t i1 = i0 + stride;
    const bool has1 = i1 < items;
    const uint32_t r0 = i0 / FV, c0 = i0 - r0 * FV;
    const uint32_t r1 = has1 ? i1 / FV : r0, c1 = has1 ? i1 - r1 * FV : c0;
    const T* u0 = u + ((size_t)r0 * 2 * FV + c0) * VEC;
    const T* u1 = u + ((size_t)r1 * 2 * FV + c1) * VEC;
    const auto a0 = ldg16_stream(u0), b0 = ldg16_stream(u0 + (size_t)FV * VEC);
    Vec16<T> a1, b1;
    if (has1) { a1 = ldg16_stream(u1); b1 = ldg16_stream(u1 + (size_t)FV * VEC); }
    Vec16<T> o0, o1;
    if constexpr (Is16<DT>::value) {
      auto u4 = [](const Vec16<T>& v) { return *reinterpret_cast<const uint4*>(&v); };
      *reinterpret_cast<uint4*>(&o0) = geglu_out_packet<DT>(u4(a0), u4(b0));
      if (has1) *reinterpret_cast<uint4*>(&o1) = geglu_out_packet<DT>(u4(a1), u4(b1));
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) o0.v[e] = E::store(geglu_out<DT>(E::load(a0.v[e]), E::load(b0.v[e])));
      if (has1) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) o1.v[e] = E::store(geglu_out<DT>(E::load(a1.v[e]), E::load(b1.v[e])));
      }
    }
    stg16(out + (size_t)i0 * VEC, o0);
    if (has1) stg16(out + (size_t)i1 * VEC, o1);
  }
}

template <int DT>
__global__ void __launch_bounds__(256)
geglu_bwd_vec(const typename Elem<DT>::T* __restrict__ g, const typename Elem<DT>::T* __restrict__ u,
              typename Elem<DT>::T* __restrict__ du, uint32_t items, uint32_t FV) {
  pdl_enter();
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VEC = Vec16<T>::N;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < items; i += stride) {
    const uint32_t r = i / FV, c = i - r * FV;
    const size_t ua = ((size_t)r * 2 * FV + c) * VEC;
    const auto av = ldg16_stream(u + ua);
    const auto bv = ldg16_stream(u + ua + (size_t)FV * VEC);
    const auto gv = ldg16_stream(g + (size_t)i * VEC);
    Vec16<T> dav, dbv;
    if constexpr (Is16<DT>::value) {
      auto u4 = [](const Vec16<T>& v) { return *reinterpret_cast<const uint4*>(&v); };
      geglu_grad_packet<DT>(u4(av), u4(bv), u4(gv), reinterpret_cast<uint4*>(&dav), reinterpret_cast<uint4*>(&dbv));
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        float da, db;
        geglu_grad<DT>(E::load(av.v[e]), E::load(bv.v[e]), E::load(gv.v[e]), &da, &db);
        dav.v[e] = E::store(da);
        dbv.v[e] = E::store(db);
      }
    }
    stg16(du + ua, dav);
    stg16(du + ua + (size_t)FV * VEC, dbv);
  }
}

// Scalar path: one element per item over rows * F.
template <int DT>
__global__ void __launch_bounds__(256)
geglu_fwd_scalar(const typename Elem<DT>::T* __restrict__ u, typename Elem<DT>::T* __restrict__ out,
                 int64_t items, int64_t F) {
  pdl_enter();
  using E = Elem<DT>;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, c = i - r * F;
    const float a = E::load(u[r * 2 * F + c]), b = E::load(u[r * 2 * F + F + c]);
    out[i] = E::store(geglu_out<DT>(a, b));
  }
}

template <int DT>
__global__ void __launch_bounds__(256)
geglu_bwd_scalar(const typename Elem<DT>::T* __restrict__ g, const typename Elem<DT>::T* __restrict__ u,
                 typename Elem<DT>::T* __restrict__ du, int64_t items, int64_t F) {
  pdl_enter();
  using E = Elem<DT>;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, c = i - r * F;
    const float a = E::load(u[r * 2 * F + c]), b = E::load(u[r * 2 * F + F + c]);
    float da, db;
    geglu_grad<DT>(a, b, E::load(g[i]), &da, &db);
    du[r * 2 * F + c] = E::store(da);
    du[r * 2 * F + F + c] = E::store(db);
  }
}

inline unsigned grid_for(int64_t items, int64_t per_block) {
  // Enough blocks to fill every SM several times over; grid-stride covers the rest.
  const int64_t cap = (int64_t)device_sm_count() * 8;
  int64_t b = (items + per_block - 1) / per_block;
  if (b > cap) b = cap;
  return (unsigned)(b > 0 ? b : 1);
}

template <int DT>
int fwd_t(const void* u, void* out, int64_t rows, int64_t F, cudaStream_t s) {
  using T = typename Elem<DT>::T;
  constexpr int VEC = Vec16<T>::N;
  const int64_t items = rows * F;
  if (F % VEC == 0 && aligned16(u) && aligned16(out) && items / VEC < 0xffffffffLL) {
    const int64_t vitems = items / VEC;
    KRSI_CUDA_TRY(launch_pdl(geglu_fwd_vec<DT>, dim3(grid_for(vitems, 512)), dim3(256), 0, s, (const T*)u, (T*)out,
                             (uint32_t)vitems, (uint32_t)(F / VEC)));
  } else {
    KRSI_CUDA_TRY(launch_pdl(geglu_fwd_scalar<DT>, dim3(grid_for(items, 256)), dim3(256), 0, s, (const T*)u, (T*)out,
                             items, F));
  }
  return KRSI_OK;
}

template <int DT>
int bwd_t(const void* g, const void* u, void* du, int64_t rows, int64_t F, cudaStream_t s) {
  using T = typename Elem<DT>::T;
  constexpr int VEC = Vec16<T>::N;
  const int64_t items = rows * F;
  if (F % VEC == 0 && aligned16(u) && aligned16(du) && aligned16(g) && items / VEC < 0xffffffffLL) {
    const int64_t vitems = items / VEC;
    KRSI_CUDA_TRY(launch_pdl(geglu_bwd_vec<DT>, dim3(grid_for(vitems, 256)), dim3(256), 0, s, (const T*)g, (const T*)u,
                             (T*)du, (uint32_t)vitems, (uint32_t)(F / VEC)));
  } else {
    KRSI_CUDA_TRY(launch_pdl(geglu_bwd_scalar<DT>, dim3(grid_for(items, 256)), dim3(256), 0, s, (const T*)g,
                             (const T*)u, (T*)du, items, F));
  }
  return KRSI_OK;
}

}  // namespace
}  // namespace krsi

using namespace krsi;

extern "C" int krsi_geglu_fwd(const void* u, void* out, int64_t rows, int64_t F, int dtype,
                              cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && F >= 0);
  if (rows == 0 || F == 0) return KRSI_OK;
  KRSI_CHECK_ARG(u && out);
  switch (dtype) {
    case KRSI_BF16: return fwd_t<KRSI_BF16>(u, out, rows, F, stream);
    case KRSI_F16: return fwd_t<KRSI_F16>(u, out, rows, F, stream);
    case KRSI_F32: return fwd_t<KRSI_F32>(u, out, rows, F, stream);
    default: return KRSI_ERR_INVALID_ARGUMENT;
  }
}

extern "C" int krsi_geglu_bwd(const void* g, const void* u, void* du, int64_t rows, int64_t F,
                              int dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && F >= 0);
  if (rows == 0 || F == 0) return KRSI_OK;
  KRSI_CHECK_ARG(g && u && du);
  switch (dtype) {
    case KRSI_BF16: return bwd_t<KRSI_BF16>(g, u, du, rows, F, stream);
    case KRSI_F16: return bwd_t<KRSI_F16>(g, u, du, rows, F, stream);
    case KRSI_F32: return bwd_t<KRSI_F32>(g, u, du, rows, F, stream);
    default: return KRSI_ERR_INVALID_ARGUMENT;
  }
}
