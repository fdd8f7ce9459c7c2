// rmsnorm.cu - RMSNorm forward/backward for B200: 128-bit coalesced row kernels with the
// rows held in registers, fp32 statistics, and a two-stage deterministic dweight reduction.
//
// Semantics follow library/rmsnorm.py of kernel-rsi:
//   forward  (rmsnorm.py:22-31, :54-59): r = 1/sqrt(sum(x^2)/n + eps); y = w * (x*r).to(w.dtype),
//            stored in x's dtype; r saved per row in fp32.
//   backward (rmsnorm.py:34-51, :62-68): n = (x*r).to(w.dtype); dw += g*n (fp32);
//            dn = (g*w) rounded to the promoted type of g and w, then fp32;
//            dx = r*dn - x*r^3*sum(dn*x)/n; dw = (sum of per-block partials).to(w.dtype).
// Layout: a row is a contiguous run of n elements handled by TPR threads (one warp for
// rows up to 512 packets, else a 256- or 1024-thread block).  Thread t owns NCH packets of
// VEC elements at columns (c*TPR + t)*VEC, so each load/store instruction of a row group is
// one fully coalesced 128-bit-per-thread transaction.  NCH is a compile-time constant, so
// the row slice stays in registers.

#include "common.cuh"

namespace krsi {
namespace {

constexpr int kBwdMaxBlocks = 296;   // fixed cap (2 x 148 SMs): the dw partial count, and
                                     // so the bits of dw, do not depend on the GPU model

template <int TPR> struct RowCfg {
  static constexpr int kThreads = TPR == 32 ? 256 : TPR;   // block size
  static constexpr int kRowsPerBlock = kThreads / TPR;      // rows processed together
};
// The forward's warp-per-row blocks hold two rows: its blocks are independent, so small blocks
// spread a few thousand rows evenly over the SMs (2048 rows: 1024 blocks, 6.9 per SM, instead of
// 256 blocks of which some SMs run two and others one).
template <int TPR> struct FwdRowCfg {
  static constexpr int kThreads = TPR == 32 ? 64 : TPR;
  static constexpr int kRowsPerBlock = kThreads / TPR;
};

// Sum over the TPR threads that share a row (a warp, or the whole block).
template <int TPR>
__device__ __forceinline__ float row_sum(float v, float* red) {
  if constexpr (TPR == 32) return warp_sum(v);
  else return block_sum<TPR>(v, red);
}

// Loads VEC consecutive elements of type T starting at p (16-byte aligned when VEC > 1).
template <int DT, int VEC>
__device__ __forceinline__ void load_vec(const typename Elem<DT>::T* p, float* out, bool stream) {
  using E = Elem<DT>;
  using T = typename E::T;
  if constexpr (VEC == 1) {
    out[0] = E::load(*p);
  } else {
    constexpr int PK = Vec16<T>::N;   // elements per 16-byte packet of this type
#pragma unroll
    for (int e = 0; e < VEC; e += PK) {
      const auto v = stream ? ldg16_stream(p + e) : ldg16(p + e);
#pragma unroll
      for (int k = 0; k < PK; ++k) out[e + k] = E::load(v.v[k]);
    }
  }
}

template <int DT, int VEC>
__device__ __forceinline__ void store_vec(typename Elem<DT>::T* p, const float* in) {
  using E = Elem<DT>;
  using T = typename E::T;
  if constexpr (VEC == 1) {
    *p = E::store(in[0]);
  } else {
    Vec16<T> o;
#pragma unroll
    for (int k = 0; k < VEC; ++k) o.v[k] = E::store(in[k]);
    stg16(p, o);
  }
}

template <int XT, int WT, int TPR, int VEC, int NCH>
__global__ void __launch_bounds__(FwdRowCfg<TPR>::kThreads)
rms_fwd_kernel(const typename Elem<XT>::T* __restrict__ x, const typename Elem<WT>::T* __restrict__ w,
               typename Elem<XT>::T* __restrict__ y, float* __restrict__ rstd, int64_t rows, int n, float eps) {
  pdl_enter();
  using WE = Elem<WT>;
  __shared__ float red[32];
  const int t = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * FwdRowCfg<TPR>::kRowsPerBlock + threadIdx.x / TPR;
  const bool live = row < rows;   // a block-per-row group is always live
  const auto* xr = x + row * n;
  float xv[NCH][VEC];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * TPR + t) * VEC;
    if (live && col < n) {
      load_vec<XT, VEC>(xr + col, xv[c], true);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) xv[c][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) ss = fmaf(xv[c][e], xv[c][e], ss);
  }
  ss = row_sum<TPR>(ss, red);
  const float r = 1.0f / sqrtf(ss / (float)n + eps);
  if (!live) return;
  if (t == 0) rstd[row] = r;
  auto* yr = y + row * n;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * TPR + t) * VEC;
    if (col < n) {
      float wv[VEC], o[VEC];
      load_vec<WT, VEC>(w + col, wv, false);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = WE::round(wv[e] * WE::round(xv[c][e] * r));
      store_vec<XT, VEC>(yr + col, o);
    }
  }
}

// Warp-per-row plans with up to 40 elements per thread keep their running dw sums in shared memory
// (lane-interleaved float4s: conflict-free) instead of registers, which fits two 256-thread blocks
// per SM: twice the rows in flight for a latency-bound backward.  The sums are the same fmaf chain
// in the same row order, so dw is bitwise unchanged.
template <int TPR, int VEC, int NCH>
constexpr bool kBwdSmemAcc = TPR == 32 && NCH * VEC <= 40 && VEC % 4 == 0;
template <int TPR, int VEC, int NCH>
constexpr int kBwdMinBlocks = kBwdSmemAcc<TPR, VEC, NCH> ? 2 : 1;
// index of (chunk c, element e) of lane t in a warp's interleaved accumulator
template <int VEC>
__device__ __forceinline__ int acc_idx(int c, int e, int t) { return ((c * (VEC / 4) + e / 4) * 32 + t) * 4 + e % 4; }

// 16-bit warp-per-row plans also stage the warp's NEXT row of g and x in shared memory with
// cp.async while the current row is reduced and stored, so a warp always has a row in flight
// (the loads of the plain loop wait a full DRAM round trip per row).  Each lane copies and
// later reads only its own 16-byte packets, so cp.async.wait_group is the only
// synchronisation.  Stage: per warp, [x | g][NCH][32 lanes] of 16 bytes, and a third part for the
// added gradient when there is one (read at the dx store, refilled after it: measured at the block
// shape, loading it from global memory at the store cost a DRAM round trip per row).
template <int XT, int TPR, int VEC, int NCH>
constexpr bool kBwdStage = kBwdSmemAcc<TPR, VEC, NCH> && sizeof(typename Elem<XT>::T) == 2 && VEC == 8;

// Copies 16 bytes from global to shared.  A slot is refilled only after the loop that reads it
// has ended and the warp has passed __syncwarp(), which orders those shared-memory reads before
// the copy's writes.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int XT, int WT, int TPR, int VEC, int NCH>
__global__ void __launch_bounds__(RowCfg<TPR>::kThreads, kBwdMinBlocks<TPR, VEC, NCH>)
rms_bwd_kernel(const typename Elem<XT>::T* __restrict__ g, const typename Elem<XT>::T* __restrict__ x,
               const typename Elem<WT>::T* __restrict__ w, const float* __restrict__ rstd,
               typename Elem<XT>::T* __restrict__ dx, float* __restrict__ dw_part, int64_t rows, int n,
               const typename Elem<XT>::T* __restrict__ gadd) {
  pdl_enter();
  using WE = Elem<WT>;
  using DE = Elem<Promote<XT, WT>::value>;   // dtype of the g*w product
  constexpr int RPB = RowCfg<TPR>::kRowsPerBlock;
  extern __shared__ __align__(16) float smem_dw[];   // [RPB][n] when RPB > 1
  __shared__ float red[32];
  const int t = threadIdx.x % TPR;
  const int sub = threadIdx.x / TPR;

  constexpr bool SACC = kBwdSmemAcc<TPR, VEC, NCH>;
  constexpr bool STAGE = kBwdStage<XT, TPR, VEC, NCH>;
  // STAGE: this warp's stage, after the RPB accumulators; [x | g | gadd] when gadd is staged
  const bool sga = STAGE && gadd != nullptr;
  uint4* stg = reinterpret_cast<uint4*>(smem_dw + RPB * (NCH * VEC * 32)) + sub * ((sga ? 3 : 2) * NCH * 32);
  float dwv[NCH][VEC];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int e = 0; e < VEC; ++e) dwv[c][e] = 0.f;
  float4* acc4 = reinterpret_cast<float4*>(smem_dw + sub * (NCH * VEC * 32));   // SACC: this warp's sums
  if constexpr (SACC) {
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int e = 0; e < VEC; e += 4) acc4[acc_idx<VEC>(c, e, t) / 4] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  const int64_t stride = (int64_t)gridDim.x * RPB;
  if constexpr (STAGE) {   // prologue: stage this warp's first row
    const int64_t row = (int64_t)blockIdx.x * RPB + sub;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * TPR + t) * VEC;
      if (row < rows && col < n) {
        cp_async16(&stg[c * 32 + t], x + row * n + col);
        cp_async16(&stg[(NCH + c) * 32 + t], g + row * n + col);
        if (sga) cp_async16(&stg[(2 * NCH + c) * 32 + t], gadd + row * n + col);
      }
    }
    cp_async_commit();
  }

  for (int64_t row0 = (int64_t)blockIdx.x * RPB; row0 < rows; row0 += stride) {
    const int64_t row = row0 + sub;
    const bool live = row < rows;
    const auto* xr = x + row * n;
    const auto* gr = g + row * n;
    float xv[NCH][VEC], dn[NCH][VEC];
    if constexpr (STAGE) cp_async_wait_all();
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * TPR + t) * VEC;
      if (live && col < n) {
        if constexpr (STAGE) {
          using E = Elem<XT>;
          Vec16<typename E::T> vx, vg;
          *reinterpret_cast<uint4*>(&vx) = stg[c * 32 + t];
          *reinterpret_cast<uint4*>(&vg) = stg[(NCH + c) * 32 + t];
#pragma unroll
          for (int e = 0; e < VEC; ++e) { xv[c][e] = E::load(vx.v[e]); dn[c][e] = E::load(vg.v[e]); }
        } else {
          load_vec<XT, VEC>(xr + col, xv[c], true);
          load_vec<XT, VEC>(gr + col, dn[c], true);   // dn holds g until converted below
        }
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) { xv[c][e] = 0.f; dn[c][e] = 0.f; }
      }
    }
    if constexpr (STAGE) __syncwarp();   // every lane's reads of the stage precede its refills
    const float r = live ? rstd[row] : 0.f;
    const int64_t nrow = row + stride;   // this warp's next row (STAGE: staged below)
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * TPR + t) * VEC;
      float wv[VEC];
      if (col < n) load_vec<WT, VEC>(w + col, wv, false);
      else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) wv[e] = 0.f;
      }
      if constexpr (SACC) {
        if (live && col < n) {
#pragma unroll
          for (int e = 0; e < VEC; e += 4) {
            float4 s = acc4[acc_idx<VEC>(c, e, t) / 4];
            s.x = fmaf(dn[c][e], WE::round(xv[c][e] * r), s.x);
            s.y = fmaf(dn[c][e + 1], WE::round(xv[c][e + 1] * r), s.y);
            s.z = fmaf(dn[c][e + 2], WE::round(xv[c][e + 2] * r), s.z);
            s.w = fmaf(dn[c][e + 3], WE::round(xv[c][e + 3] * r), s.w);
            acc4[acc_idx<VEC>(c, e, t) / 4] = s;
          }
        }
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float gg = dn[c][e];
        if constexpr (!SACC) dwv[c][e] = fmaf(gg, WE::round(xv[c][e] * r), dwv[c][e]);
        dn[c][e] = DE::round(gg * wv[e]);
        dot = fmaf(dn[c][e], xv[c][e], dot);
      }
      if constexpr (STAGE) {   // chunk c's slots were read before the __syncwarp() above
        const int col = (c * TPR + t) * VEC;
        if (nrow < rows && col < n) {
          cp_async16(&stg[c * 32 + t], x + nrow * n + col);
          cp_async16(&stg[(NCH + c) * 32 + t], g + nrow * n + col);
        }
      }
    }
    if constexpr (STAGE) cp_async_commit();
    dot = row_sum<TPR>(dot, red);
    const float k = r * r * r * (dot / (float)n);
    if (live) {
      auto* dxr = dx + row * n;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int col = (c * TPR + t) * VEC;
        if (col < n) {
          float o[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = r * dn[c][e] - xv[c][e] * k;
          if (gadd != nullptr) {   // a second gradient of x (a residual branch), added before rounding
            float ga[VEC];
            if (sga) {
              using E = Elem<XT>;
              Vec16<typename E::T> vga;
              *reinterpret_cast<uint4*>(&vga) = stg[(2 * NCH + c) * 32 + t];
#pragma unroll
              for (int e = 0; e < VEC; ++e) ga[e] = E::load(vga.v[e]);
            } else {
              load_vec<XT, VEC>(gadd + row * n + col, ga, true);
            }
#pragma unroll
            for (int e = 0; e < VEC; ++e) o[e] += ga[e];
          }
          store_vec<XT, VEC>(dxr + col, o);
        }
      }
    }
    if (sga) {   // the added gradient's slots were read above: refill them with the next row's
      __syncwarp();
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int col = (c * TPR + t) * VEC;
        if (nrow < rows && col < n) cp_async16(&stg[(2 * NCH + c) * 32 + t], gadd + nrow * n + col);
      }
      cp_async_commit();
    }
  }

  if constexpr (STAGE) cp_async_wait_all();   // nothing is left in flight (the last group is empty)

  // Per-block dw partial; the RPB row groups of a block are combined in a fixed order.
  float* out = dw_part + (int64_t)blockIdx.x * n;
  if constexpr (!SACC) {
    float* dst = RPB == 1 ? out : smem_dw + sub * n;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int col = (c * TPR + t) * VEC + e;
        if (col < n) dst[col] = dwv[c][e];
      }
  }
  if constexpr (RPB > 1) {
    __syncthreads();
    for (int col = threadIdx.x; col < n; col += blockDim.x) {
      float s = 0.f;
      if constexpr (SACC) {
        const int c = col / (TPR * VEC), rem = col % (TPR * VEC);
        const int idx = acc_idx<VEC>(c, rem % VEC, rem / VEC);
#pragma unroll
        for (int i = 0; i < RPB; ++i) s += smem_dw[i * (NCH * VEC * 32) + idx];
      } else {
#pragma unroll
        for (int i = 0; i < RPB; ++i) s += smem_dw[i * n + col];
      }
      out[col] = s;
    }
  }
}

// Stage 2 of dw: dw[col] = sum over the partial rows in a fixed order, rounded to w's dtype.
// A block covers 128 columns (one float4 per lane) with 16 warps; warp i sums partial rows
// i, i+16, ... with its loads issued 16 at a time (one L2 round trip for up to 256 partial rows),
// then the 16 warp sums are added in index order.  The order depends only on the partial count,
// so dw is bitwise reproducible.
constexpr int kRedWarps = 16;
constexpr int kRedBatch = 16;
template <int WT>
__global__ void __launch_bounds__(kRedWarps * 32)
rms_dw_reduce_kernel(const float* __restrict__ part, typename Elem<WT>::T* __restrict__ dw, int nparts, int n) {
  pdl_enter();
  __shared__ float4 acc[kRedWarps][32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int col = (blockIdx.x * 32 + lane) * 4;
  const bool vec = (n % 4) == 0;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col < n) {
    for (int p0 = wid; p0 < nparts; p0 += kRedBatch * kRedWarps) {
      float4 v[kRedBatch];
#pragma unroll
      for (int u = 0; u < kRedBatch; ++u) {
        const int p = p0 + u * kRedWarps;
        const float* src = part + (int64_t)p * n + col;
        if (p >= nparts) {
          v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (vec) {
          v[u] = __ldg(reinterpret_cast<const float4*>(src));
        } else {
          v[u].x = __ldg(src);
          v[u].y = col + 1 < n ? __ldg(src + 1) : 0.f;
          v[u].z = col + 2 < n ? __ldg(src + 2) : 0.f;
          v[u].w = col + 3 < n ? __ldg(src + 3) : 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < kRedBatch; ++u) {
        s.x += v[u].x; s.y += v[u].y; s.z += v[u].z; s.w += v[u].w;
      }
    }
  }
  acc[wid][lane] = s;
  __syncthreads();
  if (wid == 0 && col < n) {
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kRedWarps; ++i) {
      t.x += acc[i][lane].x; t.y += acc[i][lane].y; t.z += acc[i][lane].z; t.w += acc[i][lane].w;
    }
    const float tv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (col + e < n) dw[col + e] = Elem<WT>::store(tv[e]);
  }
}

// ---------------------------------------------------------------- host-side planning
struct Plan {
  int tpr, vec, nch;
};

inline int elem_size(int dt) { return dt == KRSI_F32 ? 4 : 2; }

// Warp-per-row chunk counts that are compiled; a needed count is rounded up to the next.
constexpr int kWarpNch[] = {1, 2, 3, 4, 5, 6, 8, 9, 12, 16};
constexpr int kBlockNch[] = {1, 2, 4, 8, 16};

inline bool plan_rows(int64_t n, int x_dtype, bool vec_ok, Plan* p) {
  p->vec = vec_ok ? 16 / elem_size(x_dtype) : 1;
  const int64_t need32 = (n + 32 * p->vec - 1) / (32 * p->vec);
  for (int c : kWarpNch)
    if (c >= need32) { p->tpr = 32; p->nch = c; return true; }
  for (int tp : {256, 1024}) {
    const int64_t need = (n + (int64_t)tp * p->vec - 1) / ((int64_t)tp * p->vec);
    for (int c : kBlockNch)
      if (c >= need) { p->tpr = tp; p->nch = c; return true; }
  }
  return false;
}

inline int64_t bwd_blocks(int64_t rows, const Plan& p) {
  const int rpb = p.tpr == 32 ? RowCfg<32>::kRowsPerBlock : 1;
  const int64_t need = (rows + rpb - 1) / rpb;
  return need < kBwdMaxBlocks ? need : kBwdMaxBlocks;
}

struct FwdArgs {
  const void* x; const void* w; void* y; float* rstd; int64_t rows; int n; float eps; cudaStream_t s;
};
struct BwdArgs {
  const void* g; const void* x; const void* w; const float* rstd; void* dx; void* dw; float* part;
  int64_t nblocks; int64_t rows; int n; cudaStream_t s; const void* gadd = nullptr;
};

template <int XT, int WT, int TPR, int VEC, int NCH>
int run_fwd(const FwdArgs& a) {
  using Cfg = FwdRowCfg<TPR>;
  const int64_t grid = (a.rows + Cfg::kRowsPerBlock - 1) / Cfg::kRowsPerBlock;
  if (grid > 0x7fffffff) return KRSI_ERR_UNSUPPORTED;
  KRSI_CUDA_TRY(launch_pdl(rms_fwd_kernel<XT, WT, TPR, VEC, NCH>, dim3((unsigned)grid), dim3(Cfg::kThreads), 0, a.s,
                           (const typename Elem<XT>::T*)a.x, (const typename Elem<WT>::T*)a.w,
                           (typename Elem<XT>::T*)a.y, a.rstd, a.rows, a.n, a.eps));
  return KRSI_OK;
}

template <int XT, int WT, int TPR, int VEC, int NCH>
int run_bwd(const BwdArgs& a) {
  using Cfg = RowCfg<TPR>;
  const size_t per_warp = kBwdSmemAcc<TPR, VEC, NCH> ? (size_t)NCH * VEC * 32 : (size_t)a.n;
  const size_t stage =
      kBwdStage<XT, TPR, VEC, NCH> ? (size_t)Cfg::kRowsPerBlock * (a.gadd ? 3 : 2) * NCH * 32 * 16 : 0;
  const size_t smem =
      Cfg::kRowsPerBlock > 1 ? (size_t)Cfg::kRowsPerBlock * per_warp * sizeof(float) + stage : 0;
  auto kern = rms_bwd_kernel<XT, WT, TPR, VEC, NCH>;
  if (smem > 48 * 1024)
    KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  KRSI_CUDA_TRY(launch_pdl(kern, dim3((unsigned)a.nblocks), dim3(Cfg::kThreads), smem, a.s,
                           (const typename Elem<XT>::T*)a.g, (const typename Elem<XT>::T*)a.x,
                           (const typename Elem<WT>::T*)a.w, a.rstd, (typename Elem<XT>::T*)a.dx, a.part, a.rows,
                           a.n, (const typename Elem<XT>::T*)a.gadd));
  KRSI_CUDA_TRY(launch_pdl(rms_dw_reduce_kernel<WT>, dim3((unsigned)((a.n + 127) / 128)), dim3(kRedWarps * 32), 0, a.s,
                           (const float*)a.part, (typename Elem<WT>::T*)a.dw, (int)a.nblocks, a.n));
  return KRSI_OK;
}

// Runtime (tpr, nch) -> template instance, for one (XT, WT, VEC).
template <int XT, int WT, int VEC, bool FWD, class Args>
int dispatch_shape(const Plan& p, const Args& a) {
#define KRSI_RUN(TPR, NCH) \
  if constexpr (FWD) return run_fwd<XT, WT, TPR, VEC, NCH>(a); else return run_bwd<XT, WT, TPR, VEC, NCH>(a)
  if (p.tpr == 32) {
    switch (p.nch) {
      case 1: KRSI_RUN(32, 1); case 2: KRSI_RUN(32, 2); case 3: KRSI_RUN(32, 3);
      case 4: KRSI_RUN(32, 4); case 5: KRSI_RUN(32, 5); case 6: KRSI_RUN(32, 6); case 8: KRSI_RUN(32, 8);
      case 9: KRSI_RUN(32, 9); case 12: KRSI_RUN(32, 12); case 16: KRSI_RUN(32, 16);
    }
  } else if (p.tpr == 256) {
    switch (p.nch) {
      case 1: KRSI_RUN(256, 1); case 2: KRSI_RUN(256, 2); case 4: KRSI_RUN(256, 4);
      case 8: KRSI_RUN(256, 8); case 16: KRSI_RUN(256, 16);
    }
  } else if (p.tpr == 1024) {
    switch (p.nch) {
      case 1: KRSI_RUN(1024, 1); case 2: KRSI_RUN(1024, 2); case 4: KRSI_RUN(1024, 4);
      case 8: KRSI_RUN(1024, 8); case 16: KRSI_RUN(1024, 16);
    }
  }
#undef KRSI_RUN
  return KRSI_ERR_UNSUPPORTED;
}

template <bool FWD, class Args>
int dispatch(int x_dtype, int w_dtype, const Plan& p, const Args& a) {
#define KRSI_DT(XT, WT, VW)                                                     \
  if (x_dtype == XT && w_dtype == WT)                                           \
    return p.vec == 1 ? dispatch_shape<XT, WT, 1, FWD>(p, a) : dispatch_shape<XT, WT, VW, FWD>(p, a)
  KRSI_DT(KRSI_F32, KRSI_F32, 4);
  KRSI_DT(KRSI_BF16, KRSI_BF16, 8);
  KRSI_DT(KRSI_F16, KRSI_F16, 8);
  KRSI_DT(KRSI_BF16, KRSI_F32, 8);
  KRSI_DT(KRSI_F16, KRSI_F32, 8);
#undef KRSI_DT
  return KRSI_ERR_UNSUPPORTED;
}

inline bool dtype_ok(int d) { return d == KRSI_F32 || d == KRSI_BF16 || d == KRSI_F16; }

}  // namespace
}  // namespace krsi

using namespace krsi;

extern "C" int krsi_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows, int64_t n,
                                float eps, int x_dtype, int w_dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && n >= 0 && dtype_ok(x_dtype) && dtype_ok(w_dtype));
  if (rows == 0) return KRSI_OK;
  KRSI_CHECK_ARG(n > 0 && x && w && y && rstd);
  if (n > 0x7fffffff) return KRSI_ERR_UNSUPPORTED;
  const int vw = 16 / elem_size(x_dtype);
  const bool vec_ok = (n % vw == 0) && aligned16(x) && aligned16(y) && aligned16(w);
  Plan p;
  if (!plan_rows(n, x_dtype, vec_ok, &p)) return KRSI_ERR_UNSUPPORTED;
  return dispatch<true>(x_dtype, w_dtype, p, FwdArgs{x, w, y, rstd, rows, (int)n, eps, stream});
}

extern "C" int krsi_rmsnorm_bwd_workspace_size(int64_t rows, int64_t n, size_t* bytes) {
  KRSI_CHECK_ARG(rows >= 0 && n >= 0 && bytes);
  if (n > 0x7fffffff) return KRSI_ERR_UNSUPPORTED;
  // Upper bound over every plan (the block-per-row plans use one row per block).
  const int64_t nb = rows < kBwdMaxBlocks ? rows : kBwdMaxBlocks;
  *bytes = (size_t)nb * (size_t)n * sizeof(float);
  return KRSI_OK;
}

namespace krsi {
namespace {
int rmsnorm_bwd_impl(const void* g, const void* x, const void* w, const float* rstd, const void* gadd, void* dx,
                     void* dw, void* workspace, size_t workspace_bytes, int64_t rows, int64_t n, int x_dtype,
                     int w_dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && n >= 0 && dtype_ok(x_dtype) && dtype_ok(w_dtype));
  if (n == 0) return KRSI_OK;
  KRSI_CHECK_ARG(w && dw);
  if (n > 0x7fffffff) return KRSI_ERR_UNSUPPORTED;
  if (rows == 0) {  // dw of an empty batch is zero
    KRSI_CUDA_TRY(cudaMemsetAsync(dw, 0, (size_t)n * elem_size(w_dtype), stream));
    return KRSI_OK;
  }
  KRSI_CHECK_ARG(g && x && rstd && dx);
  const int vw = 16 / elem_size(x_dtype);
  const bool vec_ok = (n % vw == 0) && aligned16(x) && aligned16(g) && aligned16(dx) && aligned16(w);
  Plan p;
  if (!plan_rows(n, x_dtype, vec_ok, &p)) return KRSI_ERR_UNSUPPORTED;
  const int64_t nblocks = bwd_blocks(rows, p);
  if (!workspace || workspace_bytes < (size_t)nblocks * (size_t)n * sizeof(float)) return KRSI_ERR_WORKSPACE;
  if (gadd && p.vec > 1 && !aligned16(gadd)) return KRSI_ERR_MISALIGNED;
  return dispatch<false>(x_dtype, w_dtype, p,
                         BwdArgs{g, x, w, rstd, dx, dw, static_cast<float*>(workspace), nblocks, rows, (int)n, stream,
                                 gadd});
}
}  // namespace
}  // namespace krsi

extern "C" int krsi_rmsnorm_bwd(const void* g, const void* x, const void* w, const float* rstd, void* dx, void* dw,
                                void* workspace, size_t workspace_bytes, int64_t rows, int64_t n, int x_dtype,
                                int w_dtype, cudaStream_t stream) {
  return rmsnorm_bwd_impl(g, x, w, rstd, nullptr, dx, dw, workspace, workspace_bytes, rows, n, x_dtype, w_dtype,
                          stream);
}

extern "C" int krsi_rmsnorm_bwd_add(const void* g, const void* x, const void* w, const float* rstd, const void* gadd,
                                    void* dx, void* dw, void* workspace, size_t workspace_bytes, int64_t rows,
                                    int64_t n, int x_dtype, int w_dtype, cudaStream_t stream) {
  if (rows > 0 && n > 0) KRSI_CHECK_ARG(gadd);
  return rmsnorm_bwd_impl(g, x, w, rstd, gadd, dx, dw, workspace, workspace_bytes, rows, n, x_dtype, w_dtype,
                          stream);
}

// ---------------------------------------------------------------- allocation-free backward
// Some callers cannot allocate device memory at the point where they run the backward: hosts
// that own every device allocation themselves (an embedding framework with its own pool), code
// that runs while other work holds the allocator, or real-time loops where a cudaMalloc would
// stall the device.  krsi_rmsnorm_bwd_noalloc gives them the same kernels with the dweight
// partial sums placed in a fixed, file-scope device array instead of a caller workspace.
namespace krsi {
namespace {

constexpr int64_t kNoAllocScratchFloats = 1 << 20;   // 4 MiB: (dw partial rows) x n <= 1,048,576
// One copy per GPU that loads this library, alive until the process exits.  Host code may not use
// the symbol as a pointer (it names a host-side stand-in): its device address is looked up per
// device with cudaGetSymbolAddress.
static __device__ __align__(256) float g_rms_noalloc_scratch[kNoAllocScratchFloats];

// Device address of the scratch array in the current context.  It is looked up on every call
// (a host-side table lookup once the module is loaded) rather than cached, so a pointer never
// outlives the context it belongs to (cudaDeviceReset, a torn-down primary context).  The first
// call on a device loads the module and must therefore come before any stream capture.
int noalloc_scratch(float** out) {
  void* p = nullptr;
  KRSI_CUDA_TRY(cudaGetSymbolAddress(&p, g_rms_noalloc_scratch));
  *out = static_cast<float*>(p);
  return KRSI_OK;
}

}  // namespace
}  // namespace krsi

extern "C" int krsi_rmsnorm_bwd_noalloc(const void* g, const void* x, const void* w, const float* rstd, void* dx,
                                        void* dw, int64_t rows, int64_t n, int x_dtype, int w_dtype,
                                        cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && n >= 0 && dtype_ok(x_dtype) && dtype_ok(w_dtype));
  if (n == 0) return KRSI_OK;
  KRSI_CHECK_ARG(w && dw);
  if (n > 0x7fffffff) return KRSI_ERR_UNSUPPORTED;
  if (rows == 0) {  // dw of an empty batch is zero
    KRSI_CUDA_TRY(cudaMemsetAsync(dw, 0, (size_t)n * elem_size(w_dtype), stream));
    return KRSI_OK;
  }
  KRSI_CHECK_ARG(g && x && rstd && dx);
  const int vw = 16 / elem_size(x_dtype);
  const bool vec_ok = (n % vw == 0) && aligned16(x) && aligned16(g) && aligned16(dx) && aligned16(w);
  Plan p;
  if (!plan_rows(n, x_dtype, vec_ok, &p)) return KRSI_ERR_UNSUPPORTED;
  const int64_t nblocks = bwd_blocks(rows, p);
  if (nblocks * n > kNoAllocScratchFloats) return KRSI_ERR_UNSUPPORTED;   // beyond the fixed scratch
  float* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != KRSI_OK) return rc;
  // Every partial row the reduction reads is written by this launch first, so the array's
  // previous contents never leak into the result and nothing needs clearing.
  return dispatch<false>(x_dtype, w_dtype, p, BwdArgs{g, x, w, rstd, dx, dw, scratch, nblocks, rows, (int)n, stream});
}
