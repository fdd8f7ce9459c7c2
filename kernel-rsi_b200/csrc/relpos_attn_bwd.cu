// relpos_attn_bwd.cu - relative-position-bias flash attention backward for B200 (sm_100a).
//
// Computes the gradients library/relpos_attention.py:62-157 computes (_bwd_dkdv, _bwd_dq and
// the torch reductions of _backward_impl), with lse in the log2 domain:
//   delta_i = sum_d dO[i,d] * O32[i,d]                       (fp32 O, :144)
//   P = exp2(s2 - lse), dV = P^T dO, dP = dO V^T, dS = P (dP - delta)
//   dK = scale dS^T Q, dQ = scale dS K, dpd[h, j-i+S-1] = sum_b dS[b,h,i,j]   (:154-156)
//
// Kernels:
//   bwd_prep   delta from dO and O32; zeroes the fp32 dQ accumulator.
//   bwd_main   one CTA per (b*H + h, 128-key block); loops over the 128-query blocks:
//                warp 0     TMA producer: K and V once; Q, dO tiles + lse/delta/bias slab
//                           per query block (2-stage ring)
//                warp 1     TMEM owner + tcgen05.mma issuer:
//                             S^T = K Q^T, dP^T = V dO^T              (SS, K = DP)
//                             dV += P^T dO, dK += dS^T Q               (TS: P^T/dS^T in TMEM)
//                             dQ  = dS K                              (SS: dS staged in smem)
//                warps 2-5  one key row per thread: P^T, dS^T (fp32) -> bf16 into TMEM and
//                           smem; dBias diagonal sums of the fp32 dS tile by a warp-shuffle
//                           scan, written as one 255-vector per tile (no S x S buffer)
//                warps 6-9  one query row per thread: dQ tile from TMEM -> fp32 vector
//                           reductions into the accumulator; at the end dK, dV -> dqkv
//   bwd_dq     dQ accumulator * scale -> dqkv (input dtype)
//   bwd_dpd    dpd[h, t] = fixed-order sum of the per-tile diagonal partials (deterministic)
// dK, dV and dpd are bitwise reproducible; dQ sums per-key-block fp32 partials in arrival
// order (like FlashAttention's dQ accumulation), so its last bits can vary run to run.
#include <string.h>

#include <type_traits>

#include "attn_common.cuh"
#include "common.cuh"
#include "watchdog.cuh"

KRSI_DEFINE_WATCHDOG(attn_bwd)

namespace krsi {
int attn_padded_dim(int64_t D);   // relpos_attn_fwd.cu

namespace {

using namespace sm100;
using attn::kTileRows;

constexpr int kBlk = 128;          // keys per CTA, queries per iteration
constexpr int kThreads = 384;       // 3 warpgroups: {producer, MMA, -, -}, compute, dQ/epilogue
constexpr uint32_t kRegsCtl = 96;   // after setmaxnreg (launch 168 x 384 = 128 x (96 + 248 + 160))
constexpr uint32_t kRegsCompute = 248;
constexpr uint32_t kRegsDq = 160;
constexpr int kBins = 160;          // per-warp diagonal bins: 32 keys x 128 queries -> 159 diagonals
constexpr int kDiag = 2 * kBlk - 1;     // 255 diagonals per 128 x 128 tile


constexpr float kLog2e = 1.4426950408889634f;

template <int DP>
struct BwdCfg {
  static constexpr uint32_t kTile = attn::Tile<DP>::kBytes;
  static constexpr int NQS = 2;                                   // Q/dO stages
  static constexpr uint32_t kKOff = 0;
  static constexpr uint32_t kVOff = kKOff + kTile;
  static constexpr uint32_t kQOff = kVOff + kTile;                // stage s: Q at kQOff + s*2*kTile
  static constexpr uint32_t kDSOff = kQOff + NQS * 2 * kTile;     // dS (bf16, MN-major SW128): 2 x 16 KB
  static constexpr uint32_t kVecOff = kDSOff + 2 * 16384;         // per stage: lse[128], delta[128], slab[256]
  static constexpr uint32_t kVecBytes = (128 + 128 + 256) * 4;
  static constexpr uint32_t kBarOff = kVecOff + NQS * kVecBytes;
  static constexpr int kNumBars = 1 + 2 * NQS + 8;
  static constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;
  static constexpr uint32_t kRowOff = kMiscOff + 16;   // resident pd / lse / delta rows (runtime length)
  static constexpr uint32_t kSmem = kRowOff + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kST = 0, kDPT = 128, kDV = 256, kDK = 256 + DP, kDQ = 256 + 2 * DP;
  static_assert(kDQ + DP <= kTmemCols, "backward TMEM plan needs DP <= 80");
};

struct BwdArgs {
  const float* pd;
  const float* lse;
  const float* delta;
  float* dq_acc;          // [B*S, H*D] fp32
  float* dbias_part;      // [B*H, n_kb, n_qb, 4 warps, kBins]
  void* dqkv;
  int64_t dqkv_stride;
  int B, S, H, D, n_blk;
  float scale_log2, scale;
  uint32_t spin_limit;
};

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}


// Resident rows (one load per CTA): pd[h, :] * log2(e) with kRowPad zeros before and 128 after
// (every key - query + S - 1 a tile forms stays inside), then lse and delta of this (b, h), each
// followed by 128 zeros for queries past S.
constexpr int kRowPad = 256;
__host__ __device__ constexpr int64_t pd_row_floats(int64_t S) { return 2 * S - 1 + kRowPad + 128; }
__host__ __device__ constexpr int64_t vec_row_floats(int64_t S) { return S + 128; }
__host__ __device__ constexpr int64_t rows_bytes(int64_t S) { return (pd_row_floats(S) + 2 * vec_row_floats(S)) * 4; }

template <int DP, bool F16, bool RES>
__global__ void __launch_bounds__(kThreads, 1)
relpos_bwd_main_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap omap,
                       const BwdArgs a) {
  using C = BwdCfg<DP>;
  constexpr int NQS = C::NQS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 1 + NQS;
  uint64_t* sdp_ready = bars + 1 + 2 * NQS;
  uint64_t* p_ready = sdp_ready + 1;
  uint64_t* ds_ready = sdp_ready + 2;
  uint64_t* dq_ready = sdp_ready + 3;
  uint64_t* dq_free = sdp_ready + 4;
  uint64_t* kdv_done = sdp_ready + 5;
  uint64_t* drain = sdp_ready + 6;
  uint64_t* row_full = sdp_ready + 7;
  float* pd_row = reinterpret_cast<float*>(smem + C::kRowOff);
  float* lse_row = pd_row + pd_row_floats(a.S);
  float* del_row = lse_row + vec_row_floats(a.S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb = blockIdx.x, bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int k0 = kb * kBlk;
  const int nq = a.n_blk;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(&qdo_full[s], RES ? 1 : 2);   // TMA expect_tx (+ vectors/slab stores)
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(sdp_ready, 1);
    mbar_init(p_ready, 128);
    mbar_init(ds_ready, 128);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 128);
    mbar_init(kdv_done, 1);
    mbar_init(drain, 1);
    mbar_init(row_full, 64);
    abort_flag[0] = 0;
    abort_flag[1] = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&omap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Each role runs entirely inside the branch that sets its register budget.
  if (warp < 4) {
    regs_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * C::kTile);
      attn::load_tile<DP>(smem + C::kKOff, &qmap, kv_full, a.H + h, k0, b);
      attn::load_tile<DP>(smem + C::kVOff, &qmap, kv_full, 2 * a.H + h, k0, b);
    }
    const int two_s = 2 * a.S - 1;
    const float* pdh = a.pd + (size_t)h * two_s;
    const float* lse_bh = a.lse + (size_t)bh * a.S;
    const float* del_bh = a.delta + (size_t)bh * a.S;

    for (int i = 0; i < nq; ++i) {
      const int s = i % NQS;
      if (i >= NQS && !mbar_wait_bounded(&qdo_empty[s], ((i / NQS) + 1) & 1, abort_flag, a.spin_limit)) {
        watchdog_fire(kWdBwdLoad);
        break;
      }
      const int q0 = i * kBlk;
      uint8_t* qt = smem + C::kQOff + s * 2 * C::kTile;
      if (lane == 0) {
        mbar_arrive_expect_tx(&qdo_full[s], 2 * C::kTile);
        attn::load_tile<DP>(qt, &qmap, &qdo_full[s], h, q0, b);
        attn::load_tile<DP>(qt + C::kTile, &omap, &qdo_full[s], h, q0, b);
      }
      if constexpr (RES) continue;
      float* vec = reinterpret_cast<float*>(smem + C::kVecOff + s * C::kVecBytes);
      for (int r = lane; r < kBlk; r += 32) {
        const int q = q0 + r;
        vec[r] = q < a.S ? __ldg(lse_bh + q) : 0.f;
        vec[128 + r] = q < a.S ? __ldg(del_bh + q) : 0.f;
      }
      // slab[t] = pd[h, k0 - q0 - 127 + t + S - 1] * log2e for t in [0, 255)
      const int base = k0 - q0 - (kBlk - 1) + a.S - 1;
      for (int t = lane; t < 256; t += 32) {
        const int pos = base + t;
        vec[256 + t] = (t < kDiag && pos >= 0 && pos < two_s) ? __ldg(pdh + pos) * kLog2e : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&qdo_full[s]);
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ resident rows (RES)
    if constexpr (RES) {
      const int tid = threadIdx.x - 64;
      const int two_s = 2 * a.S - 1;
      attn::fill_row(pd_row, (int)pd_row_floats(a.S), kRowPad, a.pd + (size_t)h * two_s, two_s, kLog2e, tid, 64);
      attn::fill_row(lse_row, (int)vec_row_floats(a.S), 0, a.lse + (size_t)bh * a.S, a.S, 1.f, tid, 64);
      attn::fill_row(del_row, (int)vec_row_floats(a.S), 0, a.delta + (size_t)bh * a.S, a.S, 1.f, tid, 64);
      mbar_arrive(row_full);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = F16 ? 0u : 1u;
      constexpr uint32_t id_sq = idesc_f16(128, kBlk, fmt, false, false);   // S^T, dP^T: K-major, N = 128
      constexpr uint32_t id_nd = idesc_f16(128, DP, fmt, false, true);      // dV, dK: B MN-major, N = DP
      constexpr uint32_t id_dq = idesc_f16(128, DP, fmt, true, true);       // dQ: A (dS) and B MN-major
      // Precomputed descriptors (see relpos_attn_fwd.cu): issue = constant add + MMA.
      const uint64_t k_kd = attn::kmajor_base(smem_u32(smem + C::kKOff));
      const uint64_t v_kd = attn::kmajor_base(smem_u32(smem + C::kVOff));
      const uint64_t k_mn = attn::mnmajor_base(smem_u32(smem + C::kKOff));
      const uint64_t q_kd0 = attn::kmajor_base(smem_u32(smem + C::kQOff));
      const uint64_t o_kd0 = attn::kmajor_base(smem_u32(smem + C::kQOff + C::kTile));
      const uint64_t q_mn0 = attn::mnmajor_base(smem_u32(smem + C::kQOff));
      const uint64_t o_mn0 = attn::mnmajor_base(smem_u32(smem + C::kQOff + C::kTile));
      // dS: [128 queries x 128 keys] MN-major, 128B swizzle, two 64-query atoms 16 KB apart
      const uint64_t ds_d = smem_desc(smem_u32(smem + C::kDSOff), 16384, 1024, kSw128);
      constexpr uint64_t kStage = (2 * C::kTile) >> 4;
      constexpr uint64_t kDsRows = (16 * 128) >> 4;   // next 16 keys of dS
      bool ok = mbar_wait_bounded(kv_full, 0, abort_flag, a.spin_limit);
      for (int i = 0; i < nq && ok; ++i) {
        const int s = i % NQS;
        const uint64_t so = (uint64_t)s * kStage;
        if (!mbar_wait_bounded(&qdo_full[s], (i / NQS) & 1, abort_flag, a.spin_limit)) { ok = false; break; }
        tc_fence_after();
        // S^T = K Q^T and dP^T = V dO^T (rows = keys)
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          mma_ss(tmem + C::kST, k_kd + kk * attn::kKSliceStep, q_kd0 + so + kk * attn::kKSliceStep, id_sq, kk > 0);
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          mma_ss(tmem + C::kDPT, v_kd + kk * attn::kKSliceStep, o_kd0 + so + kk * attn::kKSliceStep, id_sq, kk > 0);
        mma_commit(sdp_ready);
        const uint32_t acc0 = i > 0 ? 1u : 0u;
        // dV += P^T dO
        if (!mbar_wait_bounded(p_ready, i & 1, abort_flag, a.spin_limit)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          mma_ts(tmem + C::kDV, tmem + C::kST + kk * 8, o_mn0 + so + kk * attn::kKRowStep, id_nd, kk > 0 ? 1u : acc0);
        // dK += dS^T Q, then dQ = dS K (dQ's TMEM columns must have been drained)
        if (!mbar_wait_bounded(ds_ready, i & 1, abort_flag, a.spin_limit)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          mma_ts(tmem + C::kDK, tmem + C::kDPT + kk * 8, q_mn0 + so + kk * attn::kKRowStep, id_nd, kk > 0 ? 1u : acc0);
        if (i > 0 && !mbar_wait_bounded(dq_free, (i - 1) & 1, abort_flag, a.spin_limit)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          mma_ss(tmem + C::kDQ, ds_d + kk * kDsRows, k_mn + kk * attn::kKRowStep, id_dq, kk > 0 ? 1u : 0u);
        mma_commit(dq_ready);
        mma_commit(&qdo_empty[s]);
      }
      if (ok) mma_commit(kdv_done);
      else watchdog_fire(kWdBwdMma);
      // Drain: every MMA issued above has completed before TMEM is released.
      mma_commit(drain);
      for (uint32_t it = 0; it < a.spin_limit && !mbar_try_wait(drain, 0); ++it) {
      }
    }
  }
  } else if (warp < 8) {
    regs_inc<kRegsCompute>();
    // ------------------------------------------------------------ compute WG: one key per thread
    const int quarter = warp % 4;
    const int kr = quarter * 32 + lane;        // key row within the block (TMEM lane)
    const int key = k0 + kr;
    const bool key_ok = key < a.S;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t st_t = tmem + lane_addr + C::kST;
    const uint32_t dpt_t = tmem + lane_addr + C::kDPT;
    uint8_t* ds_smem = smem + C::kDSOff;
    // dBias: this warp's 32 keys x 128 queries of dS touch 159 diagonals ("bins"): bin j holds
    // key - query = 32 * quarter + 31 - j within the tile.  Each 32 x 32 sub-tile is transposed
    // along its diagonals by 32 independent shuffles (lane l reads dS[(l + m) & 31][m]), so lane l
    // owns bins 31 - l + 32 k (k = 0..4) and sums them in registers in a fixed order:
    // deterministic, no atomics, no serial chain.
    bool ok = !RES || __all_sync(0xffffffffu, mbar_wait_bounded(row_full, 0, abort_flag, a.spin_limit));
    for (int i = 0; i < nq && ok; ++i) {
      const int s = i % NQS;
      const int q0 = i * kBlk;
      const bool w_ok = mbar_wait_bounded(sdp_ready, i & 1, abort_flag, a.spin_limit) &&
                        (RES || mbar_wait_bounded(&qdo_full[s], (i / NQS) & 1, abort_flag, a.spin_limit));
      if (!__all_sync(0xffffffffu, w_ok)) {   // warp-uniform: TMEM ops below are warp-collective
        ok = false;
        break;
      }
      tc_fence_after();
      const float* vec = reinterpret_cast<const float*>(smem + C::kVecOff + s * C::kVecBytes);
      const float* lse_p = RES ? lse_row + q0 : vec;
      const float* del_p = RES ? del_row + q0 : vec + 128;
      // bias(key, q0 + q) = slab[-q]
      const float* slab = RES ? pd_row + kRowPad + key - q0 + a.S - 1 : vec + 256 + kr + (kBlk - 1);
      const int qvalid = a.S - q0;
      float p[kBlk];
      {
        uint32_t* u = reinterpret_cast<uint32_t*>(p);
#pragma unroll
        for (int c = 0; c < kBlk; c += 32) tmem_ld32(st_t + c, u + c);
        tmem_wait_ld();
      }
      // P^T = exp2(s2 - lse), zero outside the sequence; bf16/f16 copy over S^T in TMEM
#pragma unroll
      for (int qc = 0; qc < kBlk / 32; ++qc) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int q = qc * 32 + e;
          const float s2 = fmaf(p[q], a.scale_log2, slab[-q]) - lse_p[q];
          p[q] = (key_ok && q < qvalid) ? ex2_approx(s2) : 0.f;
          if (e & 1) pk[e / 2] = F16 ? pack_f16x2(p[q - 1], p[q]) : pack_bf16x2(p[q - 1], p[q]);
        }
        tmem_st16(st_t + qc * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_ready);

      // dS^T = P^T (dP^T - delta), 32 queries at a time, into TMEM (dK MMA), smem (dQ MMA)
      // and the diagonal registers (dBias)
      float dbin[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int qc = 0; qc < kBlk / 32; ++qc) {
        uint32_t dsv[32];
        tmem_ld32(dpt_t + qc * 32, dsv);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int q = qc * 32 + e;
          dsv[e] = __float_as_uint(p[q] * (__uint_as_float(dsv[e]) - del_p[q]));
        }
        uint32_t dk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          dk[e] = F16 ? pack_f16x2(__uint_as_float(dsv[2 * e]), __uint_as_float(dsv[2 * e + 1]))
                      : pack_bf16x2(__uint_as_float(dsv[2 * e]), __uint_as_float(dsv[2 * e + 1]));
        tmem_st16(dpt_t + qc * 16, dk);
        // smem copy for the dQ MMA: row kr of 64-query atom (qc/2), 16-byte chunks (qc%2)*4..+3
        uint8_t* row = ds_smem + (qc / 2) * 16384 + kr * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = (qc % 2) * 4 + u;
          *reinterpret_cast<uint4*>(row + ((chunk ^ (kr & 7)) << 4)) =
              make_uint4(dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
        }
        // diagonal transpose of this 32 x 32 sub-tile: m < 32 - lane stays on diagonal +lane
        float hi = 0.f, lo = 0.f;
#pragma unroll
        for (int m = 0; m < 32; ++m) {
          const float x = __shfl_sync(0xffffffffu, __uint_as_float(dsv[m]), (lane + m) & 31);
          if (m < 32 - lane) hi += x;
          else lo += x;
        }
        dbin[qc] += hi;
        dbin[qc + 1] += lo;
      }
      tmem_wait_st();
      fence_async_shared();   // dS smem writes -> visible to the MMA (async proxy)
      tc_fence_before();
      mbar_arrive(ds_ready);
      // this tile's diagonal sums: lane owns bins 31 - lane + 32 k
      float* out = a.dbias_part + ((((size_t)bh * a.n_blk + kb) * a.n_blk + i) * 4 + quarter) * kBins;
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const int bin = 31 - lane + 32 * k;
        if (bin < kBins) out[bin] = dbin[k];
      }
    }
    if (!ok) watchdog_fire(kWdBwdCompute);
  } else {
    regs_dec<kRegsDq>();
    // ------------------------------------------------------------ dQ WG: one query row per thread
    const int quarter = warp % 4;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t dq_t = tmem + lane_addr + C::kDQ;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(dq_ready, i & 1, abort_flag, a.spin_limit))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[DP];
      {
        uint32_t* u = reinterpret_cast<uint32_t*>(v);
#pragma unroll
        for (int c = 0; c < DP; c += 16) tmem_ld16(dq_t + c, u + c);
        tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(dq_free);
      const int q = i * kBlk + r;
      if (q < a.S) {
        float* dst = a.dq_acc + ((size_t)b * a.S + q) * ((size_t)a.H * a.D) + (size_t)h * a.D;
#pragma unroll
        for (int c = 0; c < DP; c += 4)
          if (c < a.D) red_add_v4(dst + c, v[c], v[c + 1], v[c + 2], v[c + 3]);
      }
    }
    // dK, dV (rows = keys) -> dqkv
    if (ok && !__all_sync(0xffffffffu, mbar_wait_bounded(kdv_done, 0, abort_flag, a.spin_limit))) ok = false;
    if (!ok) {
      watchdog_fire(kWdBwdDq);
    } else {
      tc_fence_after();
      using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
      const int key = k0 + r;
      const bool row_ok = key < a.S;
      T* base = reinterpret_cast<T*>(a.dqkv) + ((size_t)b * a.S + (row_ok ? key : 0)) * a.dqkv_stride;
#pragma unroll
      for (int which = 0; which < 2; ++which) {   // 0: dK (scaled), 1: dV
        const uint32_t src = tmem + lane_addr + (which == 0 ? C::kDK : C::kDV);
        T* dst = base + (size_t)(1 + which) * a.H * a.D + (size_t)h * a.D;
        const float mul = which == 0 ? a.scale : 1.f;
#pragma unroll
        for (int c = 0; c < DP; c += 16) {
          uint32_t u[16];
          tmem_ld16(src + c, u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 8) {
            if (row_ok && c + e < a.D) {
              uint4 pk;
              float f[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) f[k] = __uint_as_float(u[e + k]) * mul;
              if (F16)
                pk = make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]),
                                pack_f16x2(f[6], f[7]));
              else
                pk = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                                pack_bf16x2(f[6], f[7]));
              *reinterpret_cast<uint4*>(dst + c + e) = pk;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// delta[b*H + h, s] = sum_d dO * O32; zero the dQ accumulator.  One thread per (token, head).
template <bool F16>
__global__ void __launch_bounds__(256)
relpos_bwd_prep_kernel(const void* __restrict__ dout, const float* __restrict__ out32, float* __restrict__ delta,
                       float* __restrict__ dq_acc, int B, int S, int H, int D) {
  using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // token * H + head
  if (idx >= (int64_t)B * S * H) return;
  const int64_t tok = idx / H;
  const int hh = (int)(idx % H);
  const size_t off = (size_t)tok * H * D + (size_t)hh * D;
  const T* g = reinterpret_cast<const T*>(dout) + off;
  const float* o = out32 + off;
  float* z = dq_acc + off;
  float acc = 0.f;
  for (int d = 0; d < D; d += 8) {
    const uint4 gv = *reinterpret_cast<const uint4*>(g + d);
    const float4 o0 = *reinterpret_cast<const float4*>(o + d);
    const float4 o1 = *reinterpret_cast<const float4*>(o + d + 4);
    const T* gt = reinterpret_cast<const T*>(&gv);
    float gf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) gf[k] = F16 ? __half2float(*reinterpret_cast<const __half*>(&gt[k]))
                                            : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&gt[k]));
    acc += gf[0] * o0.x + gf[1] * o0.y + gf[2] * o0.z + gf[3] * o0.w;
    acc += gf[4] * o1.x + gf[5] * o1.y + gf[6] * o1.z + gf[7] * o1.w;
    *reinterpret_cast<float4*>(z + d) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(z + d + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int b = (int)(tok / S), s = (int)(tok % S);
  delta[((size_t)b * H + hh) * S + s] = acc;
}

// dqkv[:, q section] = dQ accumulator * scale, rounded to the input dtype.
template <bool F16>
__global__ void __launch_bounds__(256)
relpos_bwd_dq_kernel(const float* __restrict__ dq_acc, void* __restrict__ dqkv, int64_t dqkv_stride, int64_t rows,
                     int HD, float scale) {
  using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
  const int64_t per_row = HD / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const int64_t row = idx / per_row, c = (idx % per_row) * 8;
  const float4 a0 = *reinterpret_cast<const float4*>(dq_acc + row * HD + c);
  const float4 a1 = *reinterpret_cast<const float4*>(dq_acc + row * HD + c + 4);
  uint4 pk;
  if (F16)
    pk = make_uint4(sm100::pack_f16x2(a0.x * scale, a0.y * scale), sm100::pack_f16x2(a0.z * scale, a0.w * scale),
                    sm100::pack_f16x2(a1.x * scale, a1.y * scale), sm100::pack_f16x2(a1.z * scale, a1.w * scale));
  else
    pk = make_uint4(sm100::pack_bf16x2(a0.x * scale, a0.y * scale), sm100::pack_bf16x2(a0.z * scale, a0.w * scale),
                    sm100::pack_bf16x2(a1.x * scale, a1.y * scale), sm100::pack_bf16x2(a1.z * scale, a1.w * scale));
  *reinterpret_cast<uint4*>(reinterpret_cast<T*>(dqkv) + row * dqkv_stride + c) = pk;
}

// dpd[h, t] = sum over b, over the tiles (kb, qb) whose diagonal range covers g = t - (S-1) =
// key - query, and over the four key-quarter warps of each tile, of the bin holding g.  A tile at
// offset d = kb - qb holds diagonal e = g - 128 d of quarter w in bin 31 - e + 32 w.  Fixed order:
// deterministic.
__global__ void __launch_bounds__(256)
relpos_bwd_dpd_kernel(const float* __restrict__ part, float* __restrict__ dpd, int B, int S, int H, int nb) {
  const int h = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= 2 * S - 1) return;
  const int g = t - (S - 1);
  const int d_hi = (g + 127) >= 0 ? (g + 127) / 128 : -((-(g + 127) + 127) / 128);
  float acc = 0.f;
  for (int bb = 0; bb < B; ++bb) {
    const float* pb = part + (size_t)(bb * H + h) * nb * nb * 4 * kBins;
    for (int d = d_hi; d >= d_hi - 1; --d) {
      const int e = g - 128 * d;
      if (e < -(kBlk - 1) || e > kBlk - 1) continue;
      const int kb_lo = d > 0 ? d : 0, kb_hi = d > 0 ? nb : nb + d;   // qb = kb - d in [0, nb)
      for (int kbi = kb_lo; kbi < kb_hi; ++kbi) {
        const float* tile = pb + ((size_t)kbi * nb + (kbi - d)) * 4 * kBins;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int j = 31 - e + 32 * w;
          if (j >= 0 && j < kBlk + 31) acc += tile[w * kBins + j];
        }
      }
    }
  }
  dpd[(size_t)h * (2 * S - 1) + t] = acc;
}

struct WsLayout {
  size_t delta, dq, part, total;
};

inline WsLayout ws_layout(int64_t B, int64_t S, int64_t H, int64_t D) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const int64_t nb = (S + kBlk - 1) / kBlk;
  WsLayout w;
  w.delta = 0;
  w.dq = up((size_t)B * H * S * 4);
  w.part = w.dq + up((size_t)B * S * H * D * 4);
  w.total = w.part + up((size_t)B * H * nb * nb * 4 * kBins * 4);
  return w;
}

template <int DP, bool F16>
int launch_bwd(const CUtensorMap& qm, const CUtensorMap& om, const BwdArgs& a, const void* dout,
               const float* out32, float* dpd, cudaStream_t stream) {
  using C = BwdCfg<DP>;
  const int64_t tokens_heads = (int64_t)a.B * a.S * a.H;
  relpos_bwd_prep_kernel<F16><<<(unsigned)((tokens_heads + 255) / 256), 256, 0, stream>>>(
      dout, out32, const_cast<float*>(a.delta), a.dq_acc, a.B, a.S, a.H, a.D);
  KRSI_LAUNCH_CHECK();
  const size_t res_smem = C::kSmem + (size_t)rows_bytes(a.S);
  const bool res = res_smem <= 232448;   // 227 KB per CTA on sm_100
  auto kern = res ? relpos_bwd_main_kernel<DP, F16, true> : relpos_bwd_main_kernel<DP, F16, false>;
  const size_t smem = res ? res_smem : C::kSmem;
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<dim3(a.n_blk, a.B * a.H), kThreads, smem, stream>>>(qm, om, a);
  KRSI_LAUNCH_CHECK();
  const int64_t rows = (int64_t)a.B * a.S;
  const int64_t items = rows * (a.H * a.D / 8);
  relpos_bwd_dq_kernel<F16><<<(unsigned)((items + 255) / 256), 256, 0, stream>>>(a.dq_acc, a.dqkv, a.dqkv_stride,
                                                                                  rows, a.H * a.D, a.scale);
  KRSI_LAUNCH_CHECK();
  relpos_bwd_dpd_kernel<<<dim3((2 * a.S - 1 + 255) / 256, a.H), 256, 0, stream>>>(a.dbias_part, dpd, a.B, a.S, a.H,
                                                                                   a.n_blk);
  KRSI_LAUNCH_CHECK();
  return KRSI_OK;
}

template <bool F16>
int dispatch_dp(int DP, const CUtensorMap& qm, const CUtensorMap& om, const BwdArgs& a, const void* dout,
                const float* out32, float* dpd, cudaStream_t s) {
  switch (DP) {
    case 32: return launch_bwd<32, F16>(qm, om, a, dout, out32, dpd, s);
    case 64: return launch_bwd<64, F16>(qm, om, a, dout, out32, dpd, s);
    case 80: return launch_bwd<80, F16>(qm, om, a, dout, out32, dpd, s);
    default: return KRSI_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace krsi

using namespace krsi;

extern "C" int krsi_relpos_attn_bwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t D, size_t* bytes) {
  KRSI_CHECK_ARG(B >= 0 && S >= 0 && H > 0 && D > 0 && bytes);
  *bytes = ws_layout(B, S, H, D).total;
  return KRSI_OK;
}

extern "C" int krsi_relpos_attn_bwd(const void* dout, const void* qkv, int64_t qkv_row_stride, const float* pd,
                                    const float* out32, const float* lse, void* dqkv, int64_t dqkv_row_stride,
                                    float* dpd, void* workspace, size_t workspace_bytes, int64_t B, int64_t S,
                                    int64_t H, int64_t D, float scale, int dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(B >= 0 && S >= 0 && H > 0 && D > 0);
  if (S == 0) return KRSI_OK;
  KRSI_CHECK_ARG(dpd);
  if (B == 0) {
    KRSI_CUDA_TRY(cudaMemsetAsync(dpd, 0, (size_t)H * (2 * S - 1) * sizeof(float), stream));
    return KRSI_OK;
  }
  KRSI_CHECK_ARG(dout && qkv && pd && out32 && lse && dqkv);
  if (dtype != KRSI_BF16 && dtype != KRSI_F16) return KRSI_ERR_UNSUPPORTED;
  const int DP = attn_padded_dim(D);
  if (DP < 0 || DP > 80) return KRSI_ERR_UNSUPPORTED;
  KRSI_CHECK_ARG(qkv_row_stride >= 3 * H * D && dqkv_row_stride >= 3 * H * D);
  if (qkv_row_stride % 8 || dqkv_row_stride % 8 || !aligned16(qkv) || !aligned16(dqkv) || !aligned16(dout) ||
      !aligned16(out32))
    return KRSI_ERR_MISALIGNED;
  if (S > (1 << 20) || B * H > 65535) return KRSI_ERR_UNSUPPORTED;
  const WsLayout ws = ws_layout(B, S, H, D);
  if (!workspace || workspace_bytes < ws.total || !aligned16(workspace)) return KRSI_ERR_WORKSPACE;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  CUtensorMap qm, om;
  const bool f16 = dtype == KRSI_F16;
  if (!attn::make_head_map(&qm, qkv, qkv_row_stride, B, S, 3 * H, D, f16) ||
      !attn::make_head_map(&om, dout, H * D, B, S, H, D, f16))
    return KRSI_ERR_CUDA;
  BwdArgs a{pd,
            lse,
            reinterpret_cast<float*>(w + ws.delta),
            reinterpret_cast<float*>(w + ws.dq),
            reinterpret_cast<float*>(w + ws.part),
            dqkv,
            dqkv_row_stride,
            (int)B,
            (int)S,
            (int)H,
            (int)D,
            (int)((S + kBlk - 1) / kBlk),
            scale * 1.4426950408889634f,
            scale,
            kSpinLimit};
  return f16 ? dispatch_dp<true>(DP, qm, om, a, dout, out32, dpd, stream)
             : dispatch_dp<false>(DP, qm, om, a, dout, out32, dpd, stream);
}
