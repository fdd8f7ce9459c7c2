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
//   bwd_main   one CTA per (b*H + h, 128-key block); loops over the 128-query blocks with four
//              warpgroups:
//                warp 0      TMA issuer: K and V once; Q and dO tiles per query block into a
//                            2-stage ring, as soon as the block's dK MMAs released a stage
//                warp 3      stage finisher: publishes a stage once its loads landed, with the
//                            block's -lse, -delta (and bias slab when not resident).  When D
//                            leaves padding columns (D % 16 == 8) it writes K, V = 1 and Q, dO =
//                            a three-term 16-bit split of -lse / (scale log2 e) and -delta into
//                            padding columns D..D+2, so the S^T and dP^T MMAs produce S - lse/c
//                            and dP - delta directly (no per-element lse/delta reads)
//                warp 1      TMEM owner + tcgen05.mma issuer, software-pipelined so the next
//                            block's S^T is computed while the current dS is:
//                              S^T = K Q^T, dP^T = V dO^T              (SS, K = DP)
//                              dV += P^T dO, dK += dS^T Q               (TS: P^T/dS^T in TMEM)
//                              dQ  = dS K                              (SS: dS staged in smem)
//                warps 2, 4-15 first fill the resident bias rows: a reversed window of the bias
//                            row, in two copies (the second shifted by one, for aligned pairs),
//                            while warp 3 publishes the first stage
//                warps 4-11  two compute warpgroups, one key row per thread and 64 queries per
//                            warpgroup: P^T, dS^T in paired fp32 -> 16-bit into TMEM and smem;
//                            dBias diagonal sums of the fp32 dS by a warp-shuffle transpose into
//                            per-lane register bins (no S x S buffer, no atomics); at the end dK
//                            (warpgroup 0) and dV (warpgroup 1) -> dqkv
//                warps 12-15 one query row per thread: dQ tile from TMEM -> a shared-memory tile
//                            that one TMA reduce-add sums into the fp32 accumulator
//   bwd_dq     dQ accumulator * scale -> dqkv (input dtype)
//   bwd_dpd    dpd[h, t] = fixed-order sums of the per-tile diagonal partials, per tile diagonal
//              then per output (deterministic)
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

constexpr int kBlk = 128;           // keys per CTA, queries per iteration
constexpr int kHalf = 64;           // queries per compute warpgroup
constexpr int kThreads = 512;       // 4 warpgroups: control, compute (queries 0-63, 64-127), dQ/epilogue
// setmaxnreg budgets: the launch holds 128 registers x 512 threads = 65,536, and
// 128 x (104 + 160 + 160 + 88) = 65,536 are handed out, so every increase can be satisfied.
constexpr uint32_t kRegsCtl = 104;
constexpr uint32_t kRegsCompute = 160;
constexpr uint32_t kRegsDq = 88;
constexpr int kWarpsPerTile = 8;    // dBias partial rows per tile: (query half, key quarter)
constexpr int kBins = 96;           // per-warp bins: 32 keys x 64 queries -> 95 diagonals (+1 zero)
// warps 2 and 4-15 fill the resident rows (compute warps: before their first P); warp 3 publishes
// the first Q/dO stage meanwhile, so the first S^T and dP^T are computed while the rows load
constexpr int kRowFillers = 416;
__device__ __forceinline__ int filler_id() { return (int)threadIdx.x - (threadIdx.x < 96 ? 64 : 96); }
constexpr int kCopyBank = 16;       // distance (mod 32 floats) between the two bias copies

constexpr float kLog2e = 1.4426950408889634f;

// Head dims above 80 (DP = 96, 128) do not fit dQ, dK, dV and the two score tiles in the 512 TMEM
// columns, nor two Q/dO stages next to K, V and dS in shared memory.  For them:
//   * the dQ tile accumulates in the dP^T columns: dQ_i is issued after dK_i has read dS_i there
//     (the tensor pipe runs in order), and dP_{i+1} waits until dQ_i has been read out;
//   * one Q/dO stage: the next block's S^T is issued once its loads have landed, after dK_i / dQ_i
//     (which release the stage) instead of before them;
//   * dQ is staged and reduce-added in two halves of D/2 columns (half the staging memory).
template <int DP>
struct BwdCfg {
  static constexpr bool kWide = DP > 80;
  static constexpr uint32_t kTile = attn::Tile<DP>::kBytes;
  static constexpr int NQS = kWide ? 1 : 2;                       // Q/dO stages
  static constexpr int kDqParts = kWide ? 2 : 1;                  // dQ staging / reduce-add parts
  static constexpr uint32_t kKOff = 0;
  static constexpr uint32_t kVOff = kKOff + kTile;
  static constexpr uint32_t kQOff = kVOff + kTile;                // stage s: Q at kQOff + s*2*kTile
  static constexpr uint32_t kDSOff = kQOff + NQS * 2 * kTile;     // dS (bf16, MN-major SW128): 2 x 16 KB
  static constexpr uint32_t kStgOff = kDSOff + 2 * 16384;          // dQ staging: 128 rows x D / kDqParts fp32
  // per stage: -lse[128], -delta[128] and (bias not resident) the reversed bias slab [256] with its
  // copy shifted by one element [256] placed kCopyBank (mod 32) floats after it (bank-conflict-free)
  static constexpr uint32_t kVecOff = kStgOff + kTileRows * (DP / kDqParts) * 4;
  static constexpr int kSlab0 = 256, kSlab1 = 256 + 256 + kCopyBank;
  static constexpr uint32_t kVecBytes = (kSlab1 + 256) * 4;
  static constexpr uint32_t kBarOff = kVecOff + NQS * kVecBytes;
  static constexpr int kNumBars = 1 + 3 * NQS + 13;
  static constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;
  static constexpr uint32_t kRowOff = (kMiscOff + 16 + 15) & ~15u;   // resident rows (runtime length)
  static constexpr uint32_t kSmem = kRowOff + 1024;                  // + the 1 KB alignment slack
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kST = 0, kDPT = 128, kDV = 256, kDK = 256 + DP, kDQ = kWide ? kDPT : 256 + 2 * DP;
  static_assert(kDK + DP <= kTmemCols && (kWide || kDQ + DP <= kTmemCols), "backward TMEM plan");
  static_assert(kSmem <= 232448, "backward shared memory");
};

struct BwdArgs {
  const float* pd;
  const float* lse;
  const float* delta;
  float* dq_acc;          // [B*S, H*D] fp32 (the main kernel adds into it through its tensor map)
  float* dbias_part;      // [B*H, n_kb, n_qb, kWarpsPerTile, kBins]
  float* dpd_rows;        // [H, 2 n_blk - 1, batch chunks, 256]: per tile-diagonal sums (dBias stage 1)
  void* dqkv;
  int64_t dqkv_stride;
  int B, S, H, D, n_blk;
  float scale_log2, scale;
  uint32_t spin_limit;
};

// TMEM column of the 16-bit P^T / dS^T pairs of queries [16 kk, 16 kk + 16): each compute
// warpgroup packs its 64 queries into the first 32 of its own 64 fp32 columns, so neither
// overwrites columns the other has yet to read.
__host__ __device__ constexpr uint32_t packed_col(int kk) { return kk * 8 + (kk >= kHalf / 16 ? kHalf / 2 : 0); }

// Resident bias rows (one load per CTA).  The bias of (key, query) is pd[h, key - query + S - 1]; the
// keys of CTA kb and all padded queries [0, nb*128) use m in [m_top - (nb*128 + 126), m_top] with
// m_top = k0 + 127 + S - 1.  The row stores that window reversed and scaled by log2(e):
//   rev[kRevPad + t] = pd[h, m_top - t] * log2e   (zero outside [0, 2S-2]),
// so bias(k0 + kr, q) = rev[kRevPad + 127 - kr + q] ascends with the query, and a second copy
// shifted by one element (rev1[i] = rev[i + 1]) makes every pair of queries an aligned 8-byte read.
// A thread's first pair starts at kRevPad + 127 - key_row + (even), an odd index for kRevPad = 4, so
// in a half-warp the lanes on copy 0 read 16 consecutive floats and the lanes on copy 1 the 16 floats
// just after them, shifted by the copy distance minus 16.  With the copies 16 (mod 32) floats apart
// the two halves fall on disjoint banks: one wavefront per half-warp.
constexpr int kRevPad = 4;
__host__ __device__ constexpr int64_t rev_row_floats(int64_t S) {
  return (kRevPad + ((S + kBlk - 1) / kBlk) * kBlk + kBlk + 4 + 31 - kCopyBank) / 32 * 32 + kCopyBank;
}
__host__ __device__ constexpr int64_t rows_bytes(int64_t S) { return 2 * rev_row_floats(S) * 4; }

// 16-byte chunk of padding columns [D, D + 8) of row r of a tile (D % 16 == 8: the second chunk of
// 32-byte block D / 16; the 32-byte swizzle flips the chunk on every fourth row).
__device__ __forceinline__ uint4* pad_chunk(uint8_t* tile, int D, int r) {
  return reinterpret_cast<uint4*>(tile + (D / 16) * attn::kBlockBytes + r * 32 + ((1 ^ ((r >> 2) & 1)) << 4));
}
// v as hi + mid + lo, each rounded to the 16-bit input type, in the first three columns of a chunk
template <bool F16>
__device__ __forceinline__ uint4 split3(float v) {
  auto rnd = [](float x) { return F16 ? __half2float(__float2half_rn(x)) : __bfloat162float(__float2bfloat16_rn(x)); };
  const float hi = rnd(v), r1 = v - hi, mid = rnd(r1), lo = rnd(r1 - mid);
  return F16 ? make_uint4(pack_f16x2(hi, mid), pack_f16x2(lo, 0.f), 0u, 0u)
             : make_uint4(pack_bf16x2(hi, mid), pack_bf16x2(lo, 0.f), 0u, 0u);
}

template <int DP, bool F16, bool RES, bool FOLD>
__global__ void __launch_bounds__(kThreads, 1)
relpos_bwd_main_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap omap,
                       const __grid_constant__ CUtensorMap dqmap, const __grid_constant__ CUtensorMap kvmap,
                       const BwdArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  using C = BwdCfg<DP>;
  constexpr int NQS = C::NQS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 1 + NQS;
  uint64_t* qdo_tma = bars + 1 + 2 * NQS;   // the stage's TMA loads have landed (producer waits)
  uint64_t* s_ready = bars + 1 + 3 * NQS;   // S^T of the current block in TMEM
  uint64_t* dp_ready = s_ready + 1;          // dP^T of the current block in TMEM
  uint64_t* p_ready = s_ready + 2;           // P^T written (256 compute threads)
  uint64_t* ds_ready = s_ready + 3;          // dS^T written to TMEM and smem (256)
  uint64_t* dq_ready = s_ready + 4;
  uint64_t* dq_free = s_ready + 5;
  uint64_t* kdv_done = s_ready + 6;
  uint64_t* drain = s_ready + 7;
  uint64_t* row_full = s_ready + 8;
  uint64_t* stg_free = s_ready + 9;          // dQ staging tile read by the previous reduce-add (leader)
  uint64_t* stg_full = s_ready + 10;         // dQ staging tile written (128 dQ threads)
  uint64_t* kv_stg = s_ready + 11;           // [2] dK / dV rows staged for their TMA store (128 each)
  float* rev0 = reinterpret_cast<float*>(smem + C::kRowOff);
  float* rev1 = rev0 + rev_row_floats(a.S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb = blockIdx.x, bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int k0 = kb * kBlk;
  const int nq = a.n_blk;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(&qdo_full[s], 1);   // the producer, after the TMA landed and its own writes
      mbar_init(&qdo_tma[s], 1);
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_ready, 1);
    mbar_init(dp_ready, 1);
    mbar_init(p_ready, 2 * 128);
    mbar_init(ds_ready, 2 * 128);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 128);
    mbar_init(kdv_done, 1);
    mbar_init(drain, 1);
    mbar_init(row_full, kRowFillers);
    mbar_init(stg_free, 1);
    mbar_init(stg_full, 128);
    mbar_init(&kv_stg[0], 128);
    mbar_init(&kv_stg[1], 128);
    abort_flag[0] = 0;
    abort_flag[1] = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&omap);
    prefetch_tensormap(&dqmap);
    prefetch_tensormap(&kvmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Resident bias rows, filled cooperatively by warps 2 and 4-15 (kRowFillers threads).
  auto fill_rows = [&](int tid) {
    const int two_s = 2 * a.S - 1;
    const float* pdh = a.pd + (size_t)h * two_s;
    const int m_top = k0 + kBlk - 1 + a.S - 1;
    const int n = (int)rev_row_floats(a.S);
    const int top = m_top + kRevPad;   // rev[i] = pd[top - i]
    const int lo = max(0, m_top - (nq * kBlk + kBlk - 2)), hi = min(two_s - 1, m_top);
    attn::fill_row_rev2(rev0, rev1, n, top, pdh, lo, hi, kLog2e, tid, kRowFillers);
    mbar_arrive(row_full);
  };

  // dK (scaled) or dV of key row kr, TMEM -> dqkv; run by one compute warpgroup each at the end.  The
  // rows are staged as a dense [128 x D] tile in the Q/dO stage memory (free once every MMA has
  // completed) and written by one TMA store per warpgroup: whole 144-byte head rows instead of a
  // 16-byte store per thread and row.  Rows past the sequence end are clipped by the TMA.
  auto store_dkdv = [&](const int which, const int kr, const uint32_t lane_addr) {
    using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
    T* tile = reinterpret_cast<T*>(smem + C::kQOff + which * (C::kTile * NQS));   // [128][D]
    T* row = tile + (size_t)kr * a.D;
    const uint32_t src = tmem + lane_addr + (which == 0 ? C::kDK : C::kDV);
    const float mul = which == 0 ? a.scale : 1.f;
#pragma unroll
    for (int c = 0; c < DP; c += 16) {
      uint32_t u[16];
      tmem_ld16(src + c, u);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; e += 8) {
        if (c + e < a.D) {
          float f[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) f[k] = __uint_as_float(u[e + k]) * mul;
          const uint4 pk =
              F16 ? make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]),
                               pack_f16x2(f[6], f[7]))
                  : make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                               pack_bf16x2(f[6], f[7]));
          *reinterpret_cast<uint4*>(row + c + e) = pk;
        }
      }
    }
    fence_async_shared();   // staged rows -> visible to the TMA unit
    mbar_arrive(&kv_stg[which]);
    if (kr == 0) {   // one thread per warpgroup issues the store once all 128 rows are staged
      if (mbar_wait_bounded(&kv_stg[which], 0, abort_flag, a.spin_limit)) {
        tma_store_4d(&kvmap, tile, 0, (1 + which) * a.H + h, k0, b);
        bulk_commit_group();
        bulk_wait_read_all();   // the tile must stay in place until the TMA has read it
      } else {
        watchdog_fire(kWdBwdCompute);
      }
    }
  };

  // Each role runs entirely inside the branch that sets its register budget.
  if (warp < 4) {
    regs_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // Loads K, V once, then each block's Q and dO as soon as its stage is released (no other work,
    // so a released stage is refilled at once).
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * C::kTile);
      attn::load_tile<DP>(smem + C::kKOff, &qmap, kv_full, a.H + h, k0, b);
      attn::load_tile<DP>(smem + C::kVOff, &qmap, kv_full, 2 * a.H + h, k0, b);
      for (int i = 0; i < nq; ++i) {
        const int s = i % NQS;
        if (i >= NQS && !mbar_wait_bounded(&qdo_empty[s], ((i / NQS) + 1) & 1, abort_flag, a.spin_limit)) {
          watchdog_fire(kWdBwdLoad);
          break;
        }
        uint8_t* qt = smem + C::kQOff + s * 2 * C::kTile;
        mbar_arrive_expect_tx(&qdo_tma[s], 2 * C::kTile);
        attn::load_tile<DP>(qt, &qmap, &qdo_tma[s], h, i * kBlk, b);
        attn::load_tile<DP>(qt + C::kTile, &omap, &qdo_tma[s], h, i * kBlk, b);
      }
    }
  } else if (warp == 2) {
    if constexpr (RES) fill_rows(filler_id());
  } else if (warp == 3) {
    // ------------------------------------------------------------ stage finisher
    // Publishes each stage once its TMA loads have landed, after writing the block's per-query
    // vectors (unfolded) or the padding columns (folded) and, when the bias row is not resident,
    // the block's bias slab.
    const int two_s = 2 * a.S - 1;
    const float* pdh = a.pd + (size_t)h * two_s;
    const float* lse_bh = a.lse + (size_t)bh * a.S;
    const float* del_bh = a.delta + (size_t)bh * a.S;
    // A block's vectors are fetched into registers one block ahead, so filling a stage never
    // waits on global memory: -lse and -delta (zero past S) and, when the bias row is not
    // resident, slab[t] = pd[h, k0 - q0 + 127 - t + S - 1] * log2e for t in [0, 255) (so that
    // bias(k0 + kr, q0 + q) = slab[127 - kr + q]) with its copy slab1[t] = slab[t + 1].
    float nl[4], nd[4], sl0[8], sl1[8];
    auto fetch = [&](int blk) {
      const int q0 = blk * kBlk;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int q = q0 + lane + 32 * k;
        nl[k] = q < a.S ? -__ldg(lse_bh + q) : 0.f;
        nd[k] = q < a.S ? -__ldg(del_bh + q) : 0.f;
      }
      if constexpr (!RES) {
        const int top = k0 - q0 + kBlk - 1 + a.S - 1;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int tt = lane + 32 * k, pos = top - tt;
          sl0[k] = (tt < 2 * kBlk - 1 && pos >= 0 && pos < two_s) ? __ldg(pdh + pos) * kLog2e : 0.f;
          sl1[k] = (tt + 1 < 2 * kBlk - 1 && pos - 1 >= 0 && pos - 1 < two_s) ? __ldg(pdh + pos - 1) * kLog2e : 0.f;
        }
      }
    };
    const float inv_c = 1.f / a.scale_log2;   // Q padding carries -lse / (scale log2 e)
    fetch(0);
    for (int i = 0; i < nq; ++i) {
      const int s = i % NQS;
      uint8_t* qt = smem + C::kQOff + s * 2 * C::kTile;
      float* vec = reinterpret_cast<float*>(smem + C::kVecOff + s * C::kVecBytes);
      // the vectors and slab live outside the TMA tiles and the stage is free (its previous
      // block's readers finished before the producer reloaded it): write them before the wait
      if (!__all_sync(0xffffffffu, i < NQS || mbar_wait_bounded(&qdo_empty[s], ((i / NQS) + 1) & 1, abort_flag,
                                                                 a.spin_limit))) {
        watchdog_fire(kWdBwdLoad);
        break;
      }
      if constexpr (!FOLD) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          vec[lane + 32 * k] = nl[k];
          vec[128 + lane + 32 * k] = nd[k];
        }
      }
      if constexpr (!RES) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          vec[C::kSlab0 + lane + 32 * k] = sl0[k];
          vec[C::kSlab1 + lane + 32 * k] = sl1[k];
        }
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&qdo_tma[s], (i / NQS) & 1, abort_flag, a.spin_limit))) {
        watchdog_fire(kWdBwdLoad);
        break;
      }
      if constexpr (FOLD) {
        if (i == 0) {   // K and V: ones in the three padding columns (once; they stay resident)
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(kv_full, 0, abort_flag, a.spin_limit))) {
            watchdog_fire(kWdBwdLoad);
            break;
          }
          const uint32_t one2 = F16 ? pack_f16x2(1.f, 1.f) : pack_bf16x2(1.f, 1.f);
          const uint32_t one1 = F16 ? pack_f16x2(1.f, 0.f) : pack_bf16x2(1.f, 0.f);
          const uint4 one3 = make_uint4(one2, one1, 0u, 0u);   // 1 in columns D, D+1, D+2
          for (int r = lane; r < kBlk; r += 32) {
            *pad_chunk(smem + C::kKOff, a.D, r) = one3;
            *pad_chunk(smem + C::kVOff, a.D, r) = one3;
          }
        }
        // over the TMA's zero fill of the padding columns
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int r = lane + 32 * k;
          *pad_chunk(qt, a.D, r) = split3<F16>(nl[k] * inv_c);
          *pad_chunk(qt + C::kTile, a.D, r) = split3<F16>(nd[k]);
        }
        fence_async_shared();   // generic writes to MMA operands -> visible to the async proxy
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&qdo_full[s]);
      if (i + 1 < nq) fetch(i + 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the issue loop (warp-uniform descriptors); one elected lane issues.
    {
      auto wait_all = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.spin_limit));
      };
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
      auto issue_s = [&](int s) {        // S^T = K Q^T (rows = keys)
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          mma_ss_e(tmem + C::kST, k_kd + kk * attn::kKSliceStep, q_kd0 + s * kStage + kk * attn::kKSliceStep, id_sq,
                 kk > 0);
      };
      auto issue_dp = [&](int s) {       // dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          mma_ss_e(tmem + C::kDPT, v_kd + kk * attn::kKSliceStep, o_kd0 + s * kStage + kk * attn::kKSliceStep, id_sq,
                 kk > 0);
      };
      // Order per block i (in-order tensor pipe, so every overwrite follows the reads before it):
      //   [P_i] dV_i, S_{i+1} -> s_ready   [dS_i] dK_i, dQ_i, dP_{i+1} -> dp_ready
      bool ok = wait_all(kv_full, 0) &&
                wait_all(&qdo_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        mma_commit_e(s_ready);
        issue_dp(0);
        mma_commit_e(dp_ready);
      }
      for (int i = 0; i < nq && ok; ++i) {
        const int s = i % NQS, s1 = (i + 1) % NQS;
        const uint64_t so = (uint64_t)s * kStage;
        const uint32_t acc0 = i > 0 ? 1u : 0u;
        const bool next = i + 1 < nq;
        auto next_s = [&]() {   // the next block's S^T, once its Q and dO have landed
          if (!wait_all(&qdo_full[s1], ((i + 1) / NQS) & 1)) return false;
          tc_fence_after();
          issue_s(s1);
          mma_commit_e(s_ready);
          return true;
        };
        // dV += P^T dO, then (two stages) the next block's S^T
        if (!wait_all(p_ready, i & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          mma_ts_e(tmem + C::kDV, tmem + C::kST + packed_col(kk), o_mn0 + so + kk * attn::kKRowStep, id_nd, kk > 0 ? 1u : acc0);
        if (NQS > 1 && next && !next_s()) { ok = false; break; }
        // dK += dS^T Q, dQ = dS K (dQ's TMEM columns drained), then the next block's dP^T
        if (!wait_all(ds_ready, i & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          mma_ts_e(tmem + C::kDK, tmem + C::kDPT + packed_col(kk), q_mn0 + so + kk * attn::kKRowStep, id_nd, kk > 0 ? 1u : acc0);
        mma_commit_e(&qdo_empty[s]);   // Q and dO of this block are no longer read (dQ uses dS and K)
        if (i > 0 && !wait_all(dq_free, (i - 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          mma_ss_e(tmem + C::kDQ, ds_d + kk * kDsRows, k_mn + kk * attn::kKRowStep, id_dq, kk > 0 ? 1u : 0u);
        mma_commit_e(dq_ready);
        if (next) {
          if (NQS == 1 && !next_s()) { ok = false; break; }
          // wide heads: dQ_i sits in the dP^T columns until the dQ warps have read it out
          if (C::kWide && !wait_all(dq_free, i & 1)) { ok = false; break; }
          tc_fence_after();
          issue_dp(s1);
          mma_commit_e(dp_ready);
        }
      }
      if (ok) mma_commit_e(kdv_done);
      else watchdog_fire(kWdBwdMma);
      // Drain: every MMA issued above has completed before TMEM is released.
      mma_commit_e(drain);
      for (uint32_t it = 0; it < a.spin_limit && !mbar_try_wait(drain, 0); ++it) {
      }
    }
  }
  } else if (warp < 12) {
    regs_inc<kRegsCompute>();
    if constexpr (RES) fill_rows(filler_id());
    // ------------------------------------------------------------ compute: one key x 64 queries per thread
    const int quarter = warp % 4, half = (warp - 4) / 4;
    const int kr = quarter * 32 + lane;        // key row within the block (TMEM lane)
    const int qh = half * kHalf;               // first query of this warpgroup within the block
    const bool key_ok = k0 + kr < a.S;
    const bool keys_full = k0 + kBlk <= a.S;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t st_t = tmem + lane_addr + C::kST;
    const uint32_t dpt_t = tmem + lane_addr + C::kDPT;
    uint8_t* ds_row = smem + C::kDSOff + half * 16384 + kr * 128;   // this key's row of the dS atom
    const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
    // dBias: this warp's 32 keys x 64 queries of dS touch 95 diagonals ("bins"): bin j holds
    // key - query = 32 * quarter - 64 * half + 31 - j within the tile.  Each 32 x 32 sub-tile is
    // transposed along its diagonals by 32 independent shuffles (lane l reads dS[(l + m) & 31][m]),
    // so lane l owns bins 31 - l + 32 k (k = 0..2) and sums them in registers in a fixed order:
    // deterministic, no atomics, no serial chain.
    bool ok = !RES || __all_sync(0xffffffffu, mbar_wait_bounded(row_full, 0, abort_flag, a.spin_limit));
    for (int i = 0; i < nq && ok; ++i) {
      const int s = i % NQS;
      const int q0 = i * kBlk;
      const bool w_ok = mbar_wait_bounded(s_ready, i & 1, abort_flag, a.spin_limit) &&
                        mbar_wait_bounded(&qdo_full[s], (i / NQS) & 1, abort_flag, a.spin_limit);
      if (!__all_sync(0xffffffffu, w_ok)) {   // warp-uniform: TMEM ops below are warp-collective
        ok = false;
        break;
      }
      tc_fence_after();
      const float* vec = reinterpret_cast<const float*>(smem + C::kVecOff + s * C::kVecBytes);
      const ulonglong2* nlse2 = reinterpret_cast<const ulonglong2*>(vec + qh);
      const ulonglong2* ndel2 = reinterpret_cast<const ulonglong2*>(vec + 128 + qh);
      // bias(key, q0 + qh + q) = bq[q], read as aligned pairs from whichever copy makes them aligned
      const int bbase = RES ? kRevPad + kBlk - 1 - kr + q0 + qh : kBlk - 1 - kr + qh;
      const float* c0 = RES ? rev0 : vec + C::kSlab0;
      const float* c1 = RES ? rev1 : vec + C::kSlab1;
      const uint64_t* bq2 = reinterpret_cast<const uint64_t*>((bbase & 1) ? c1 + bbase - 1 : c0 + bbase);
      const bool full = keys_full && q0 + kBlk <= a.S;
      const int qvalid = a.S - q0 - qh;        // queries of this warpgroup inside the sequence

      // P^T = exp2(s2 - lse) in paired fp32, 32 queries at a time (bounded register use), exp2 on
      // the SFU (measured faster here than moving a share to the FMA pipe); 16-bit copy over S^T
      uint64_t p2[kHalf / 2];
#pragma unroll
      for (int qc = 0; qc < kHalf / 32; ++qc) {
        uint32_t u[32];
        tmem_ld32(st_t + qh + qc * 32, u);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const ulonglong2 nl = FOLD ? ulonglong2{} : nlse2[qc * 8 + j];
#pragma unroll
          for (int tq = 0; tq < 2; ++tq) {
            const int e = 2 * j + tq;      // pair within the chunk: queries 2e, 2e + 1
            const int pe = qc * 16 + e;    // pair within this warpgroup's 64 queries
            uint64_t x = f2_fma(f2_pack(__uint_as_float(u[2 * e]), __uint_as_float(u[2 * e + 1])), scale2, bq2[pe]);
            if constexpr (!FOLD) x = f2_add(x, tq ? nl.y : nl.x);
            float x0, x1, y0, y1;
            f2_unpack(x, x0, x1);
            y0 = ex2_approx(x0);
            y1 = ex2_approx(x1);
            if (!full) {
              y0 = (key_ok && 2 * pe < qvalid) ? y0 : 0.f;
              y1 = (key_ok && 2 * pe + 1 < qvalid) ? y1 : 0.f;
            }
            p2[pe] = f2_pack(y0, y1);
            pk[e] = F16 ? pack_f16x2(y0, y1) : pack_bf16x2(y0, y1);
          }
        }
        // packed into this warpgroup's own columns, which it has already read
        tmem_st16(st_t + qh + qc * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_ready);

      // dS^T = P^T (dP^T - delta), 32 queries at a time, into TMEM (dK MMA), smem (dQ MMA)
      // and the diagonal registers (dBias)
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(dp_ready, i & 1, abort_flag, a.spin_limit))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float dbin[3] = {0.f, 0.f, 0.f};
#pragma unroll
      for (int qc = 0; qc < kHalf / 32; ++qc) {
        uint32_t dsv[32];
        tmem_ld32(dpt_t + qh + qc * 32, dsv);
        tmem_wait_ld();
        uint32_t dk[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const ulonglong2 nd = FOLD ? ulonglong2{} : ndel2[qc * 8 + j];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int e = 2 * j + t;     // pair within the chunk
            const uint64_t dp = f2_pack(__uint_as_float(dsv[2 * e]), __uint_as_float(dsv[2 * e + 1]));
            const uint64_t d = f2_mul(p2[qc * 16 + e], FOLD ? dp : f2_add(dp, t ? nd.y : nd.x));
            float d0, d1;
            f2_unpack(d, d0, d1);
            dsv[2 * e] = __float_as_uint(d0);
            dsv[2 * e + 1] = __float_as_uint(d1);
            dk[e] = F16 ? pack_f16x2(d0, d1) : pack_bf16x2(d0, d1);
          }
        }
        tmem_st16(dpt_t + qh + qc * 16, dk);
        // smem copy for the dQ MMA: row kr of atom `half`, 16-byte chunks qc*4 .. qc*4+3
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = qc * 4 + u;
          *reinterpret_cast<uint4*>(ds_row + ((chunk ^ (kr & 7)) << 4)) =
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
      float* out = a.dbias_part +
                   ((((size_t)bh * a.n_blk + kb) * a.n_blk + i) * kWarpsPerTile + half * 4 + quarter) * kBins;
#pragma unroll
      for (int k = 0; k < 3; ++k) out[31 - lane + 32 * k] = dbin[k];
    }
    // dK (warpgroup 0) or dV (warpgroup 1) of this key row -> dqkv, while warps 12-15 drain the
    // last dQ tile
    if (ok && !__all_sync(0xffffffffu, mbar_wait_bounded(kdv_done, 0, abort_flag, a.spin_limit))) ok = false;
    if (!ok) {
      watchdog_fire(kWdBwdCompute);
    } else {
      tc_fence_after();
      store_dkdv(half, kr, lane_addr);
    }
  } else {
    regs_dec<kRegsDq>();
    if constexpr (RES) fill_rows(filler_id());
    // ------------------------------------------------------------ dQ WG: one query row per thread
    const int quarter = warp % 4;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t dq_t = tmem + lane_addr + C::kDQ;
    const bool leader = threadIdx.x == 3 * 128;
    const int pc = a.D / C::kDqParts;                 // columns per staged part (a multiple of 4)
    float* stg_row = reinterpret_cast<float*>(smem + C::kStgOff) + (size_t)r * pc;   // pitch pc floats
    bool ok = true;
    for (int i = 0; i < nq && ok; ++i) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(dq_ready, i & 1, abort_flag, a.spin_limit))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int part = 0; part < C::kDqParts; ++part) {
        const uint32_t ph = (uint32_t)(i * C::kDqParts + part) & 1u;
        // the staging tile is free once the previous reduce-add has read it (mbarriers, not
        // bar.sync, so that every wait stays bounded)
        if (leader) {
          bulk_wait_read_all();
          mbar_arrive(stg_free);
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(stg_free, ph, abort_flag, a.spin_limit))) {
          ok = false;
          break;
        }
        const int lo = part * pc, hi = lo + pc;
#pragma unroll
        for (int c = 0; c < DP; c += 16) {
          if (c + 16 <= lo || c >= hi) continue;   // warp-uniform
          uint32_t u[16];
          tmem_ld16(dq_t + c, u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            if (c + e >= lo && c + e < hi)
              *reinterpret_cast<uint4*>(stg_row + c + e - lo) = make_uint4(u[e], u[e + 1], u[e + 2], u[e + 3]);
        }
        if (part == C::kDqParts - 1) {   // every column of this dQ tile has left TMEM
          tc_fence_before();
          mbar_arrive(dq_free);
        }
        fence_async_shared();   // staging writes -> visible to the TMA unit
        mbar_arrive(stg_full);
        if (leader) {
          if (!mbar_wait_bounded(stg_full, ph, abort_flag, a.spin_limit)) {
            ok = false;
          } else {
            tma_reduce_add_3d(&dqmap, smem + C::kStgOff, h * a.D + lo, i * kBlk, b);
            bulk_commit_group();
          }
        }
        if (!__all_sync(0xffffffffu, ok)) {   // the leader's failure ends its whole warp
          ok = false;
          break;
        }
      }
    }
    if (leader) bulk_wait_all();
    if (!ok) watchdog_fire(kWdBwdDq);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

// delta[b*H + h, s] = sum_d dO * O32; zero the dQ accumulator.  A CTA takes 32 consecutive
// (token, head) pairs, i.e. 32 * D contiguous elements of dO / O32 / dQ, one 8-element chunk per
// thread (fully coalesced 16- and 32-byte accesses); each pair's D/8 chunk products are then summed
// in chunk order from shared memory.
template <bool F16>
__global__ void __launch_bounds__(32 * 16)
relpos_bwd_prep_kernel(const void* __restrict__ dout, const float* __restrict__ out32, float* __restrict__ delta,
                       float* __restrict__ dq_acc, int64_t pairs, int S, int H, int cph) {
  pdl_enter();
  using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
  __shared__ float part[32 * 16];
  const int64_t p0 = (int64_t)blockIdx.x * 32;
  const int64_t c = p0 * cph + threadIdx.x;   // this thread's 8-element chunk
  float acc = 0.f;
  if (c < pairs * cph) {
    const uint4 gv = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(dout) + 8 * c);
    const float4 o0 = *reinterpret_cast<const float4*>(out32 + 8 * c);
    const float4 o1 = *reinterpret_cast<const float4*>(out32 + 8 * c + 4);
    const T* gt = reinterpret_cast<const T*>(&gv);
    float gf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) gf[k] = F16 ? __half2float(*reinterpret_cast<const __half*>(&gt[k]))
                                            : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&gt[k]));
    acc = gf[0] * o0.x + gf[1] * o0.y + gf[2] * o0.z + gf[3] * o0.w;
    acc += gf[4] * o1.x + gf[5] * o1.y + gf[6] * o1.z + gf[7] * o1.w;
    *reinterpret_cast<float4*>(dq_acc + 8 * c) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(dq_acc + 8 * c + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  const int64_t pr = p0 + threadIdx.x;
  if (threadIdx.x < 32 && pr < pairs) {
    float s = 0.f;
    for (int k = 0; k < cph; ++k) s += part[threadIdx.x * cph + k];
    const int64_t tok = pr / H;
    const int hh = (int)(pr % H);
    delta[((tok / S) * H + hh) * S + tok % S] = s;
  }
}

// dqkv[:, q section] = dQ accumulator * scale, rounded to the input dtype.
template <bool F16>
__global__ void __launch_bounds__(256)
relpos_bwd_dq_kernel(const float* __restrict__ dq_acc, void* __restrict__ dqkv, int64_t dqkv_stride, int64_t rows,
                     int HD, float scale) {
  pdl_enter();
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

// dBias reduction, stage 1: one CTA per (tile diagonal d = kb - qb, head h, batch chunk c).  Thread
// (w, j) sums bin j of warp w over the chunk's batch elements and the tiles on diagonal d (each
// tile's 8 x 96 bins are one contiguous 3 KB row, so the CTA's loads are coalesced); then, per tile
// diagonal e = key - query in [-127, 127], the bins holding e (warp (half, quarter) keeps e in bin
// 32 quarter - 64 half + 31 - e) are added in warp order.  rows[h, d + nb - 1, c, e + 127].  The
// batch is split into up to kDiagChunks chunks so that enough CTAs stream the partials (one CTA per
// (d, h) left most SMs idle); fixed order throughout: deterministic.
constexpr int kDiagThreads = kWarpsPerTile * kBins;   // 768
constexpr int kDiagChunks = 8;
__host__ __device__ inline int diag_chunks(int B) { return B < kDiagChunks ? B : kDiagChunks; }
__global__ void __launch_bounds__(kDiagThreads)
relpos_bwd_dpd_diag_kernel(const float* __restrict__ part, float* __restrict__ rows, int B, int H, int nb) {
  pdl_enter();
  __shared__ float acc[kDiagThreads];
  const int d = (int)blockIdx.x - (nb - 1), h = blockIdx.y, c = blockIdx.z, nc = diag_chunks(B);
  const int kb_lo = d > 0 ? d : 0, kb_hi = d > 0 ? nb : nb + d;   // qb = kb - d in [0, nb)
  const int bb_lo = c * B / nc, bb_hi = (c + 1) * B / nc;
  float s = 0.f;
  for (int bb = bb_lo; bb < bb_hi; ++bb) {
    const float* pb = part + (size_t)(bb * H + h) * nb * nb * kDiagThreads;
    for (int kb = kb_lo; kb < kb_hi; ++kb) s += __ldg(pb + ((size_t)kb * nb + (kb - d)) * kDiagThreads + threadIdx.x);
  }
  acc[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x < 2 * kBlk - 1) {
    const int e = (int)threadIdx.x - (kBlk - 1);
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsPerTile; ++w) {
      const int j = 32 * (w % 4) - 64 * (w / 4) + 31 - e;
      if (j >= 0 && j < kBins) v += acc[w * kBins + j];
    }
    rows[(((size_t)h * (2 * nb - 1) + blockIdx.x) * nc + c) * 256 + threadIdx.x] = v;
  }
}

// dBias reduction, stage 2: dpd[h, t] for g = t - (S - 1) = key - query: the two tile diagonals
// whose range covers g (d_hi = ceil-ish (g - 127) / 128 and d_hi - 1), in that order, each summed
// over the batch chunks in chunk order.
__global__ void __launch_bounds__(256)
relpos_bwd_dpd_kernel(const float* __restrict__ rows, float* __restrict__ dpd, int S, int H, int nb, int nc) {
  pdl_enter();
  const int h = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= 2 * S - 1) return;
  const int g = t - (S - 1);
  const int d_hi = (g + 127) >= 0 ? (g + 127) / 128 : -((-(g + 127) + 127) / 128);
  float acc = 0.f;
  for (int d = d_hi; d >= d_hi - 1; --d) {
    const int e = g - 128 * d;
    if (e < -(kBlk - 1) || e > kBlk - 1 || d <= -nb || d >= nb) continue;
    const float* r = rows + ((size_t)h * (2 * nb - 1) + (d + nb - 1)) * nc * 256 + (e + kBlk - 1);
    for (int c = 0; c < nc; ++c) acc += r[(size_t)c * 256];
  }
  dpd[(size_t)h * (2 * S - 1) + t] = acc;
}

struct WsLayout {
  size_t delta, dq, part, rows, total;
};

inline WsLayout ws_layout(int64_t B, int64_t S, int64_t H, int64_t D) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const int64_t nb = (S + kBlk - 1) / kBlk;
  WsLayout w;
  w.delta = 0;
  w.dq = up((size_t)B * H * S * 4);
  w.part = w.dq + up((size_t)B * S * H * D * 4);
  w.rows = w.part + up((size_t)B * H * nb * nb * kWarpsPerTile * kBins * 4);
  w.total = w.rows + up((size_t)H * (2 * nb - 1) * diag_chunks((int)B) * 256 * 4);
  return w;
}

template <int DP, bool F16>
int launch_bwd(const CUtensorMap& qm, const CUtensorMap& om, const CUtensorMap& dqm, const CUtensorMap& kvm,
               const BwdArgs& a, const void* dout, const float* out32, float* dpd, cudaStream_t stream) {
  using C = BwdCfg<DP>;
  const int64_t tokens_heads = (int64_t)a.B * a.S * a.H;
  KRSI_CUDA_TRY(launch_pdl(relpos_bwd_prep_kernel<F16>, dim3((unsigned)((tokens_heads + 31) / 32)),
                           dim3(32 * (a.D / 8)), 0, stream, dout, out32, const_cast<float*>(a.delta), a.dq_acc,
                           tokens_heads, a.S, a.H, a.D / 8));
  const size_t res_smem = C::kSmem + (size_t)rows_bytes(a.S);
  const bool res = res_smem <= 232448;   // 227 KB per CTA on sm_100
  const bool fold = a.D % 16 == 8;       // padding columns D..D+2 free for -lse / -delta
  auto kern = res ? (fold ? relpos_bwd_main_kernel<DP, F16, true, true> : relpos_bwd_main_kernel<DP, F16, true, false>)
                  : (fold ? relpos_bwd_main_kernel<DP, F16, false, true> : relpos_bwd_main_kernel<DP, F16, false, false>);
  const size_t smem = res ? res_smem : C::kSmem;
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  KRSI_CUDA_TRY(launch_pdl(kern, dim3(a.n_blk, a.B * a.H), dim3(kThreads), smem, stream, qm, om, dqm, kvm, a));
  const int64_t rows = (int64_t)a.B * a.S;
  const int64_t items = rows * (a.H * a.D / 8);
  KRSI_CUDA_TRY(launch_pdl(relpos_bwd_dq_kernel<F16>, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, stream,
                           (const float*)a.dq_acc, a.dqkv, a.dqkv_stride, rows, a.H * a.D, a.scale));
  KRSI_CUDA_TRY(launch_pdl(relpos_bwd_dpd_diag_kernel, dim3(2 * a.n_blk - 1, a.H, diag_chunks(a.B)),
                           dim3(kDiagThreads), 0, stream, (const float*)a.dbias_part, a.dpd_rows, a.B, a.H, a.n_blk));
  KRSI_CUDA_TRY(launch_pdl(relpos_bwd_dpd_kernel, dim3((2 * a.S - 1 + 255) / 256, a.H), dim3(256), 0, stream,
                           (const float*)a.dpd_rows, dpd, a.S, a.H, a.n_blk, diag_chunks(a.B)));
  return KRSI_OK;
}

template <bool F16>
int dispatch_dp(int DP, const CUtensorMap& qm, const CUtensorMap& om, const CUtensorMap& dqm, const CUtensorMap& kvm,
                const BwdArgs& a, const void* dout, const float* out32, float* dpd, cudaStream_t s) {
  switch (DP) {
    case 32: return launch_bwd<32, F16>(qm, om, dqm, kvm, a, dout, out32, dpd, s);
    case 64: return launch_bwd<64, F16>(qm, om, dqm, kvm, a, dout, out32, dpd, s);
    case 80: return launch_bwd<80, F16>(qm, om, dqm, kvm, a, dout, out32, dpd, s);
    case 96: return launch_bwd<96, F16>(qm, om, dqm, kvm, a, dout, out32, dpd, s);
    case 128: return launch_bwd<128, F16>(qm, om, dqm, kvm, a, dout, out32, dpd, s);
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
  if (DP < 0) return KRSI_ERR_UNSUPPORTED;
  KRSI_CHECK_ARG(qkv_row_stride >= 3 * H * D && dqkv_row_stride >= 3 * H * D);
  if (qkv_row_stride % 8 || dqkv_row_stride % 8 || !aligned16(qkv) || !aligned16(dqkv) || !aligned16(dout) ||
      !aligned16(out32))
    return KRSI_ERR_MISALIGNED;
  if (S > (1 << 20) || B * H > 65535) return KRSI_ERR_UNSUPPORTED;
  const WsLayout ws = ws_layout(B, S, H, D);
  if (!workspace || workspace_bytes < ws.total || !aligned16(workspace)) return KRSI_ERR_WORKSPACE;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  CUtensorMap qm, om, dqm, kvm;
  const bool f16 = dtype == KRSI_F16;
  if (!attn::make_head_map(&qm, qkv, qkv_row_stride, B, S, 3 * H, D, f16) ||
      !attn::make_head_map(&om, dout, H * D, B, S, H, D, f16) ||
      !attn::make_rows_f32_map(&dqm, reinterpret_cast<float*>(w + ws.dq), B, S, H, D, DP > 80 ? D / 2 : D) ||
      !attn::make_head_rows_map(&kvm, dqkv, dqkv_row_stride, B, S, 3 * H, D, f16))
    return KRSI_ERR_CUDA;
  BwdArgs a{pd,
            lse,
            reinterpret_cast<float*>(w + ws.delta),
            reinterpret_cast<float*>(w + ws.dq),
            reinterpret_cast<float*>(w + ws.part),
            reinterpret_cast<float*>(w + ws.rows),
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
  return f16 ? dispatch_dp<true>(DP, qm, om, dqm, kvm, a, dout, out32, dpd, stream)
             : dispatch_dp<false>(DP, qm, om, dqm, kvm, a, dout, out32, dpd, stream);
}
