// relpos_attn_fwd.cu - relative-position-bias flash attention forward for B200 (sm_100a).
//
// Computes what library/relpos_attention.py:26-59 (_fwd) computes, for every (b, h):
//   s2[i, j] = (q_i . k_j * scale + pd[h, j - i + S - 1]) * log2(e)
//   m_i = max_j s2, l_i = sum_j exp2(s2 - m_i), out_i = sum_j exp2(s2 - m_i) v_j / l_i,
//   lse_i = m_i + log2(l_i); out in the input dtype, out32 in fp32.
//
// Structure: a persistent grid (one CTA per SM) whose CTAs loop over work items = two 128-query
// tiles of one (b, h); 12 warps = 3 warpgroups; setmaxnreg moves registers from warpgroup 0 to the
// softmax warpgroups:
//   warp 0      TMA producer (tile layout: attn_common.cuh): each item's Q as soon as the previous
//               item's last Q K^T completed, and per 128-key block a K tile and a V tile (3-stage
//               ring that runs on across items);
//   warps 2-3   the items' bias windows pd[h, ...] * log2(e) in shared memory (two copies, one
//               shifted by an element, for aligned pair reads), double-buffered: the next item's
//               window is filled while the current one is read (the first item's with the softmax
//               warps' help); sequences too long for it fall back to per-block slabs the producer
//               writes;
//   warp 1      TMEM owner (512 columns) and the single-thread tcgen05.mma issuer.  Each S tile
//               is computed in two halves of 64 keys: S_{t,h} = Q_t K_h^T (SS, N = 64, K = DP)
//               and O_t += P_{t,h} V_h (TS: P read from TMEM, one N = DP instruction per 16
//               keys).  As soon as the softmax warps hand back a half's P, its P V and the next
//               block's Q K^T for the same half are issued, so the MMAs of one half run while
//               the softmax warps work on the other; the next item's first S halves are issued
//               right after the current item's last P V, so they run while O is written out;
//   warps 4-7   softmax for query tile 0, warps 8-11 for tile 1 (one query row per thread,
//               row = TMEM lane), half by half: S from TMEM -> bias add (paired fp32 FMAs) ->
//               online softmax with the rescale of O skipped unless the running max grows by
//               more than 2^8; exp2 on the SFU for 3/4 of the elements and on the FMA pipe
//               (sm100.cuh) for 1/4 -> P (bf16/f16) written back over the S half in TMEM -> at
//               the item's end O / l to memory.
// Every wait is bounded (watchdog.cuh); a stalled pipeline ends the CTA with an error word.
#include <string.h>

#include <type_traits>

#include "attn_common.cuh"
#include "common.cuh"
#include "watchdog.cuh"

KRSI_DEFINE_WATCHDOG(attn_fwd)

namespace krsi {
namespace {

using namespace sm100;
using attn::kTileRows;

constexpr int kBN = 128;            // keys per block
constexpr int kHalf = 64;           // keys per S half: each half has its own Q K^T, softmax step and P V
constexpr int kQTiles = 2;          // query tiles per work item
constexpr int kItemRows = kQTiles * kTileRows;   // queries per work item
constexpr int kThreads = 384;       // 3 warpgroups: {producer, MMA, window fill}, softmax tile 0, tile 1
constexpr uint32_t kRegsCtl = 112;  // per-thread registers of warpgroup 0 after setmaxnreg
constexpr uint32_t kRegsSm = 192;   // softmax warpgroups (launch 168 x 384 >= 128 x (112 + 2 x 192))
constexpr int kSlab = 384;          // floats per bias slab (2*128 + 128 - 1 = 383 used)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units: P <= 2^8 between rescales
constexpr int kInitFillers = 320;          // warps 2-11 fill the first item's bias window
constexpr int kBgFillers = 64;             // warps 2-3 fill the later items' windows

template <int DP>
struct FwdCfg {
  static constexpr int NS = DP <= 96 ? 3 : 2;                      // K/V pipeline stages
  static constexpr uint32_t kTile = attn::Tile<DP>::kBytes;         // one 128 x DP tile
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKVOff = kQOff + kQTiles * kTile;
  static constexpr uint32_t kSlabOff = kKVOff + NS * 2 * kTile;
  static constexpr uint32_t kBarOff = kSlabOff + NS * kSlab * 4;
  // q_full, q_empty, kv_full/empty, s_ready/p_ready/o_sync per (tile, half), o_final/o_free per
  // tile, drain, row_init, row_full[2], row_free[2]
  static constexpr int kNumBars = 2 + 2 * NS + 3 * 2 * kQTiles + 2 * kQTiles + 1 + 1 + 2 + 2;
  static constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;
  static constexpr uint32_t kRowOff = (kMiscOff + 16 + 15) & ~15u;  // bias windows (runtime length)
  static constexpr uint32_t kSmem = kRowOff + 1024;                 // static part + alignment slack
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kSCol = 0;                              // S_t at t*128
  static constexpr uint32_t kOCol = 256;                            // O_t at 256 + t*DP
  static_assert(kOCol + kQTiles * DP <= kTmemCols, "TMEM budget");
};

struct FwdArgs {
  const float* pd;
  void* out;
  float* out32;
  float* lse;
  int B, S, H, D;
  float scale_log2;   // scale * log2(e)
  int n_kb;           // key blocks
  int n_qp;           // query pairs (work items per head)
  uint32_t spin_limit;
  int out32_v8;       // out32 is 32-byte aligned: 256-bit stores
  uint32_t obox_off;  // shared-memory offset of the output staging boxes (0: per-thread stores)
};

// Output staging: each softmax warp writes its 32 rows of O in 16-column chunks into two boxes, the
// fp32 one [32 rows x 16] (64-byte rows, 64-byte swizzle) and the 16-bit one [32 x 16] (32-byte rows,
// 32-byte swizzle), and one lane stores both with TMA (maps over (D, H, S, B): columns past D and rows
// past S are clipped).  Measured against per-thread stores (32 rows per warp instruction), same box:
// 29.8 vs 31.0 us at B 2 S 1024, 299.7 vs 304.2 us at B 8 S 2048, 343.1 vs 341.5 us at B 32 S 1024.
// (With the output stores removed altogether the last took 283.5 us: most of their cost is the
// 226 MB of HBM writes themselves, which staging cannot remove.)
constexpr uint32_t kOBox32 = 32 * 16 * 4;
constexpr uint32_t kOBoxWarp = kOBox32 + 32 * 16 * 2;   // 3 KB per softmax warp
constexpr uint32_t kOBoxBytes = 8 * kOBoxWarp;

// Bias windows.  The bias of (query q, key k) is pd[h, k - q + S - 1].  A work item (queries q0 ..
// q0 + 255, all keys) forms indices kRowPad + k - q + S - 1 in [w0 + 2, w0 + win_floats - 4] with
// w0 = even(max(kRowPad + S - 1 - q0 - 257, 0)); the window stores them from w0 on, scaled by
// log2(e), in two copies (the second shifted by one element) so that every thread reads its bias
// values as 8-byte aligned pairs (copy 0 when its start index is even, copy 1 when odd).  Lane l
// of a warp starts at B0 - l with B0 of the parity of S - 1: in a half-warp the copy-0 lanes read
// 16 consecutive floats and the copy-1 lanes 16 more, shifted by the copy distance - 16 (S even) or
// - 18 (S odd); copies 16 or 18 (mod 32) floats apart put the two halves on disjoint banks.  Two
// windows (double buffer): the next item's window is filled while the current one is read.
constexpr int kRowPad = 256;
__host__ __device__ constexpr int64_t win_floats(int64_t S) {
  return (((S + kBN - 1) / kBN) * kBN + 264 + 31 - ((S & 1) ? 18 : 16)) / 32 * 32 + ((S & 1) ? 18 : 16);
}
__host__ __device__ constexpr int64_t win_bytes(int64_t S) { return 4 * win_floats(S) * 4; }   // 2 windows x 2 copies
__device__ __forceinline__ int win_start(int S, int q0) { return max(kRowPad + S - 1 - q0 - 257, 0) & ~1; }

// dst[i] = src[i + off] * log2(e) for i in [0, n), zero where i + off is outside [0, len), by nthr
// cooperating threads.  The source range handed to fill_row is clipped to the window (fill_row
// writes dst[pad + p] for every source element p it is given).
__device__ __forceinline__ void fill_shifted(float* dst, int n, int off, const float* __restrict__ src, int len,
                                             int tid, int nthr) {
  if (off >= 0) attn::fill_row(dst, n, 0, src + min(off, len), min(max(len - off, 0), n), kLog2e, tid, nthr);
  else attn::fill_row(dst, n, min(-off, n), src, min(len, max(n + off, 0)), kLog2e, tid, nthr);
}

// Persistent: one CTA per SM; work item it = (b*H + h) * n_qp + query pair, CTA c takes items
// c, c + gridDim.x, ...  Across items the K/V ring, TMEM and the barriers carry on: Q of the next
// item is loaded as soon as the last Q K^T of the current one has completed, its first S tiles are
// computed while the softmax warps write the current item's output, and its bias window is filled
// in the background by warps 2-3.
template <int DP, bool F16, bool RES>
__global__ void __launch_bounds__(kThreads, 1)
relpos_fwd_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap o32map,
                  const __grid_constant__ CUtensorMap o16map, const FwdArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  using C = FwdCfg<DP>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + NS;
  uint64_t* s_ready = kv_empty + NS;            // [tile * 2 + half]: S half computed
  uint64_t* p_ready = s_ready + 2 * kQTiles;    // [tile * 2 + half]: P half written to TMEM
  uint64_t* o_sync = p_ready + 2 * kQTiles;     // [tile * 2 + half]: P V of that half completed
  uint64_t* o_final = o_sync + 2 * kQTiles;
  uint64_t* o_free = o_final + kQTiles;
  uint64_t* drain = o_free + kQTiles;
  uint64_t* row_init = drain + 1;
  uint64_t* row_full = row_init + 1;   // [2]
  uint64_t* row_free = row_full + 2;   // [2]
  const int wf = (int)win_floats(a.S);
  float* wins = reinterpret_cast<float*>(smem + C::kRowOff);   // window w, copy c at (2w + c) * wf
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  float* slabs = reinterpret_cast<float*>(smem + C::kSlabOff);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_kb = a.n_kb;
  const int n_items = a.B * a.H * a.n_qp;
  const int my_items = (int)blockIdx.x < n_items ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto item_bh = [&](int k) { return ((int)blockIdx.x + k * (int)gridDim.x) / a.n_qp; };
  auto item_q0 = [&](int k) { return (((int)blockIdx.x + k * (int)gridDim.x) % a.n_qp) * kItemRows; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], RES ? 1 : 2);   // TMA expect_tx arrival (+ bias-slab arrival)
      mbar_init(&kv_empty[s], 1);            // tcgen05.commit
    }
    for (int i = 0; i < 2 * kQTiles; ++i) {
      mbar_init(&s_ready[i], 1);
      mbar_init(&p_ready[i], 128);
      mbar_init(&o_sync[i], 1);
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(&o_final[t], 1);
      mbar_init(&o_free[t], 128);
    }
    mbar_init(drain, 1);
    mbar_init(row_init, kInitFillers);
    for (int w = 0; w < 2; ++w) {
      mbar_init(&row_full[w], kBgFillers);
      mbar_init(&row_free[w], 2 * 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&tmap);
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The bias window of item k into window k & 1 (RES), by `nthr` threads.
  auto fill_window = [&](int k, int tid, int nthr) {
    const int two_s = 2 * a.S - 1;
    const float* pdh = a.pd + (size_t)(item_bh(k) % a.H) * two_s;
    const int w0 = win_start(a.S, item_q0(k));
    float* c0 = wins + (size_t)(2 * (k & 1)) * wf;
    fill_shifted(c0, wf, w0 - kRowPad, pdh, two_s, tid, nthr);
    fill_shifted(c0 + wf, wf, w0 - kRowPad + 1, pdh, two_s, tid, nthr);   // copy 1: c1[i] = c0[i + 1]
  };
  // Each role runs entirely inside the branch that sets its register budget, so ptxas compiles
  // it against that budget.
  if (warp < 4) {
    regs_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int g = 0;   // global key-block counter (K/V ring position)
    for (int k = 0; k < my_items; ++k) {
      const int bh = item_bh(k), b = bh / a.H, h = bh % a.H, q0 = item_q0(k);
      if (k > 0 && !mbar_wait_bounded(q_empty, (k - 1) & 1, abort_flag, a.spin_limit)) {
        watchdog_fire(kWdFwdLoad);
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, kQTiles * C::kTile);
        for (int t = 0; t < kQTiles; ++t)
          attn::load_tile<DP>(smem + C::kQOff + t * C::kTile, &tmap, q_full, h, q0 + t * kTileRows, b);
      }
      const int two_s = 2 * a.S - 1;
      const float* pdh = a.pd + (size_t)h * two_s;
      bool ok = true;
      for (int j = 0; j < n_kb; ++j, ++g) {
        const int s = g % NS;
        if (g >= NS && !mbar_wait_bounded(&kv_empty[s], ((g / NS) + 1) & 1, abort_flag, a.spin_limit)) {
          ok = false;
          break;
        }
        uint8_t* kt = smem + C::kKVOff + (2 * s) * C::kTile;
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_full[s], 2 * C::kTile);
          attn::load_tile<DP>(kt, &tmap, &kv_full[s], a.H + h, j * kBN, b);
          attn::load_tile<DP>(kt + C::kTile, &tmap, &kv_full[s], 2 * a.H + h, j * kBN, b);
        }
        if constexpr (RES) continue;
        // bias slab: slab[idx] = pd[h, j*128 - q0 - 255 + idx + S - 1] * log2e, zero outside the table
        float* slab = slabs + s * kSlab;
        const int base = j * kBN - q0 - (kItemRows - 1) + a.S - 1;
        for (int idx = lane; idx < kSlab; idx += 32) {
          const int pos = base + idx;
          slab[idx] = (pos >= 0 && pos < two_s) ? __ldg(pdh + pos) * kLog2e : 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&kv_full[s]);
      }
      if (!ok) {
        watchdog_fire(kWdFwdLoad);
        break;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ bias windows (RES)
    if constexpr (RES) {
      const int tid = threadIdx.x - 64;
      if (my_items > 0) {
        fill_window(0, tid, kInitFillers);
        mbar_arrive(row_init);
      }
      for (int k = 1; k < my_items; ++k) {
        // window k & 1 is free once every softmax thread has finished item k - 2
        if (k >= 2 && !__all_sync(0xffffffffu, mbar_wait_bounded(&row_free[k & 1], ((k - 2) >> 1) & 1, abort_flag,
                                                                   a.spin_limit))) {
          watchdog_fire(kWdFwdLoad);
          break;
        }
        fill_window(k, tid, kBgFillers);
        mbar_arrive(&row_full[k & 1]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs this branch with warp-uniform descriptors and one elected lane issues each
    // MMA and commit: measured on B200, a single-lane issue loop takes 47 cycles per M128 N64/N80 TS
    // MMA where the tensor pipe needs 32/40.  Waits are warp-uniform so every lane takes one path.
    {
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.spin_limit));
      };
      constexpr uint32_t fmt = F16 ? 0u : 1u;
      constexpr uint32_t id_qk = idesc_f16(128, kHalf, fmt, false, false);   // S half = Q K_h^T: both K-major
      constexpr uint32_t id_pv = idesc_f16(128, DP, fmt, false, true);       // O += P_h V_h: V MN-major, N = DP
      // Descriptors are precomputed; an issue is a constant add and the MMA itself, which keeps
      // one thread issuing at the tensor pipe's rate.
      const uint64_t q_desc = attn::kmajor_base(smem_u32(smem + C::kQOff));
      const uint64_t k_desc0 = attn::kmajor_base(smem_u32(smem + C::kKVOff));
      const uint64_t v_desc0 = attn::mnmajor_base(smem_u32(smem + C::kKVOff + C::kTile));
      constexpr uint64_t kStageStep = (2 * C::kTile) >> 4;
      constexpr uint64_t kQTileStep = C::kTile >> 4;
      constexpr uint64_t kHalfRowStep = (kHalf * 32) >> 4;   // K rows 64.. of every 16-column block
      // S_{t,h} = Q_t K^T over keys [64h, 64h + 64) of block g, into columns t*128 + 64h
      auto issue_qk = [&](int t, int h, int g) {
        const uint64_t qd = q_desc + (uint64_t)t * kQTileStep;
        const uint64_t kd = k_desc0 + (uint64_t)(g % NS) * kStageStep + (uint64_t)h * kHalfRowStep;
        const uint32_t d = tmem + C::kSCol + t * kBN + h * kHalf;
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          mma_ss_e(d, qd + kk * attn::kKSliceStep, kd + kk * attn::kKSliceStep, id_qk, kk > 0 ? 1u : 0u);
      };
      // O_t += P_{t,h} V_h: P (2 x 16-bit per column) in the first 32 columns of its S half
      auto issue_pv = [&](int t, int h, int g, bool first) {
        const uint64_t vd = v_desc0 + (uint64_t)(g % NS) * kStageStep;
        const uint32_t p_tmem = tmem + C::kSCol + t * kBN + h * kHalf;
        const uint32_t d = tmem + C::kOCol + t * DP;
        const uint32_t acc0 = first ? 0u : 1u;
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk)
          mma_ts_e(d, p_tmem + kk * 8, vd + (h * (kHalf / 16) + kk) * attn::kKRowStep, id_pv, kk > 0 ? 1u : acc0);
      };
      bool ok = my_items > 0 && wait(q_full, 0) &&
                wait(&kv_full[0], 0);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < 2; ++h)
          for (int t = 0; t < kQTiles; ++t) {
            issue_qk(t, h, 0);
            mma_commit_e(&s_ready[2 * t + h]);
          }
        if (n_kb == 1) mma_commit_e(q_empty);   // item 0's only Q K^T is issued
      }
      // Per block, the halves are served in the order (t0, h0), (t1, h0), (t0, h1), (t1, h1): P V of
      // a half, then (inside an item) the next block's Q K^T into the same S half, so the softmax
      // warps work on one half while the other half's MMAs run.
      int g = 0;
      for (int k = 0; k < my_items && ok; ++k) {
        for (int j = 0; j < n_kb && ok; ++j, ++g) {
          // the next block: (k, j + 1) or the next item's first
          const bool last_j = j + 1 == n_kb;
          const bool has_next = !last_j || k + 1 < my_items;
          auto wait_next = [&]() {   // K/V of block g + 1 (and, for a new item, its Q) landed
            return wait(&kv_full[(g + 1) % NS], ((g + 1) / NS) & 1) &&
                   (!last_j || wait(q_full, (k + 1) & 1));
          };
          for (int h = 0; h < 2 && ok; ++h)
            for (int t = 0; t < kQTiles; ++t) {
              if (!wait(&p_ready[2 * t + h], g & 1) ||
                  (j == 0 && h == 0 && k > 0 && !wait(&o_free[t], (k - 1) & 1)) ||
                  (!last_j && t == 0 && h == 0 && !wait_next())) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_pv(t, h, g, j == 0 && h == 0);
              mma_commit_e(&o_sync[2 * t + h]);
              if (last_j) {
                if (h == 1) mma_commit_e(&o_final[t]);
              } else {
                issue_qk(t, h, g + 1);
                mma_commit_e(&s_ready[2 * t + h]);
              }
            }
          // an item's last block: every P V first (its output is written out while the next item's
          // Q and first K/V arrive), then the next item's first S halves
          if (ok && last_j && has_next) {
            if (!wait_next()) {
              ok = false;
            } else {
              tc_fence_after();
              for (int h = 0; h < 2; ++h)
                for (int t = 0; t < kQTiles; ++t) {
                  issue_qk(t, h, g + 1);
                  mma_commit_e(&s_ready[2 * t + h]);
                }
            }
          }
          if (!ok) break;
          // the Q K^T just issued was the last one of its item: its Q may be replaced
          if (has_next && (last_j ? n_kb == 1 : j + 2 == n_kb)) mma_commit_e(q_empty);
          mma_commit_e(&kv_empty[g % NS]);
        }
      }
      if (!ok && my_items > 0) watchdog_fire(kWdFwdMma);
      // Drain: every MMA issued above has completed before TMEM is released.
      mma_commit_e(drain);
      for (uint32_t i = 0; i < a.spin_limit && !mbar_try_wait(drain, 0); ++i) {
      }
    }
  }
  } else {
    regs_inc<kRegsSm>();
    if constexpr (RES) {
      if (my_items > 0) {
        fill_window(0, threadIdx.x - 64, kInitFillers);
        mbar_arrive(row_init);
      }
    }
    // ------------------------------------------------------------ softmax (warps 4..11)
    const int t = (warp - 4) / 4;                       // query tile
    const int quarter = warp % 4;                       // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;                  // row within the tile
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_tmem = tmem + lane_addr + C::kSCol + t * kBN;
    const uint32_t o_tmem = tmem + lane_addr + C::kOCol + t * DP;
    const int slab_base = (kQTiles - 1 - t) * kTileRows + (kTileRows - 1) - r;   // slab[slab_base + c]
    const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
    bool ok = true;
    int g = 0;
    for (int k = 0; k < my_items && ok; ++k) {
      const int bh = item_bh(k), b = bh / a.H, q0 = item_q0(k);
      const int q = q0 + t * kTileRows + r;             // query index within the sequence
      // window: bias(q, key j*128 + c) = win[bidx + c], bidx = kRowPad + j*128 - q + S - 1 - w0
      const float* bias_q = nullptr;
      if constexpr (RES) {
        const bool w_ok = k == 0 ? mbar_wait_bounded(row_init, 0, abort_flag, a.spin_limit)
                                 : mbar_wait_bounded(&row_full[k & 1], ((k - 1) >> 1) & 1, abort_flag, a.spin_limit);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        const int bidx0 = kRowPad - q + a.S - 1 - win_start(a.S, q0);
        const float* c0 = wins + (size_t)(2 * (k & 1)) * wf;
        bias_q = (bidx0 & 1) ? c0 + wf + bidx0 - 1 : c0 + bidx0;   // 8-byte aligned pairs
      }
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n_kb && ok; ++j, ++g) {
        const int s = g % NS;
        for (int h = 0; h < 2; ++h) {
          const bool w_ok = mbar_wait_bounded(&s_ready[2 * t + h], g & 1, abort_flag, a.spin_limit) &&
                            (RES || h > 0 || mbar_wait_bounded(&kv_full[s], (g / NS) & 1, abort_flag, a.spin_limit));
          if (!__all_sync(0xffffffffu, w_ok)) {   // warp-uniform: TMEM loads/stores are warp-collective
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sh_tmem = s_tmem + h * kHalf;
          uint32_t u[kHalf];
          tmem_ld32(sh_tmem, u);
          tmem_ld32(sh_tmem + 32, u + 32);
          tmem_wait_ld();
          // v = s * scale * log2(e) + bias * log2(e), two columns per instruction
          uint64_t v2[kHalf / 2];
          if constexpr (RES) {
            const uint64_t* bp = reinterpret_cast<const uint64_t*>(bias_q + j * kBN + h * kHalf);
#pragma unroll
            for (int i = 0; i < kHalf / 2; ++i)
              v2[i] = f2_fma(f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), scale2, bp[i]);
          } else {
            const float* slab = slabs + s * kSlab + slab_base + h * kHalf;
#pragma unroll
            for (int i = 0; i < kHalf / 2; ++i)
              v2[i] = f2_fma(f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), scale2,
                             f2_pack(slab[2 * i], slab[2 * i + 1]));
          }
          const int valid = a.S - j * kBN - h * kHalf;      // keys of this half inside the sequence
          if (valid < kHalf) {                              // only the last block of a ragged sequence
#pragma unroll
            for (int i = 0; i < kHalf / 2; ++i) {
              float lo, hi;
              f2_unpack(v2[i], lo, hi);
              v2[i] = f2_pack(2 * i < valid ? lo : -INFINITY, 2 * i + 1 < valid ? hi : -INFINITY);
            }
          }
          // row max: 3-input max, 4 independent chains
          float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < kHalf / 2; ++i) {
            float lo, hi;
            f2_unpack(v2[i], lo, hi);
            mxa[i % 4] = max3(mxa[i % 4], lo, hi);
          }
          const float mx = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3]));
          const float m_new = fmaxf(m_run, mx);
          // true on the item's first half (m_run = -inf); a fully masked half (m_new = m_run) never
          const bool need = m_new - m_run > kRescaleThreshold;
          float alpha = 1.f, m_use = m_run;
          const bool warp_rescale = __any_sync(0xffffffffu, need);
          if (warp_rescale) {
            m_use = m_new;
            alpha = ex2_approx(m_run - m_new);              // 0 on the first half
          }
          // p = 2^(v - m): three of every four pairs on the SFU, one on the FMA pipe (balances the
          // SFU against the issue slots); row sum in 4 paired chains; P packed to 16-bit pairs
          const uint64_t negm2 = f2_pack(-m_use, -m_use);
          uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
          uint32_t pk[kHalf / 2];
#pragma unroll
          for (int i = 0; i < kHalf / 2; ++i) {
            float x0, x1, p0, p1;
            f2_unpack(f2_add(v2[i], negm2), x0, x1);
            if (i % 4 == 3) {
              exp2_poly3_x2(x0, x1, p0, p1);
            } else {
              p0 = ex2_approx(x0);
              p1 = ex2_approx(x1);
            }
            acc2[i % 4] = f2_add(acc2[i % 4], f2_pack(p0, p1));
            pk[i] = F16 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
          }
          float sum_lo, sum_hi;
          f2_unpack(f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3])), sum_lo, sum_hi);
          const float sum = sum_lo + sum_hi;
          l_run = l_run * alpha + sum;
          m_run = m_use;
          tmem_st32(sh_tmem, pk);
          if (warp_rescale && (j > 0 || h > 0)) {
            // O_t must hold exactly the P V of every earlier half.  The previous half's P V is
            // the last one issued for this tile: wait for it (the one before it completed before
            // this half's S was computed), then scale O_t.
            const int hp = h ^ 1, gp = h ? g : g - 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_sync[2 * t + hp], gp & 1, abort_flag, a.spin_limit))) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < DP; c += 16) {
              uint32_t ov[16];
              tmem_ld16(o_tmem + c, ov);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
              tmem_st16(o_tmem + c, ov);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&p_ready[2 * t + h]);
        }
      }
      if (!ok) break;
      if constexpr (RES) mbar_arrive(&row_free[k & 1]);   // this item's window is no longer read
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_final[t], k & 1, abort_flag, a.spin_limit))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // All lanes run the warp-collective TMEM loads; rows past the sequence end skip the stores.
      const bool row_ok = q < a.S;
      const float inv_l = 1.0f / l_run;
      const size_t row = (size_t)b * a.S + (row_ok ? q : 0);
      const size_t ld = (size_t)a.H * a.D;
      float* o32 = a.out32 + row * ld + (size_t)(bh % a.H) * a.D;
      using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
      T* o16 = reinterpret_cast<T*>(a.out) + row * ld + (size_t)(bh % a.H) * a.D;
      // O in column groups of up to 96 (one group for DP <= 96): a group is read from TMEM, then
      // stored; O_t is released for the next item's first P V once its last group is read.
      constexpr int kGrp = DP <= 96 ? DP : DP / 2;
#pragma unroll
      for (int c0 = 0; c0 < DP; c0 += kGrp) {
        float ofin[kGrp];
#pragma unroll
        for (int c = 0; c < kGrp; c += 16) {
          uint32_t ov[16];
          tmem_ld16(o_tmem + c0 + c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) ofin[c + e] = __uint_as_float(ov[e]) * inv_l;
        }
        if (c0 + kGrp == DP) {   // O_t has been read: the next item's first P V may overwrite it
          tc_fence_before();
          mbar_arrive(&o_free[t]);
        }
        if (a.obox_off != 0) {   // staged: boxes of 16 columns, two TMA stores per chunk
          uint8_t* box32 = smem + a.obox_off + (warp - 4) * kOBoxWarp;
          uint8_t* box16 = box32 + kOBox32;
          const int qrow0 = q0 + t * kTileRows + quarter * 32;   // the warp's first row
#pragma unroll
          for (int c = 0; c < kGrp; c += 16) {
            if (c0 + c >= a.D) break;   // warp-uniform
            if (lane == 0) bulk_wait_read_all();   // the previous chunk's boxes have been read
            __syncwarp();
            const float* f = ofin + c;
            uint4* b32 = reinterpret_cast<uint4*>(box32 + lane * 64);
#pragma unroll
            for (int p4 = 0; p4 < 4; ++p4)
              b32[p4 ^ ((lane >> 1) & 3)] = make_uint4(__float_as_uint(f[4 * p4]), __float_as_uint(f[4 * p4 + 1]),
                                                       __float_as_uint(f[4 * p4 + 2]), __float_as_uint(f[4 * p4 + 3]));
            uint4* b16 = reinterpret_cast<uint4*>(box16 + lane * 32);
#pragma unroll
            for (int p8 = 0; p8 < 2; ++p8) {
              const float* h8 = f + 8 * p8;
              b16[p8 ^ ((lane >> 2) & 1)] =
                  F16 ? make_uint4(pack_f16x2(h8[0], h8[1]), pack_f16x2(h8[2], h8[3]), pack_f16x2(h8[4], h8[5]),
                                   pack_f16x2(h8[6], h8[7]))
                      : make_uint4(pack_bf16x2(h8[0], h8[1]), pack_bf16x2(h8[2], h8[3]),
                                   pack_bf16x2(h8[4], h8[5]), pack_bf16x2(h8[6], h8[7]));
            }
            fence_async_shared();   // staged boxes -> visible to the TMA unit
            __syncwarp();
            if (lane == 0 && qrow0 < a.S) {
              tma_store_4d(&o32map, box32, c0 + c, bh % a.H, qrow0, b);
              tma_store_4d(&o16map, box16, c0 + c, bh % a.H, qrow0, b);
              bulk_commit_group();
            }
          }
          continue;
        }
#pragma unroll
        for (int c = 0; c < kGrp; c += 8) {
          if (row_ok && c0 + c < a.D) {   // D is a multiple of 8: whole 8-column groups are in or out
            const float* f = ofin + c;
            float* d32p = o32 + c0 + c;
            if (a.out32_v8) {   // one 32-byte store per 8 columns (each row's chunk is its own line)
              asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(d32p), "f"(f[0]),
                           "f"(f[1]), "f"(f[2]), "f"(f[3]), "f"(f[4]), "f"(f[5]), "f"(f[6]), "f"(f[7])
                           : "memory");
            } else {
              float4* d32 = reinterpret_cast<float4*>(d32p);
              d32[0] = make_float4(f[0], f[1], f[2], f[3]);
              d32[1] = make_float4(f[4], f[5], f[6], f[7]);
            }
            const uint4 pk = F16 ? make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]),
                                              pack_f16x2(f[4], f[5]), pack_f16x2(f[6], f[7]))
                                 : make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                              pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
            *reinterpret_cast<uint4*>(o16 + c0 + c) = pk;
          }
        }
      }
      if (row_ok) a.lse[(size_t)bh * a.S + q] = m_run + __log2f(l_run);
    }
    if (a.obox_off != 0 && lane == 0) bulk_wait_all();   // every output store has completed
    if (!ok) watchdog_fire(kWdFwdSoftmax);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

constexpr size_t kMaxSmem = 232448;   // 227 KB per CTA on sm_100

// 4-D view (D, H, S, B) of a [B*S, H*D] output (element size es) for the staging boxes' TMA stores:
// box (16, 1, 32, 1), so a store clips at column D of its head and at row S of its sequence.
bool make_out_box_map(CUtensorMap* map, const void* base, int64_t B, int64_t S, int64_t H, int64_t D, int es,
                      CUtensorMapDataType dt, CUtensorMapSwizzle sw) {
  attn::EncodeTiledFn enc = attn::encode_fn();
  if (!enc) return false;
  memset(map, 0, sizeof(*map));
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(D * es), (cuuint64_t)(H * D * es), (cuuint64_t)(S * H * D * es)};
  cuuint32_t box[4] = {16, 1, 32, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int DP, bool F16>
int launch_fwd(const CUtensorMap& tmap, const CUtensorMap& o32map, const CUtensorMap& o16map, FwdArgs a,
               bool maps_ok, cudaStream_t stream) {
  using C = FwdCfg<DP>;
  const size_t res_smem = C::kSmem + (size_t)win_bytes(a.S);
  const bool res = res_smem <= kMaxSmem;
  auto kern = res ? relpos_fwd_kernel<DP, F16, true> : relpos_fwd_kernel<DP, F16, false>;
  size_t smem = res ? res_smem : C::kSmem;
  // the output staging boxes after everything else (512-byte aligned for the 64-byte swizzle), when
  // they fit; smem - 1024 is the layout's end (the last 1024 bytes are alignment slack)
  const size_t box_off = (smem - 1024 + 511) & ~size_t(511);
  if (maps_ok && box_off + kOBoxBytes + 1024 <= kMaxSmem) {
    a.obox_off = (uint32_t)box_off;
    smem = box_off + kOBoxBytes + 1024;
  } else {
    a.obox_off = 0;
  }
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t items = (int64_t)a.B * a.H * a.n_qp;   // persistent: at most one CTA per SM
  const int grid = (int)(items < device_sm_count() ? items : device_sm_count());
  KRSI_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, tmap, o32map, o16map, a));
  return KRSI_OK;
}

template <bool F16>
int dispatch_dp(int DP, const CUtensorMap& tmap, const CUtensorMap& o32m, const CUtensorMap& o16m, const FwdArgs& a,
                bool maps_ok, cudaStream_t s) {
  switch (DP) {
    case 32: return launch_fwd<32, F16>(tmap, o32m, o16m, a, maps_ok, s);
    case 64: return launch_fwd<64, F16>(tmap, o32m, o16m, a, maps_ok, s);
    case 80: return launch_fwd<80, F16>(tmap, o32m, o16m, a, maps_ok, s);
    case 96: return launch_fwd<96, F16>(tmap, o32m, o16m, a, maps_ok, s);
    case 128: return launch_fwd<128, F16>(tmap, o32m, o16m, a, maps_ok, s);
    default: return KRSI_ERR_UNSUPPORTED;
  }
}

}  // namespace

// Padded head width used by both attention kernels (compiled variants: 32, 64, 80, 96, 128).
int attn_padded_dim(int64_t D) {
  if (D <= 0 || D > 128 || D % 8 != 0) return -1;
  const int dp = (int)((D + 15) / 16 * 16);
  if (dp <= 32) return 32;
  if (dp <= 64) return 64;
  if (dp <= 80) return 80;
  if (dp <= 96) return 96;
  return 128;
}

}  // namespace krsi

using namespace krsi;

extern "C" int krsi_relpos_attn_fwd(const void* qkv, int64_t qkv_row_stride, const float* pd, void* out,
                                    float* out32, float* lse, int64_t B, int64_t S, int64_t H, int64_t D,
                                    float scale, int dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(B >= 0 && S >= 0 && H > 0 && D > 0);
  if (B == 0 || S == 0) return KRSI_OK;
  KRSI_CHECK_ARG(qkv && pd && out && out32 && lse);
  if (dtype != KRSI_BF16 && dtype != KRSI_F16) return KRSI_ERR_UNSUPPORTED;
  const int DP = attn_padded_dim(D);
  if (DP < 0) return KRSI_ERR_UNSUPPORTED;
  KRSI_CHECK_ARG(qkv_row_stride >= 3 * H * D);
  if (qkv_row_stride % 8 != 0 || !aligned16(qkv) || !aligned16(out) || !aligned16(out32))
    return KRSI_ERR_MISALIGNED;
  if (S > (1 << 24) || B * H > 65535) return KRSI_ERR_UNSUPPORTED;
  CUtensorMap tmap;
  if (!attn::make_head_map(&tmap, qkv, qkv_row_stride, B, S, 3 * H, D, dtype == KRSI_F16)) return KRSI_ERR_CUDA;
  if (B * H * ((S + kItemRows - 1) / kItemRows) > INT32_MAX) return KRSI_ERR_UNSUPPORTED;
  FwdArgs a{pd, out, out32, lse, (int)B, (int)S, (int)H, (int)D, scale * 1.4426950408889634f,
            (int)((S + kBN - 1) / kBN), (int)((S + kItemRows - 1) / kItemRows), kSpinLimit,
            (reinterpret_cast<uintptr_t>(out32) & 31) == 0 ? 1 : 0, 0u};
  CUtensorMap o32m, o16m;
  const bool maps_ok = make_out_box_map(&o32m, out32, B, S, H, D, 4, CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                        CU_TENSOR_MAP_SWIZZLE_64B) &&
                       make_out_box_map(&o16m, out, B, S, H, D, 2,
                                        dtype == KRSI_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                        CU_TENSOR_MAP_SWIZZLE_32B);
  if (!maps_ok) memset(&o32m, 0, sizeof(o32m)), memset(&o16m, 0, sizeof(o16m));
  return dtype == KRSI_F16 ? dispatch_dp<true>(DP, tmap, o32m, o16m, a, maps_ok, stream)
                           : dispatch_dp<false>(DP, tmap, o32m, o16m, a, maps_ok, stream);
}
