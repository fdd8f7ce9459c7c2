// linear_geglu.cu - the T5 feed-forward's merged gate|value projection with GEGLU in the GEMM's
// epilogue, for B200 (sm_100a):
//   u = x W^T          x [rows, K], W [2F, K] (nn.Linear layout: rows [0, F) gate, [F, 2F) value)
//   out = geglu(u)     = (gelu_tanh(u[:, :F]).to(dtype) * u[:, F:]).to(dtype), gelu.cuh's arithmetic
// in one kernel: the standalone GEGLU forward's read of u (2F values per row) and its launch are gone.
// u is still written, because the GEGLU backward (geglu.py:38-52) reads it.  This is the fusion of
// the projection and library/geglu.py's forward (geglu.py:104-108 -> _geglu_fwd, geglu.py:55-61,
// 27-35) that the reference's T5 block runs as `geglu(h @ wi.T)`.
//
// Structure: a persistent grid (one CTA per SM, 12 warps) over output tiles of 128 rows x 128
// F-columns, each an M128 x N256 tcgen05 accumulator whose first 128 columns are the gate
// columns [n0, n0 + 128) and whose last 128 are the matching value columns [F + n0, F + n0 + 128):
//   warp 0      TMA producer: per 64-wide K block, the x tile [128 x 64] and the two W tiles (gate
//               rows, value rows) [128 x 64] each, 128-byte swizzle, into a 4-stage ring;
//   warp 1      TMEM owner (512 columns: two 256-column accumulators) and the MMA issuer: 4 x
//               (M128 N256 K16) per K block, SS, both operands K-major;
//   warps 4-11  epilogue, one row per thread (row = TMEM lane; warps 4-7 take the tile's first 64
//               F-columns, warps 8-11 the last 64), 16 columns at a time: accumulator -> u (bf16/f16,
//               the GEMM output's rounding) -> GEGLU on the rounded values -> the warp's [32 x 16]
//               boxes of u (gate, value) and out staged in shared memory (32-byte swizzle: conflict-
//               free 16-byte writes) -> three TMA stores, so no thread waits on global stores.
// The two accumulators alternate, so tile i's epilogue runs while tile i+1's MMAs do.
// Measured on B200 at [32768 x 1152] x [9216 x 1152]: the mainloop alone runs at 1521 TFLOP/s;
// storing u straight from registers (one row per lane: 32 lines per warp store) held the epilogue
// back to 894 TFLOP/s for the whole op, which the staged TMA stores remove.
// This one-CTA kernel serves up to 128 rows; larger problems run linear_geglu_pair_kernel (below):
// the same roles on tiles of 256 rows shared by the two CTAs of a cluster (cta_group::2), each CTA
// loading half of the operands.  The file also holds the backward, GEGLU's backward in the epilogue
// of the down projection's input gradient (linear_geglu_bwd_kernel, linear_geglu_bwd_pair_kernel).
// Every wait is bounded (watchdog.cuh); a stalled pipeline ends the CTA with an error word.
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "attn_common.cuh"
#include "common.cuh"
#include "gelu.cuh"
#include "watchdog.cuh"

KRSI_DEFINE_WATCHDOG(gemm)

namespace krsi {
namespace {

using namespace sm100;

constexpr int kBM = 128;                 // rows per tile (UMMA M)
constexpr int kBF = 128;                 // F-columns per tile: UMMA N = 2 * kBF (gate | value)
constexpr int kBN = 2 * kBF;
constexpr int kBK = 64;                  // K per stage: one 128-byte swizzle row of 16-bit elements
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4;             // epilogue warps 4..11
constexpr int kEpiWarps = 8;
constexpr uint32_t kATile = kBM * kBK * 2;          // 16 KB
constexpr uint32_t kBTile = kBF * kBK * 2;          // 16 KB per half (gate or value rows)
constexpr uint32_t kStageBytes = kATile + 2 * kBTile;
constexpr int kChunk = 16;                          // F-columns per epilogue step
constexpr uint32_t kBoxBytes = 32 * kChunk * 2;     // one warp's [32 rows x 16 columns] box: 1 KB
constexpr uint32_t kOutOff = kStages * kStageBytes;  // per epilogue warp: u gate, u value, out boxes
constexpr uint32_t kBarOff = kOutOff + kEpiWarps * 3 * kBoxBytes;
// full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr int kNumBars = 2 * kStages + 2 + 2 + 1;
constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;
constexpr uint32_t kSmem = kMiscOff + 16 + 1024;    // + slack for the 1024-byte alignment
constexpr uint32_t kTmemCols = 2 * kBN;
static_assert(kTmemCols <= 512, "TMEM budget");

struct GemmArgs {
  void* u;
  void* out;
  int rows, K, F;
  int n_ftiles;       // F-column tiles
  int n_tiles;        // row tiles x F-column tiles
  int n_kb;           // K blocks
  uint32_t spin_limit;
};

using gelu::Pair;
using gelu::narrow;
using gelu::widen;

// After an abort: wait (bounded) until the last kStages K blocks the producer issued have landed, so
// no TMA load is still writing this CTA's shared memory when it exits.
template <int S>
__device__ __forceinline__ void drain_loads(uint64_t* full, int issued, uint32_t limit) {
  for (int j = issued > S ? issued - S : 0; j < issued; ++j) {
    for (uint32_t n = 0; n < limit && !mbar_try_wait(&full[j % S], (j / S) & 1); ++n) {
    }
  }
}

// K-major operand in the 128-byte swizzle: 8-row groups of 8 x 128 B (SBO = 1024 B); the K step of
// 16 elements inside the swizzle row advances the start address by 32 B.
__device__ __forceinline__ uint64_t kmajor_sw128(uint32_t addr) { return smem_desc(addr, 16, 1024, kSw128); }

// The forward epilogue of one warp (warps kEpiWarp0.. of a CTA): for each of the CTA's tiles, wait for
// its accumulator, read it out 16 columns at a time, hand the accumulator back (`release`), and write u
// and out through staged boxes and TMA stores.  `row_of(i)` is the tile's first row handled by this
// CTA, `col_of(i)` its first F-column.  Returns false after an abort.
template <bool F16, typename RowOf, typename ColOf, typename Release>
__device__ __forceinline__ bool fwd_epilogue(uint8_t* smem, uint32_t tmem, int warp, int lane, int my_tiles,
                                             uint64_t* acc_full, volatile int* abort_flag, const CUtensorMap* ugmap,
                                             const CUtensorMap* uvmap, const CUtensorMap* omap, const GemmArgs& a,
                                             RowOf row_of, ColOf col_of, Release release) {
  const int ew = warp - kEpiWarp0;
  const int quarter = ew % 4;                 // TMEM lane quarter of this warp (warp % 4)
  const int half = ew / 4;                    // which 64 of the tile's 128 F-columns
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  uint8_t* boxes = smem + kOutOff + ew * 3 * kBoxBytes;   // [u gate | u value | out], 32-byte rows
  // this lane's row, 16-byte packet p of a box in the 32-byte swizzle (chunk bit ^= row bit 2)
  auto slot = [&](int box, int p) {
    return reinterpret_cast<uint4*>(boxes + box * kBoxBytes + lane * 32 + ((p ^ ((lane >> 2) & 1)) << 4));
  };
  bool ok = true;
  for (int i = 0; i < my_tiles; ++i) {
    const int acc = i & 1;
    const int row0 = row_of(i) + quarter * 32;   // this warp's first row
    const int c_base = col_of(i) + half * 64;    // first F-column of this warp's 64
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[acc], (i >> 1) & 1, abort_flag, a.spin_limit))) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t acc_addr = tmem + lane_addr + acc * kBN + half * 64;
#pragma unroll 1
    for (int c0 = 0; c0 < 64; c0 += kChunk) {
      uint32_t gv[kChunk], vv[kChunk];
      tmem_ld16(acc_addr + c0, gv);              // gate columns
      tmem_ld16(acc_addr + kBF + c0, vv);        // value columns
      tmem_wait_ld();
      if (c0 + kChunk == 64) {                   // the accumulator has been read: the MMA may reuse it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release(acc);
      }
      // per pair of columns: u rounded as the GEMM output, then gelu.cuh's geglu_out on the
      // rounded values (gel rounded, times the value, rounded) in its paired form
      using P = Pair<F16>;
      uint32_t ug[kChunk / 2], uv[kChunk / 2], o[kChunk / 2];
#pragma unroll
      for (int e = 0; e < kChunk / 2; ++e) {
        ug[e] = P::pack(__uint_as_float(gv[2 * e]), __uint_as_float(gv[2 * e + 1]));
        uv[e] = P::pack(__uint_as_float(vv[2 * e]), __uint_as_float(vv[2 * e + 1]));
        const uint32_t gel = narrow<F16>(gelu::gelu_parts2(widen<F16>(ug[e])).gel);
        o[e] = narrow<F16>(f2_mul(widen<F16>(gel), widen<F16>(uv[e])));
      }
      // the previous step's boxes must have been read by the TMA unit before they are rewritten
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        *slot(0, p) = make_uint4(ug[4 * p], ug[4 * p + 1], ug[4 * p + 2], ug[4 * p + 3]);
        *slot(1, p) = make_uint4(uv[4 * p], uv[4 * p + 1], uv[4 * p + 2], uv[4 * p + 3]);
        *slot(2, p) = make_uint4(o[4 * p], o[4 * p + 1], o[4 * p + 2], o[4 * p + 3]);
      }
      fence_async_shared();                      // staged boxes -> visible to the TMA unit
      __syncwarp();
      const int col = c_base + c0;
      if (lane == 0 && col < a.F && row0 < a.rows) {   // the maps clip rows >= rows and columns >= F
        tma_store_2d(ugmap, boxes, col, row0);
        tma_store_2d(uvmap, boxes + kBoxBytes, col, row0);
        tma_store_2d(omap, boxes + 2 * kBoxBytes, col, row0);
        bulk_commit_group();
      }
    }
  }
  if (lane == 0) bulk_wait_all();               // every store has completed before the CTA exits
  return ok;
}

template <bool F16>
__global__ void __launch_bounds__(kThreads, 1)
linear_geglu_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                    const __grid_constant__ CUtensorMap ugmap, const __grid_constant__ CUtensorMap uvmap,
                    const __grid_constant__ CUtensorMap omap, const GemmArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kMiscOff + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int my_tiles = (int)blockIdx.x < a.n_tiles ? (a.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto tile_of = [&](int i) { return (int)blockIdx.x + i * (int)gridDim.x; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);      // producer's expect_tx arrival + the TMA bytes
      mbar_init(&empty[s], 1);     // tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);            // tcgen05.commit
      mbar_init(&acc_empty[b], kEpiWarps);   // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&wmap);
  }
  if (warp == kEpiWarp0 && lane == 0) {
    prefetch_tensormap(&ugmap);
    prefetch_tensormap(&uvmap);
    prefetch_tensormap(&omap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    bool ok = true;
    int it = 0;   // K blocks issued so far (ring position)
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int t = tile_of(i);
      const int m0 = (t / a.n_ftiles) * kBM, n0 = (t % a.n_ftiles) * kBF;
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kStages;
        if (it >= kStages &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], ((it / kStages) - 1) & 1, abort_flag, a.spin_limit))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(st, &xmap, &full[s], kb * kBK, m0);
          tma_load_2d(st + kATile, &wmap, &full[s], kb * kBK, n0);                  // gate rows
          tma_load_2d(st + kATile + kBTile, &wmap, &full[s], kb * kBK, a.F + n0);   // value rows
        }
        __syncwarp();
      }
    }
    if (!ok) {
      watchdog_fire(kWdGemmLoad);
      drain_loads<kStages>(full, it, a.spin_limit);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp, elected lane)
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.spin_limit));
    };
    constexpr uint32_t idesc = idesc_f16(kBM, kBN, F16 ? 0u : 1u, false, false);
    const uint64_t desc0 = kmajor_sw128(smem_u32(smem));
    constexpr uint64_t kStageStep = kStageBytes >> 4;
    constexpr uint64_t kBStep = kATile >> 4;
    constexpr uint64_t kKStep = 32 >> 4;   // 16 elements of 2 bytes
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int acc = i & 1;
      if (i >= 2 && !wait(&acc_empty[acc], ((i >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kBN;
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kStages;
        if (!wait(&full[s], (it / kStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = desc0 + (uint64_t)s * kStageStep;
        const uint64_t bd = ad + kBStep;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_ss_e(d, ad + kk * kKStep, bd + kk * kKStep, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit_e(&empty[s]);   // the stage is free once these MMAs have read it
      }
      if (!ok) break;
      mma_commit_e(&acc_full[acc]);
    }
    if (!ok && my_tiles > 0) watchdog_fire(kWdGemmMma);
    // Drain: every MMA issued above has completed before TMEM is released.
    mma_commit_e(drain);
    for (uint32_t i = 0; i < a.spin_limit && !mbar_try_wait(drain, 0); ++i) {
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const bool ok = fwd_epilogue<F16>(
        smem, tmem, warp, lane, my_tiles, acc_full, abort_flag, &ugmap, &uvmap, &omap, a,
        [&](int i) { return (tile_of(i) / a.n_ftiles) * kBM; }, [&](int i) { return (tile_of(i) % a.n_ftiles) * kBF; },
        [&](int acc) { mbar_arrive(&acc_empty[acc]); });
    if (!ok) watchdog_fire(kWdGemmEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------- forward on CTA pairs (cta_group::2)
// The same op on tiles of 256 rows x 128 F-columns shared by the two CTAs of a cluster: each CTA loads
// its own 128 rows of x and half of the W tile (the even CTA the gate rows, the odd CTA the value
// rows), 32 KB per K block instead of 48, and the even CTA issues M256 N256 K16 MMAs that read both
// CTAs' shared memory and accumulate into both CTAs' TMEM (its 128 rows x [gate | value] each).  Both
// CTAs' loads complete on the even CTA's stage barriers; the even CTA's MMA completions are signalled
// to the barriers of both; both CTAs' epilogue warps hand the accumulator back to the even CTA.  Six
// stages fit where four did, so more of the operand stream is in flight (the one-CTA kernel's MMA
// warp waits for operands ~55% of each tile).
constexpr int kPairStages = 6;
constexpr uint32_t kPairStageBytes = kATile + kBTile;              // 128 rows of x + 128 rows of W
constexpr uint32_t kPairOutOff = kPairStages * kPairStageBytes;
static_assert(kPairOutOff == kOutOff, "the forward epilogue's boxes sit at the same offset");
constexpr uint32_t kPairBarOff = kPairOutOff + kEpiWarps * 3 * kBoxBytes;
// full[S] (used in the even CTA), empty[S], acc_full[2], acc_empty[2] (even CTA), drain (even CTA)
constexpr int kPairNumBars = 2 * kPairStages + 2 + 2 + 1;
constexpr uint32_t kPairMiscOff = kPairBarOff + kPairNumBars * 8;
constexpr uint32_t kPairSmem = kPairMiscOff + 16 + 1024;
static_assert(kPairSmem <= 232448, "shared memory budget");

template <bool F16>
__global__ void __launch_bounds__(kThreads, 1)
linear_geglu_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                         const __grid_constant__ CUtensorMap ugmap, const __grid_constant__ CUtensorMap uvmap,
                         const __grid_constant__ CUtensorMap omap, const GemmArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPairStages;
  uint64_t* acc_full = bars + 2 * kPairStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kPairMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kPairMiscOff + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  const int pair = (int)blockIdx.x / 2, n_pairs = (int)gridDim.x / 2;
  const int my_tiles = pair < a.n_tiles ? (a.n_tiles - 1 - pair) / n_pairs + 1 : 0;
  auto tile_of = [&](int i) { return pair + i * n_pairs; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);      // the even CTA's expect_tx arrival + both CTAs' TMA bytes
      mbar_init(&empty[s], 1);     // the even CTA's tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);                // the even CTA's tcgen05.commit
      mbar_init(&acc_empty[b], 2 * kEpiWarps);   // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&wmap);
  }
  if (warp == kEpiWarp0 && lane == 0) {
    prefetch_tensormap(&ugmap);
    prefetch_tensormap(&uvmap);
    prefetch_tensormap(&omap);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();   // both CTAs' barriers initialised and TMEM allocated before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int t = tile_of(i);
      const int m0 = (t / a.n_ftiles) * (2 * kBM) + (int)rank * kBM, n0 = (t % a.n_ftiles) * kBF;
      const int wrow = even ? n0 : a.F + n0;   // the even CTA holds the gate rows, the odd the value rows
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kPairStages;
        if (it >= kPairStages && !__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], ((it / kPairStages) - 1) & 1,
                                                                            abort_flag, a.spin_limit))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * kPairStageBytes;
          const uint32_t bar = mapa_shared(&full[s], 0);
          if (even) mbar_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
          tma_load_2d_pair(st, &xmap, bar, kb * kBK, m0);
          tma_load_2d_pair(st + kATile, &wmap, bar, kb * kBK, wrow);
        }
        __syncwarp();
      }
    }
    if (!ok) {
      watchdog_fire(kWdGemmLoad);
      if (even) drain_loads<kPairStages>(full, it, a.spin_limit);   // covers both CTAs' loads of each stage
    }
  } else if (warp == 1 && even) {
    // ------------------------------------------------------------ MMA issuer (even CTA, elected lane)
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.spin_limit));
    };
    constexpr uint32_t idesc = idesc_f16(2 * kBM, kBN, F16 ? 0u : 1u, false, false);
    const uint64_t desc0 = kmajor_sw128(smem_u32(smem));
    constexpr uint64_t kStageStep = kPairStageBytes >> 4;
    constexpr uint64_t kBStep = kATile >> 4;
    constexpr uint64_t kKStep = 32 >> 4;
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int acc = i & 1;
      if (i >= 2 && !wait(&acc_empty[acc], ((i >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kBN;
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kPairStages;
        if (!wait(&full[s], (it / kPairStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = desc0 + (uint64_t)s * kStageStep;
        const uint64_t bd = ad + kBStep;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_ss_pair_e(d, ad + kk * kKStep, bd + kk * kKStep, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit_pair_e(mapa_shared(&empty[s], 0));   // stage s free in both CTAs
        mma_commit_pair_e(mapa_shared(&empty[s], 1));
      }
      if (!ok) break;
      mma_commit_pair_e(mapa_shared(&acc_full[acc], 0));
      mma_commit_pair_e(mapa_shared(&acc_full[acc], 1));
    }
    if (!ok && my_tiles > 0) watchdog_fire(kWdGemmMma);
    mma_commit_pair_e(mapa_shared(drain, 0));
    for (uint32_t i = 0; i < a.spin_limit && !mbar_try_wait(drain, 0); ++i) {
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue (both CTAs, own rows)
    const bool ok = fwd_epilogue<F16>(
        smem, tmem, warp, lane, my_tiles, acc_full, abort_flag, &ugmap, &uvmap, &omap, a,
        [&](int i) { return (tile_of(i) / a.n_ftiles) * (2 * kBM) + (int)rank * kBM; },
        [&](int i) { return (tile_of(i) % a.n_ftiles) * kBF; },
        [&](int acc) {
          if (even) mbar_arrive(&acc_empty[acc]);
          else mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
        });
    if (!ok) watchdog_fire(kWdGemmEpilogue);
  }

  tc_fence_before();
  cluster_sync();   // the even CTA's MMAs (which read this CTA's shared memory and TMEM) are done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// ---------------------------------------------------------------- backward: du = geglu_bwd(dy @ w, u)
// The down projection's input gradient g = dy @ w (dy [rows, K], w [K, F]: the down projection's
// nn.Linear weight, read MN-major) with GEGLU's backward in the epilogue: g never goes to memory.
// Tiles of 128 rows x 256 F-columns; per K block the dy tile [128 x 64] (K-major) and four w boxes
// [64 K-rows x 64 columns] (MN-major), 48 KB per stage.  Each epilogue warp owns 32 rows x 128
// columns, 16 at a time: its u-gate and u-value boxes arrive by TMA (the next step's are requested as
// soon as the current ones are in registers), g comes from TMEM rounded as the GEMM output, and
// du-gate, du-value leave through staged boxes and TMA stores.
// The u boxes come from HBM (u was written a whole forward ago), about a microsecond away, and a step
// takes less: each warp keeps a ring of three u slots with the next two steps' loads in flight.  The
// ring's 48 KB come out of the operand ring, which has three stages here (measured with one u slot:
// every step waited for its own load, 449 us per call at the block's shape).
constexpr int kBwdBN = 256;                                   // F-columns per tile (UMMA N)
constexpr int kBwdStages = 3;
constexpr int kUSlots = 3;                                    // u boxes per epilogue warp: 2 loads ahead
constexpr uint32_t kBwdWBox = 64 * kBK * 2;                   // one [64 K-rows x 64 columns] w box: 8 KB
constexpr uint32_t kBwdStageBytes = kATile + 4 * kBwdWBox;
constexpr uint32_t kBwdIoBytes = (2 * kUSlots + 2) * kBoxBytes;   // per epilogue warp: u slots, du gate, du value
constexpr uint32_t kBwdIoOff = kBwdStages * kBwdStageBytes;
constexpr uint32_t kBwdBarOff = kBwdIoOff + kEpiWarps * kBwdIoBytes;
// full[S], empty[S], acc_full[2], acc_empty[2], drain, u_full[epilogue warps][slots]
constexpr int kBwdNumBars = 2 * kBwdStages + 2 + 2 + 1 + kEpiWarps * kUSlots;
constexpr uint32_t kBwdMiscOff = kBwdBarOff + kBwdNumBars * 8;
constexpr uint32_t kBwdSmem = kBwdMiscOff + 16 + 1024;
static_assert(kBwdSmem <= 232448, "shared memory budget");

// MN-major operand in the 128-byte swizzle: 64-column atoms of 8 K-rows x 128 B (SBO = 1024 B), the
// next 64 columns one box further (LBO = 8 KB); the K step of 16 rows advances the start by 2 KB.
__device__ __forceinline__ uint64_t mnmajor_sw128(uint32_t addr) { return smem_desc(addr, kBwdWBox, 1024, kSw128); }

// The backward epilogue of one warp (warps kEpiWarp0.. of a CTA, NG groups of 4 warps): for each of
// the CTA's tiles, read g out of TMEM 16 columns at a time (group g takes the 16-column chunks g,
// g + NG, ...), hand the accumulator back (`release`), bring in the matching u boxes through a ring
// of kUSlots (`io_base`: this CTA's per-warp boxes, `u_full`: their barriers), and write du through
// staged boxes and TMA stores.  `row_of(i)` is the tile's first row handled by this CTA,
// `col_base_of(i)` its first F-column.  Returns false after an abort.
template <bool F16, int NG, typename RowOf, typename ColOf, typename Release>
__device__ __forceinline__ bool bwd_epilogue(uint8_t* io_base, uint64_t* u_full, uint32_t tmem, int warp, int lane,
                                             int my_tiles, uint64_t* acc_full, volatile int* abort_flag,
                                             const CUtensorMap* ugmap, const CUtensorMap* uvmap,
                                             const CUtensorMap* dugmap, const CUtensorMap* duvmap, const GemmArgs& a,
                                             RowOf row_of, ColOf col_base_of, Release release) {
  using P = Pair<F16>;
  constexpr int kChunks = kBwdBN / kChunk;    // 16-column chunks per tile
  const int ew = warp - kEpiWarp0;
  const int quarter = ew % 4;
  const int grp = ew / 4;                     // chunks grp, grp + NG, ...
  const int kSteps = (kChunks - grp + NG - 1) / NG;   // this warp's chunks per tile
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  uint8_t* io = io_base + ew * kBwdIoBytes;   // [slot][u gate | u value], then du gate, du value
  uint8_t* du_boxes = io + 2 * kUSlots * kBoxBytes;
  uint64_t* ubar = &u_full[ew * kUSlots];
  const int n_steps = my_tiles * kSteps;
  auto slot = [&](uint8_t* box, int p) {
    return reinterpret_cast<uint4*>(box + lane * 32 + ((p ^ ((lane >> 2) & 1)) << 4));
  };
  auto row0_of = [&](int i) { return row_of(i) + quarter * 32; };
  auto col_of = [&](int i, int c) { return col_base_of(i) + (grp + NG * c) * kChunk; };
  // step q's u boxes (gate and value columns of this warp's rows; zero past rows or F) into slot q % 3
  auto load_u = [&](int q) {
    if (lane == 0) {
      const int i = q / kSteps, c = q % kSteps, r = q % kUSlots;
      uint8_t* box = io + r * 2 * kBoxBytes;
      mbar_arrive_expect_tx(&ubar[r], 2 * kBoxBytes);
      tma_load_2d(box, ugmap, &ubar[r], col_of(i, c), row0_of(i));
      tma_load_2d(box + kBoxBytes, uvmap, &ubar[r], col_of(i, c), row0_of(i));
    }
  };
  int issued = 0;             // u loads issued (steps 0 .. issued - 1)
  for (; issued < kUSlots - 1 && issued < n_steps; ++issued) load_u(issued);
  bool ok = true;
  int q = 0;                  // steps whose u has arrived
  for (int i = 0; i < my_tiles && ok; ++i) {
    const int acc = i & 1;
    const int row0 = row0_of(i);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[acc], (i >> 1) & 1, abort_flag, a.spin_limit))) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t acc_addr = tmem + lane_addr + acc * kBwdBN;
#pragma unroll 1
    for (int c = 0; c < kSteps; ++c) {
      uint32_t gv[kChunk];
      tmem_ld16(acc_addr + (grp + NG * c) * kChunk, gv);
      tmem_wait_ld();
      if (c + 1 == kSteps) {                  // the accumulator has been read: the MMA may reuse it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release(acc);
      }
      const int r = q % kUSlots;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&ubar[r], (q / kUSlots) & 1, abort_flag, a.spin_limit))) {
        ok = false;
        break;
      }
      ++q;
      uint8_t* ubox = io + r * 2 * kBoxBytes;
      uint4 av[2], bv[2];
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2) {
        av[p2] = *slot(ubox, p2);
        bv[p2] = *slot(ubox + kBoxBytes, p2);
      }
      __syncwarp();                           // every lane has its u: slot r may be refilled
      if (issued < n_steps) load_u(issued++); // two steps ahead, into the slot read one step ago
      const uint32_t aw[8] = {av[0].x, av[0].y, av[0].z, av[0].w, av[1].x, av[1].y, av[1].z, av[1].w};
      const uint32_t bw[8] = {bv[0].x, bv[0].y, bv[0].z, bv[0].w, bv[1].x, bv[1].y, bv[1].z, bv[1].w};
      // per pair of columns: g rounded as the GEMM output, then gelu.cuh's geglu_grad arithmetic in
      // its paired form
      uint32_t dg[kChunk / 2], dv[kChunk / 2];
#pragma unroll
      for (int e = 0; e < kChunk / 2; ++e) {
        const uint64_t g2 = widen<F16>(P::pack(__uint_as_float(gv[2 * e]), __uint_as_float(gv[2 * e + 1])));
        const uint64_t a2 = widen<F16>(aw[e]);
        const gelu::GeluParts2 pp = gelu::gelu_parts2(a2);
        dv[e] = narrow<F16>(f2_mul(g2, widen<F16>(narrow<F16>(pp.gel))));                  // db
        const uint64_t dgel = widen<F16>(narrow<F16>(f2_mul(g2, widen<F16>(bw[e]))));
        dg[e] = narrow<F16>(gelu::geglu_dgate2(a2, pp.t, dgel));
      }
      if (lane == 0) bulk_wait_read_all();    // the previous step's du boxes have been read
      __syncwarp();
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2) {
        *slot(du_boxes, p2) = make_uint4(dg[4 * p2], dg[4 * p2 + 1], dg[4 * p2 + 2], dg[4 * p2 + 3]);
        *slot(du_boxes + kBoxBytes, p2) = make_uint4(dv[4 * p2], dv[4 * p2 + 1], dv[4 * p2 + 2], dv[4 * p2 + 3]);
      }
      fence_async_shared();
      __syncwarp();
      const int col = col_of(i, c);
      if (lane == 0 && col < a.F && row0 < a.rows) {
        tma_store_2d(dugmap, du_boxes, col, row0);
        tma_store_2d(duvmap, du_boxes + kBoxBytes, col, row0);
        bulk_commit_group();
      }
    }
  }
  for (int j = q; j < issued; ++j)            // after an abort: the u loads in flight land first
    for (uint32_t n = 0; n < a.spin_limit && !mbar_try_wait(&ubar[j % kUSlots], (j / kUSlots) & 1); ++n) {
    }
  if (lane == 0) bulk_wait_all();
  return ok;
}

template <bool F16>
__global__ void __launch_bounds__(kThreads, 1)
linear_geglu_bwd_kernel(const __grid_constant__ CUtensorMap dymap, const __grid_constant__ CUtensorMap wmap,
                        const __grid_constant__ CUtensorMap ugmap, const __grid_constant__ CUtensorMap uvmap,
                        const __grid_constant__ CUtensorMap dugmap, const __grid_constant__ CUtensorMap duvmap,
                        const GemmArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBwdBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kBwdStages;
  uint64_t* acc_full = bars + 2 * kBwdStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* u_full = drain + 1;   // [epilogue warp][slot]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kBwdMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kBwdMiscOff + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int my_tiles = (int)blockIdx.x < a.n_tiles ? (a.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto tile_of = [&](int i) { return (int)blockIdx.x + i * (int)gridDim.x; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int w = 0; w < kEpiWarps * kUSlots; ++w) mbar_init(&u_full[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&dymap);
    prefetch_tensormap(&wmap);
  }
  if (warp == kEpiWarp0 && lane == 0) {
    prefetch_tensormap(&ugmap);
    prefetch_tensormap(&uvmap);
    prefetch_tensormap(&dugmap);
    prefetch_tensormap(&duvmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int t = tile_of(i);
      const int m0 = (t / a.n_ftiles) * kBM, n0 = (t % a.n_ftiles) * kBwdBN;
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kBwdStages;
        if (it >= kBwdStages && !__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], ((it / kBwdStages) - 1) & 1,
                                                                            abort_flag, a.spin_limit))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * kBwdStageBytes;
          mbar_arrive_expect_tx(&full[s], kBwdStageBytes);
          tma_load_2d(st, &dymap, &full[s], kb * kBK, m0);
#pragma unroll
          for (int j = 0; j < 4; ++j)   // w rows (K) kb*64.., columns n0 + 64 j..
            tma_load_2d(st + kATile + j * kBwdWBox, &wmap, &full[s], n0 + 64 * j, kb * kBK);
        }
        __syncwarp();
      }
    }
    if (!ok) {
      watchdog_fire(kWdGemmLoad);
      drain_loads<kBwdStages>(full, it, a.spin_limit);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.spin_limit));
    };
    constexpr uint32_t idesc = idesc_f16(kBM, kBwdBN, F16 ? 0u : 1u, false, true);   // w MN-major
    const uint64_t adesc0 = kmajor_sw128(smem_u32(smem));
    const uint64_t bdesc0 = mnmajor_sw128(smem_u32(smem + kATile));
    constexpr uint64_t kStageStep = kBwdStageBytes >> 4;
    constexpr uint64_t kAKStep = 32 >> 4;             // 16 K-columns of 2 bytes
    constexpr uint64_t kBKStep = (16 * 128) >> 4;     // 16 K-rows of 128 bytes
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int acc = i & 1;
      if (i >= 2 && !wait(&acc_empty[acc], ((i >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kBwdBN;
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kBwdStages;
        if (!wait(&full[s], (it / kBwdStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = adesc0 + (uint64_t)s * kStageStep;
        const uint64_t bd = bdesc0 + (uint64_t)s * kStageStep;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_ss_e(d, ad + kk * kAKStep, bd + kk * kBKStep, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit_e(&empty[s]);
      }
      if (!ok) break;
      mma_commit_e(&acc_full[acc]);
    }
    if (!ok && my_tiles > 0) watchdog_fire(kWdGemmMma);
    mma_commit_e(drain);
    for (uint32_t i = 0; i < a.spin_limit && !mbar_try_wait(drain, 0); ++i) {
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const bool ok = bwd_epilogue<F16, kEpiWarps / 4>(
        smem + kBwdIoOff, u_full, tmem, warp, lane, my_tiles, acc_full, abort_flag, &ugmap, &uvmap, &dugmap, &duvmap, a,
        [&](int i) { return (tile_of(i) / a.n_ftiles) * kBM; }, [&](int i) { return (tile_of(i) % a.n_ftiles) * kBwdBN; },
        [&](int acc) { mbar_arrive(&acc_empty[acc]); });
    if (!ok) watchdog_fire(kWdGemmEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------- backward on CTA pairs (cta_group::2)
// The backward on tiles of 256 rows x 256 F-columns shared by a cluster of two: each CTA loads its own
// 128 rows of dy and half of the w columns (two 64-column boxes: the even CTA the first 128 columns of
// the tile, the odd CTA the last 128), 32 KB per K block, five stages beside the epilogue's u/du boxes;
// the even CTA issues M256 N256 K16 MMAs; each CTA's epilogue finishes its own 128 rows.
// The epilogue (the GELU derivative on every element) bounds this kernel, so it runs 12 warps, three
// per scheduler, where the operand stages' smaller footprint leaves room for their boxes.
constexpr int kPairBwdStages = 4;
constexpr int kPairBwdEpiWarps = 12;
constexpr int kPairBwdThreads = (kEpiWarp0 + kPairBwdEpiWarps) * 32;   // 512: 128 registers per thread
constexpr uint32_t kPairBwdStageBytes = kATile + 2 * kBwdWBox;
constexpr uint32_t kPairBwdIoOff = kPairBwdStages * kPairBwdStageBytes;
constexpr uint32_t kPairBwdBarOff = kPairBwdIoOff + kPairBwdEpiWarps * kBwdIoBytes;
constexpr int kPairBwdNumBars = 2 * kPairBwdStages + 2 + 2 + 1 + kPairBwdEpiWarps * kUSlots;
constexpr uint32_t kPairBwdMiscOff = kPairBwdBarOff + kPairBwdNumBars * 8;
constexpr uint32_t kPairBwdSmem = kPairBwdMiscOff + 16 + 1024;
static_assert(kPairBwdSmem <= 232448, "shared memory budget");

template <bool F16>
__global__ void __launch_bounds__(kPairBwdThreads, 1)
linear_geglu_bwd_pair_kernel(const __grid_constant__ CUtensorMap dymap, const __grid_constant__ CUtensorMap wmap,
                             const __grid_constant__ CUtensorMap ugmap, const __grid_constant__ CUtensorMap uvmap,
                             const __grid_constant__ CUtensorMap dugmap, const __grid_constant__ CUtensorMap duvmap,
                             const GemmArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPairBwdBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPairBwdStages;
  uint64_t* acc_full = bars + 2 * kPairBwdStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* u_full = drain + 1;   // [epilogue warp][slot]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kPairBwdMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kPairBwdMiscOff + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  const int pair = (int)blockIdx.x / 2, n_pairs = (int)gridDim.x / 2;
  const int my_tiles = pair < a.n_tiles ? (a.n_tiles - 1 - pair) / n_pairs + 1 : 0;
  auto tile_of = [&](int i) { return pair + i * n_pairs; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairBwdStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kPairBwdEpiWarps);
    }
    mbar_init(drain, 1);
    for (int w = 0; w < kPairBwdEpiWarps * kUSlots; ++w) mbar_init(&u_full[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&dymap);
    prefetch_tensormap(&wmap);
  }
  if (warp == kEpiWarp0 && lane == 0) {
    prefetch_tensormap(&ugmap);
    prefetch_tensormap(&uvmap);
    prefetch_tensormap(&dugmap);
    prefetch_tensormap(&duvmap);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int t = tile_of(i);
      const int m0 = (t / a.n_ftiles) * (2 * kBM) + (int)rank * kBM;
      const int n0 = (t % a.n_ftiles) * kBwdBN + (int)rank * (kBwdBN / 2);   // this CTA's 128 columns
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kPairBwdStages;
        if (it >= kPairBwdStages && !__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], ((it / kPairBwdStages) - 1) & 1,
                                                                                abort_flag, a.spin_limit))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * kPairBwdStageBytes;
          const uint32_t bar = mapa_shared(&full[s], 0);
          if (even) mbar_arrive_expect_tx(&full[s], 2 * kPairBwdStageBytes);
          tma_load_2d_pair(st, &dymap, bar, kb * kBK, m0);
          tma_load_2d_pair(st + kATile, &wmap, bar, n0, kb * kBK);
          tma_load_2d_pair(st + kATile + kBwdWBox, &wmap, bar, n0 + 64, kb * kBK);
        }
        __syncwarp();
      }
    }
    if (!ok) {
      watchdog_fire(kWdGemmLoad);
      if (even) drain_loads<kPairBwdStages>(full, it, a.spin_limit);
    }
  } else if (warp == 1 && even) {
    // ------------------------------------------------------------ MMA issuer (even CTA, elected lane)
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, a.spin_limit));
    };
    constexpr uint32_t idesc = idesc_f16(2 * kBM, kBwdBN, F16 ? 0u : 1u, false, true);   // w MN-major
    const uint64_t adesc0 = kmajor_sw128(smem_u32(smem));
    const uint64_t bdesc0 = mnmajor_sw128(smem_u32(smem + kATile));
    constexpr uint64_t kStageStep = kPairBwdStageBytes >> 4;
    constexpr uint64_t kAKStep = 32 >> 4;
    constexpr uint64_t kBKStep = (16 * 128) >> 4;
    bool ok = true;
    int it = 0;
    for (int i = 0; i < my_tiles && ok; ++i) {
      const int acc = i & 1;
      if (i >= 2 && !wait(&acc_empty[acc], ((i >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + acc * kBwdBN;
      for (int kb = 0; kb < a.n_kb; ++kb, ++it) {
        const int s = it % kPairBwdStages;
        if (!wait(&full[s], (it / kPairBwdStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = adesc0 + (uint64_t)s * kStageStep;
        const uint64_t bd = bdesc0 + (uint64_t)s * kStageStep;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_ss_pair_e(d, ad + kk * kAKStep, bd + kk * kBKStep, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        mma_commit_pair_e(mapa_shared(&empty[s], 0));
        mma_commit_pair_e(mapa_shared(&empty[s], 1));
      }
      if (!ok) break;
      mma_commit_pair_e(mapa_shared(&acc_full[acc], 0));
      mma_commit_pair_e(mapa_shared(&acc_full[acc], 1));
    }
    if (!ok && my_tiles > 0) watchdog_fire(kWdGemmMma);
    mma_commit_pair_e(mapa_shared(drain, 0));
    for (uint32_t i = 0; i < a.spin_limit && !mbar_try_wait(drain, 0); ++i) {
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue (both CTAs, own rows)
    const bool ok = bwd_epilogue<F16, kPairBwdEpiWarps / 4>(
        smem + kPairBwdIoOff, u_full, tmem, warp, lane, my_tiles, acc_full, abort_flag, &ugmap, &uvmap, &dugmap,
        &duvmap, a, [&](int i) { return (tile_of(i) / a.n_ftiles) * (2 * kBM) + (int)rank * kBM; },
        [&](int i) { return (tile_of(i) % a.n_ftiles) * kBwdBN; },
        [&](int acc) {
          if (even) mbar_arrive(&acc_empty[acc]);
          else mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
        });
    if (!ok) watchdog_fire(kWdGemmEpilogue);
  }

  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// 2-D view (cols, rows) of a row-major 16-bit matrix with `pitch` elements between rows, copied in
// boxes of box_cols x box_rows with the given swizzle.  Loads read elements past cols or rows as
// zero; stores skip them.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t pitch, bool f16,
              uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  attn::EncodeTiledFn enc = attn::encode_fn();
  if (!enc) return false;
  memset(map, 0, sizeof(*map));
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)pitch * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}
// The three box shapes: K-major operand tiles [128 rows x 64] (128-byte swizzle), MN-major weight tiles
// [64 K-rows x 64 columns] (128-byte swizzle), and the epilogue's per-warp [32 rows x 16] boxes
// (32-byte swizzle).
bool operand_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, bool f16) {
  return make_map(m, base, rows, cols, cols, f16, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
}
bool mn_operand_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, bool f16) {
  return make_map(m, base, rows, cols, cols, f16, 64, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
}
bool box_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t pitch, bool f16) {
  return make_map(m, base, rows, cols, pitch, f16, kChunk, 32, CU_TENSOR_MAP_SWIZZLE_32B);
}

// Clusters of two of the pair kernel that fit on the device at once (0: no pair launch possible), per
// device, queried once.
// KRSI_GEMM_PAIRS=0 in the environment runs the one-CTA kernels for every size (for a device partition
// that cannot schedule clusters of two, or to compare the two paths, which give the same bits).  Read
// on every call.
inline bool pairs_enabled() {
  const char* v = getenv("KRSI_GEMM_PAIRS");
  return v == nullptr || strcmp(v, "0") != 0;
}

template <bool F16>
int pair_clusters() {
  static std::atomic<int> cached[64];   // clusters + 1 once queried (0: not yet); races only repeat the query
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    auto kern = linear_geglu_pair_kernel<F16>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmem) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (device_sm_count() / 2));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kPairSmem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();   // a refused query leaves no sticky error behind
    v = n + 1;
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v - 1;
}

template <bool F16>
int launch_pair(const CUtensorMap& xm, const CUtensorMap& wm, const CUtensorMap& ugm, const CUtensorMap& uvm,
                const CUtensorMap& om, const GemmArgs& a, int max_clusters, cudaStream_t stream) {
  auto kern = linear_geglu_pair_kernel<F16>;
  const int clusters = a.n_tiles < max_clusters ? a.n_tiles : max_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  KRSI_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, xm, wm, ugm, uvm, om, a));
  return KRSI_OK;
}

template <bool F16>
int launch(const CUtensorMap& xm, const CUtensorMap& wm, const CUtensorMap& ugm, const CUtensorMap& uvm,
           const CUtensorMap& om, const GemmArgs& a, cudaStream_t stream) {
  auto kern = linear_geglu_kernel<F16>;
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  const int grid = a.n_tiles < device_sm_count() ? a.n_tiles : device_sm_count();
  KRSI_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(kThreads), kSmem, stream, xm, wm, ugm, uvm, om, a));
  return KRSI_OK;
}

template <bool F16>
int bwd_pair_clusters() {
  static std::atomic<int> cached[64];   // clusters + 1 once queried (0: not yet); races only repeat the query
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    auto kern = linear_geglu_bwd_pair_kernel<F16>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairBwdSmem) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (device_sm_count() / 2));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kPairBwdSmem;
      cfg.blockDim = dim3(kPairBwdThreads);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    v = n + 1;
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v - 1;
}

template <bool F16>
int launch_bwd_pair(const CUtensorMap& dym, const CUtensorMap& wm, const CUtensorMap& ugm, const CUtensorMap& uvm,
                    const CUtensorMap& dugm, const CUtensorMap& duvm, const GemmArgs& a, int max_clusters,
                    cudaStream_t stream) {
  auto kern = linear_geglu_bwd_pair_kernel<F16>;
  const int clusters = a.n_tiles < max_clusters ? a.n_tiles : max_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kPairBwdThreads);
  cfg.dynamicSmemBytes = kPairBwdSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  KRSI_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, dym, wm, ugm, uvm, dugm, duvm, a));
  return KRSI_OK;
}

template <bool F16>
int launch_bwd(const CUtensorMap& dym, const CUtensorMap& wm, const CUtensorMap& ugm, const CUtensorMap& uvm,
               const CUtensorMap& dugm, const CUtensorMap& duvm, const GemmArgs& a, cudaStream_t stream) {
  auto kern = linear_geglu_bwd_kernel<F16>;
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBwdSmem));
  const int grid = a.n_tiles < device_sm_count() ? a.n_tiles : device_sm_count();
  KRSI_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(kThreads), kBwdSmem, stream, dym, wm, ugm, uvm, dugm, duvm, a));
  return KRSI_OK;
}

}  // namespace
}  // namespace krsi

using namespace krsi;

extern "C" int krsi_linear_geglu_fwd(const void* x, const void* w, void* u, void* out, int64_t rows, int64_t K,
                                     int64_t F, int dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && K > 0 && F > 0);
  if (rows == 0) return KRSI_OK;
  KRSI_CHECK_ARG(x && w && u && out);
  if (dtype != KRSI_BF16 && dtype != KRSI_F16) return KRSI_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and row strides (K % 8); epilogue: 16-byte packets of 8 columns (F % 8)
  if (K % 8 != 0 || F % 8 != 0) return KRSI_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w) || !aligned16(u) || !aligned16(out)) return KRSI_ERR_MISALIGNED;
  if (rows > INT32_MAX - kBM || K > INT32_MAX || 2 * F > INT32_MAX - kBF) return KRSI_ERR_UNSUPPORTED;
  const bool f16 = dtype == KRSI_F16;
  CUtensorMap xm, wm, ugm, uvm, om;
  const size_t esz = 2;
  if (!operand_map(&xm, x, rows, K, f16) || !operand_map(&wm, w, 2 * F, K, f16) ||
      !box_map(&ugm, u, rows, F, 2 * F, f16) || !box_map(&uvm, static_cast<const char*>(u) + F * esz, rows, F, 2 * F, f16) ||
      !box_map(&om, out, rows, F, F, f16))
    return KRSI_ERR_CUDA;
  const int64_t n_rt = (rows + kBM - 1) / kBM, n_ft = (F + kBF - 1) / kBF;
  if (n_rt * n_ft > INT32_MAX) return KRSI_ERR_UNSUPPORTED;
  GemmArgs a{u, out, (int)rows, (int)K, (int)F, (int)n_ft, (int)(n_rt * n_ft), (int)((K + kBK - 1) / kBK),
             kSpinLimit};
  // More than one row tile: CTA pairs (M = 256 tiles), when the device runs clusters of two of them.
  const int clusters = rows > kBM && pairs_enabled() ? (f16 ? pair_clusters<true>() : pair_clusters<false>()) : 0;
  if (clusters > 0) {
    GemmArgs pa = a;
    pa.n_tiles = (int)(((rows + 2 * kBM - 1) / (2 * kBM)) * n_ft);
    return f16 ? launch_pair<true>(xm, wm, ugm, uvm, om, pa, clusters, stream)
               : launch_pair<false>(xm, wm, ugm, uvm, om, pa, clusters, stream);
  }
  return f16 ? launch<true>(xm, wm, ugm, uvm, om, a, stream) : launch<false>(xm, wm, ugm, uvm, om, a, stream);
}

extern "C" int krsi_linear_geglu_bwd(const void* dy, const void* w, const void* u, void* du, int64_t rows,
                                     int64_t K, int64_t F, int dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(rows >= 0 && K > 0 && F > 0);
  if (rows == 0) return KRSI_OK;
  KRSI_CHECK_ARG(dy && w && u && du);
  if (dtype != KRSI_BF16 && dtype != KRSI_F16) return KRSI_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and row strides (K % 8 for dy, F % 8 for w, u and du)
  if (K % 8 != 0 || F % 8 != 0) return KRSI_ERR_UNSUPPORTED;
  if (!aligned16(dy) || !aligned16(w) || !aligned16(u) || !aligned16(du)) return KRSI_ERR_MISALIGNED;
  if (rows > INT32_MAX - kBM || K > INT32_MAX - kBK || 2 * F > INT32_MAX - kBwdBN) return KRSI_ERR_UNSUPPORTED;
  const bool f16 = dtype == KRSI_F16;
  const size_t esz = 2;
  CUtensorMap dym, wm, ugm, uvm, dugm, duvm;
  if (!operand_map(&dym, dy, rows, K, f16) || !mn_operand_map(&wm, w, K, F, f16) ||
      !box_map(&ugm, u, rows, F, 2 * F, f16) || !box_map(&uvm, static_cast<const char*>(u) + F * esz, rows, F, 2 * F, f16) ||
      !box_map(&dugm, du, rows, F, 2 * F, f16) ||
      !box_map(&duvm, static_cast<char*>(du) + F * esz, rows, F, 2 * F, f16))
    return KRSI_ERR_CUDA;
  const int64_t n_rt = (rows + kBM - 1) / kBM, n_ft = (F + kBwdBN - 1) / kBwdBN;
  if (n_rt * n_ft > INT32_MAX) return KRSI_ERR_UNSUPPORTED;
  GemmArgs a{nullptr, du, (int)rows, (int)K, (int)F, (int)n_ft, (int)(n_rt * n_ft), (int)((K + kBK - 1) / kBK),
             kSpinLimit};
  const int clusters =
      rows > kBM && pairs_enabled() ? (f16 ? bwd_pair_clusters<true>() : bwd_pair_clusters<false>()) : 0;
  if (clusters > 0) {
    GemmArgs pa = a;
    pa.n_tiles = (int)(((rows + 2 * kBM - 1) / (2 * kBM)) * n_ft);
    return f16 ? launch_bwd_pair<true>(dym, wm, ugm, uvm, dugm, duvm, pa, clusters, stream)
               : launch_bwd_pair<false>(dym, wm, ugm, uvm, dugm, duvm, pa, clusters, stream);
  }
  return f16 ? launch_bwd<true>(dym, wm, ugm, uvm, dugm, duvm, a, stream)
             : launch_bwd<false>(dym, wm, ugm, uvm, dugm, duvm, a, stream);
}
