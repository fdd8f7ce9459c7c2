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
//               F-columns, warps 8-11 the last 64): accumulator -> u (bf16/f16, the GEMM output's
//               rounding) -> GEGLU on the rounded values -> u and out stored straight from registers.
// The two accumulators alternate, so tile i's epilogue runs while tile i+1's MMAs do.
// Every wait is bounded (watchdog.cuh); a stalled pipeline ends the CTA with an error word.
#include <string.h>

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
constexpr uint32_t kBarOff = kStages * kStageBytes;
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

// K-major operand in the 128-byte swizzle: 8-row groups of 8 x 128 B (SBO = 1024 B); the K step of
// 16 elements inside the swizzle row advances the start address by 32 B.
__device__ __forceinline__ uint64_t kmajor_sw128(uint32_t addr) { return smem_desc(addr, 16, 1024, kSw128); }

template <bool F16>
__global__ void __launch_bounds__(kThreads, 1)
linear_geglu_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                    const GemmArgs a) {
  pdl_enter();   // before any global access and before claiming TMEM
  constexpr int DT = F16 ? KRSI_F16 : KRSI_BF16;
  using E = Elem<DT>;
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
    if (!ok) watchdog_fire(kWdGemmLoad);
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
    using T = typename E::T;
    const int ew = warp - kEpiWarp0;
    const int quarter = ew % 4;                 // TMEM lane quarter of this warp (warp % 4)
    const int half = ew / 4;                    // which 64 of the tile's 128 F-columns
    const int r = quarter * 32 + lane;          // row within the tile
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int64_t two_f = 2 * (int64_t)a.F;
    bool ok = true;
    for (int i = 0; i < my_tiles; ++i) {
      const int t = tile_of(i);
      const int acc = i & 1;
      const int row = (t / a.n_ftiles) * kBM + r;
      const int c_base = (t % a.n_ftiles) * kBF + half * 64;   // first F-column of this thread's 64
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[acc], (i >> 1) & 1, abort_flag, a.spin_limit))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t acc_addr = tmem + lane_addr + acc * kBN + half * 64;
      T* urow = reinterpret_cast<T*>(a.u) + (int64_t)row * two_f;
      T* orow = reinterpret_cast<T*>(a.out) + (int64_t)row * a.F;
      const bool row_ok = row < a.rows;
#pragma unroll 1
      for (int c0 = 0; c0 < 64; c0 += 32) {
        uint32_t gv[32], vv[32];
        tmem_ld32(acc_addr + c0, gv);              // gate columns
        tmem_ld32(acc_addr + kBF + c0, vv);        // value columns
        tmem_wait_ld();
        if (c0 + 32 == 64) {                       // the accumulator has been read: the MMA may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
#pragma unroll
        for (int p = 0; p < 32; p += 8) {
          const int col = c_base + c0 + p;
          if (!row_ok || col >= a.F) continue;     // F is a multiple of 8: whole packets are in or out
          Vec16<T> ug, uv, o;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const T ga = E::store(__uint_as_float(gv[p + e]));   // u, rounded as the GEMM output
            const T vb = E::store(__uint_as_float(vv[p + e]));
            ug.v[e] = ga;
            uv.v[e] = vb;
            o.v[e] = E::store(gelu::geglu_out<DT>(E::load(ga), E::load(vb)));
          }
          stg16(urow + col, ug);
          stg16(urow + a.F + col, uv);
          stg16(orow + col, o);
        }
      }
    }
    if (!ok) watchdog_fire(kWdGemmEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// 2-D view (K, rows) of a row-major [rows, K] 16-bit matrix, box (64, 128), 128-byte swizzle.
// Elements past K or rows read as zero.
bool make_kmajor_map(CUtensorMap* map, const void* base, int64_t rows, int64_t K, bool f16) {
  attn::EncodeTiledFn enc = attn::encode_fn();
  if (!enc) return false;
  memset(map, 0, sizeof(*map));
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool F16>
int launch(const CUtensorMap& xm, const CUtensorMap& wm, const GemmArgs& a, cudaStream_t stream) {
  auto kern = linear_geglu_kernel<F16>;
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  const int grid = a.n_tiles < device_sm_count() ? a.n_tiles : device_sm_count();
  KRSI_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(kThreads), kSmem, stream, xm, wm, a));
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
  CUtensorMap xm, wm;
  if (!make_kmajor_map(&xm, x, rows, K, f16) || !make_kmajor_map(&wm, w, 2 * F, K, f16)) return KRSI_ERR_CUDA;
  const int64_t n_rt = (rows + kBM - 1) / kBM, n_ft = (F + kBF - 1) / kBF;
  if (n_rt * n_ft > INT32_MAX) return KRSI_ERR_UNSUPPORTED;
  GemmArgs a{u, out, (int)rows, (int)K, (int)F, (int)n_ft, (int)(n_rt * n_ft), (int)((K + kBK - 1) / kBK),
             kSpinLimit};
  return f16 ? launch<true>(xm, wm, a, stream) : launch<false>(xm, wm, a, stream);
}
