// relpos_attn_fwd.cu - relative-position-bias flash attention forward for B200 (sm_100a).
//
// Computes what library/relpos_attention.py:26-59 (_fwd) computes, for every (b, h):
//   s2[i, j] = (q_i . k_j * scale + pd[h, j - i + S - 1]) * log2(e)
//   m_i = max_j s2, l_i = sum_j exp2(s2 - m_i), out_i = sum_j exp2(s2 - m_i) v_j / l_i,
//   lse_i = m_i + log2(l_i); out in the input dtype, out32 in fp32.
//
// Structure (one CTA = two 128-query tiles of one (b, h), 12 warps = 3 warpgroups; setmaxnreg
// moves registers from warpgroup 0 to the softmax warpgroups):
//   warp 0      TMA producer (tile layout: attn_common.cuh): Q once, then per 128-key block a K
//               tile and a V tile (3-stage ring);
//   warps 2-3   the bias row pd[h, :] * log2(e), resident in shared memory for the CTA's life
//               (two copies, one shifted by an element, for aligned pair reads), fetched with
//               128-bit loads; sequences too long for it fall back to a per-block slab the
//               producer writes;
//   warp 1      TMEM owner (512 columns) and the single-thread tcgen05.mma issuer:
//               S_t = Q_t K^T (SS, K = DP) into TMEM, O_t += P_t V (TS: P read from TMEM, one
//               N = DP instruction per 16 keys);
//   warps 4-7   softmax for query tile 0, warps 8-11 for tile 1 (one query row per thread,
//               row = TMEM lane): S from TMEM -> bias add (paired fp32 FMAs) -> online softmax
//               with the rescale of O skipped unless the running max grows by more than 2^8;
//               exp2 on the SFU for 3/4 of the elements and on the FMA pipe (sm100.cuh) for
//               1/4 -> P (bf16/f16) written back over S in TMEM -> at the end O / l to memory.
// The two query tiles ping-pong so one tile's softmax overlaps the other tile's MMAs.
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
constexpr int kQTiles = 2;          // query tiles per CTA
constexpr int kThreads = 384;       // 3 warpgroups: {producer, MMA, -, -}, softmax tile 0, tile 1
constexpr uint32_t kRegsCtl = 96;   // per-thread registers of warpgroup 0 after setmaxnreg
constexpr uint32_t kRegsSm = 200;   // softmax warpgroups (launch 168 x 384 >= 128 x (96 + 2 x 200))
constexpr int kSlab = 384;          // floats per bias slab (2*128 + 128 - 1 = 383 used)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units: P <= 2^8 between rescales
constexpr int kRowFillers = 320;           // warps 2-11 fill the resident bias window

template <int DP>
struct FwdCfg {
  static constexpr int NS = DP <= 96 ? 3 : 2;                      // K/V pipeline stages
  static constexpr uint32_t kTile = attn::Tile<DP>::kBytes;         // one 128 x DP tile
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKVOff = kQOff + kQTiles * kTile;
  static constexpr uint32_t kSlabOff = kKVOff + NS * 2 * kTile;
  static constexpr uint32_t kBarOff = kSlabOff + NS * kSlab * 4;
  static constexpr int kNumBars = 1 + 2 * NS + 3 * kQTiles + 2;     // q_full, kv_full/empty, s/p/o, drain, row
  static constexpr uint32_t kMiscOff = kBarOff + kNumBars * 8;
  static constexpr uint32_t kRowOff = kMiscOff + 16;                // resident bias row (runtime length)
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
  uint32_t spin_limit;
};

// Resident bias row: pd[h, :] * log2(e) with kRowPad zeros before it and 128 after, so every
// index a CTA forms (key - query + S - 1 for keys and queries up to 127 past S) stays inside.
// Two copies, the second shifted by one element, so that every thread reads its 128 bias values
// as 8-byte aligned pairs (copy 0 when its start index is even, copy 1 when odd).  Lane l of a warp
// starts at B0 - l with B0 of the parity of S - 1; in a half-warp the copy-0 lanes then read 16
// consecutive floats and the copy-1 lanes 16 more, shifted by the copy distance - 16 (S even) or
// - 18 (S odd).  Spacing the copies 16 or 18 (mod 32) floats apart puts the two halves on disjoint
// banks: one wavefront per half-warp.
constexpr int kRowPad = 256;
__host__ __device__ constexpr int64_t row_floats(int64_t S) {
  return (2 * S - 1 + kRowPad + 128 + 31 - ((S & 1) ? 18 : 16)) / 32 * 32 + ((S & 1) ? 18 : 16);
}
__host__ __device__ constexpr int64_t row_bytes(int64_t S) { return 2 * row_floats(S) * 4; }



// dst[i] = src[i - pad] * log2(e) for i in [w0, w1), zero where i - pad is outside [0, len), by
// kRowFillers cooperating threads.
__device__ __forceinline__ void fill_row_window(float* dst, int w0, int w1, int pad, const float* __restrict__ src,
                                                int len, int tid) {
  const int s0 = max(w0 - pad, 0), s1 = min(w1 - pad, len);
  attn::fill_row(dst + w0, w1 - w0, s0 + pad - w0, src + s0, max(s1 - s0, 0), kLog2e, tid, kRowFillers);
}

template <int DP, bool F16, bool RES>
__global__ void __launch_bounds__(kThreads, 1)
relpos_fwd_kernel(const __grid_constant__ CUtensorMap tmap, const FwdArgs a) {
  using C = FwdCfg<DP>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 1 + NS;
  uint64_t* s_ready = bars + 1 + 2 * NS;
  uint64_t* p_ready = s_ready + kQTiles;
  uint64_t* o_final = p_ready + kQTiles;
  uint64_t* drain = o_final + kQTiles;
  uint64_t* row_full = drain + 1;
  float* row0 = reinterpret_cast<float*>(smem + C::kRowOff);
  float* row1 = row0 + row_floats(a.S);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  float* slabs = reinterpret_cast<float*>(smem + C::kSlabOff);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * (kQTiles * kTileRows);
  const int n_kb = a.n_kb;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], RES ? 1 : 2);   // TMA expect_tx arrival (+ bias-slab arrival)
      mbar_init(&kv_empty[s], 1);    // tcgen05.commit
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(&s_ready[t], 1);
      mbar_init(&p_ready[t], 128);
      mbar_init(&o_final[t], 1);
    }
    mbar_init(drain, 1);
    mbar_init(row_full, kRowFillers);
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
  // Resident bias window (RES), filled by warps 2-11 (the softmax warps are idle until their first
  // S tile): only the indices this CTA forms, kRowPad + key - query + S - 1 for its 256 queries and
  // all keys, plus one on each side for the shifted copy.
  auto fill_window = [&]() {
    const int two_s = 2 * a.S - 1;
    const float* pdh = a.pd + (size_t)h * two_s;
    const int n = (int)row_floats(a.S);
    const int tid = threadIdx.x - 64;
    const int w0 = max(kRowPad + a.S - 1 - (q0 + kQTiles * kTileRows - 1) - 1, 0);
    const int w1 = min(kRowPad + a.S - 1 - q0 + n_kb * kBN + 1, n);
    fill_row_window(row0, w0, w1, kRowPad, pdh, two_s, tid);
    fill_row_window(row1, w0, w1, kRowPad - 1, pdh, two_s, tid);   // row1[i] = row0[i + 1]
    mbar_arrive(row_full);
  };
  // Each role runs entirely inside the branch that sets its register budget, so ptxas compiles
  // it against that budget.
  if (warp < 4) {
    regs_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQTiles * C::kTile);
      for (int t = 0; t < kQTiles; ++t)
        attn::load_tile<DP>(smem + C::kQOff + t * C::kTile, &tmap, q_full, h, q0 + t * kTileRows, b);
    }
    const int two_s = 2 * a.S - 1;
    const float* pdh = a.pd + (size_t)h * two_s;

    for (int j = 0; j < n_kb; ++j) {
      const int s = j % NS;
      if (j >= NS && !mbar_wait_bounded(&kv_empty[s], ((j / NS) + 1) & 1, abort_flag, a.spin_limit)) {
        watchdog_fire(kWdFwdLoad);
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
      const int base = j * kBN - q0 - (kQTiles * kTileRows - 1) + a.S - 1;
      for (int idx = lane; idx < kSlab; idx += 32) {
        const int pos = base + idx;
        slab[idx] = (pos >= 0 && pos < two_s) ? __ldg(pdh + pos) * kLog2e : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_full[s]);
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ resident bias window (RES)
    if constexpr (RES) fill_window();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = F16 ? 0u : 1u;
      constexpr uint32_t id_qk = idesc_f16(128, kBN, fmt, false, false);   // S = Q K^T: both K-major
      constexpr uint32_t id_pv = idesc_f16(128, DP, fmt, false, true);     // O += P V: V MN-major, N = DP
      // Descriptors are precomputed; an issue is a constant add and the MMA itself, which keeps
      // one thread issuing at the tensor pipe's rate.
      const uint64_t q_desc = attn::kmajor_base(smem_u32(smem + C::kQOff));
      const uint64_t k_desc0 = attn::kmajor_base(smem_u32(smem + C::kKVOff));
      const uint64_t v_desc0 = attn::mnmajor_base(smem_u32(smem + C::kKVOff + C::kTile));
      constexpr uint64_t kStageStep = (2 * C::kTile) >> 4;
      constexpr uint64_t kQTileStep = C::kTile >> 4;
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, a.spin_limit) &&
                mbar_wait_bounded(&kv_full[0], 0, abort_flag, a.spin_limit);
      auto issue_qk = [&](int t, int j) {
        const uint64_t qd = q_desc + (uint64_t)t * kQTileStep;
        const uint64_t kd = k_desc0 + (uint64_t)(j % NS) * kStageStep;
        const uint32_t d = tmem + C::kSCol + t * kBN;
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          mma_ss(d, qd + kk * attn::kKSliceStep, kd + kk * attn::kKSliceStep, id_qk, kk > 0 ? 1u : 0u);
      };
      auto issue_pv = [&](int t, int j) {
        const uint64_t vd = v_desc0 + (uint64_t)(j % NS) * kStageStep;
        const uint32_t p_tmem = tmem + C::kSCol + t * kBN;   // P: 2 x 16-bit per column
        const uint32_t d = tmem + C::kOCol + t * DP;
        const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_ts(d, p_tmem + kk * 8, vd + kk * attn::kKRowStep, id_pv, kk > 0 ? 1u : acc0);
      };
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < kQTiles; ++t) {
          issue_qk(t, 0);
          mma_commit(&s_ready[t]);
        }
        for (int j = 0; j < n_kb && ok; ++j) {
          const bool has_next = j + 1 < n_kb;
          if (has_next && !mbar_wait_bounded(&kv_full[(j + 1) % NS], ((j + 1) / NS) & 1, abort_flag, a.spin_limit)) {
            ok = false;
            break;
          }
          for (int t = 0; t < kQTiles; ++t) {
            if (!mbar_wait_bounded(&p_ready[t], j & 1, abort_flag, a.spin_limit)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, j);
            if (has_next) {
              issue_qk(t, j + 1);
              mma_commit(&s_ready[t]);
            } else {
              mma_commit(&o_final[t]);
            }
          }
          if (!ok) break;
          mma_commit(&kv_empty[j % NS]);
        }
      }
      if (!ok) watchdog_fire(kWdFwdMma);
      // Drain: every MMA issued above has completed before TMEM is released.
      mma_commit(drain);
      for (uint32_t i = 0; i < a.spin_limit && !mbar_try_wait(drain, 0); ++i) {
      }
    }
  }
  } else {
    regs_inc<kRegsSm>();
    if constexpr (RES) fill_window();
    // ------------------------------------------------------------ softmax (warps 4..11)
    const int t = (warp - 4) / 4;                       // query tile
    const int quarter = warp % 4;                       // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;                  // row within the tile
    const int q = q0 + t * kTileRows + r;               // query index within the sequence
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_tmem = tmem + lane_addr + C::kSCol + t * kBN;
    const uint32_t o_tmem = tmem + lane_addr + C::kOCol + t * DP;
    const int slab_base = (kQTiles - 1 - t) * kTileRows + (kTileRows - 1) - r;   // slab[slab_base + c]
    // resident row: bias(q, key j*128 + c) = row0[bidx + c], bidx = kRowPad + j*128 - q + S - 1
    const int bidx0 = kRowPad - q + a.S - 1;
    const float* bias_q = (bidx0 & 1) ? row1 + bidx0 - 1 : row0 + bidx0;   // 8-byte aligned pairs
    const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = !RES || __all_sync(0xffffffffu, mbar_wait_bounded(row_full, 0, abort_flag, a.spin_limit));
    for (int j = 0; j < n_kb && ok; ++j) {
      const int s = j % NS;
      const bool w_ok = mbar_wait_bounded(&s_ready[t], j & 1, abort_flag, a.spin_limit) &&
                        (RES || mbar_wait_bounded(&kv_full[s], (j / NS) & 1, abort_flag, a.spin_limit));
      if (!__all_sync(0xffffffffu, w_ok)) {   // warp-uniform: TMEM loads/stores are warp-collective
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t u[kBN];
#pragma unroll
      for (int c = 0; c < kBN; c += 32) tmem_ld32(s_tmem + c, u + c);
      tmem_wait_ld();
      // v = s * scale * log2(e) + bias * log2(e), two columns per instruction
      uint64_t v2[kBN / 2];
      if constexpr (RES) {
        const uint64_t* bp = reinterpret_cast<const uint64_t*>(bias_q + j * kBN);
#pragma unroll
        for (int i = 0; i < kBN / 2; ++i)
          v2[i] = f2_fma(f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), scale2, bp[i]);
      } else {
        const float* slab = slabs + s * kSlab + slab_base;
#pragma unroll
        for (int i = 0; i < kBN / 2; ++i)
          v2[i] = f2_fma(f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), scale2,
                         f2_pack(slab[2 * i], slab[2 * i + 1]));
      }
      const int valid = a.S - j * kBN;                  // keys of this block inside the sequence
      if (valid < kBN) {                                // only the last block of a ragged sequence
#pragma unroll
        for (int i = 0; i < kBN / 2; ++i) {
          float lo, hi;
          f2_unpack(v2[i], lo, hi);
          v2[i] = f2_pack(2 * i < valid ? lo : -INFINITY, 2 * i + 1 < valid ? hi : -INFINITY);
        }
      }
      // row max: 3-input max, 4 independent chains
      float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < kBN / 2; ++i) {
        float lo, hi;
        f2_unpack(v2[i], lo, hi);
        mxa[i % 4] = max3(mxa[i % 4], lo, hi);
      }
      const float mx = fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3]));
      const float m_new = fmaxf(m_run, mx);
      const bool need = m_new - m_run > kRescaleThreshold;   // true on the first block (m_run = -inf)
      float alpha = 1.f, m_use = m_run;
      const bool warp_rescale = __any_sync(0xffffffffu, need);
      if (warp_rescale) {
        m_use = m_new;
        alpha = ex2_approx(m_run - m_new);              // 0 on the first block
      }
      // p = 2^(v - m): three of every four pairs on the SFU, one on the FMA pipe (balances the
      // SFU against the issue slots); row sum in 4 paired chains; P packed to 16-bit pairs
      const uint64_t negm2 = f2_pack(-m_use, -m_use);
      uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int i = 0; i < kBN / 2; ++i) {
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
      tmem_st32(s_tmem, pk);
      tmem_st32(s_tmem + 32, pk + 32);
      if (warp_rescale && j > 0) {
        // O_t holds the sum through block j-1 (PV(t, j-1) completed before S_t(j) was ready).
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
      mbar_arrive(&p_ready[t]);
    }
    if (ok && !__all_sync(0xffffffffu, mbar_wait_bounded(&o_final[t], 0, abort_flag, a.spin_limit))) ok = false;
    if (!ok) {
      watchdog_fire(kWdFwdSoftmax);
    } else {
      tc_fence_after();
      // All lanes run the warp-collective TMEM loads; rows past the sequence end skip the stores.
      const bool row_ok = q < a.S;
      const float inv_l = 1.0f / l_run;
      const size_t row = (size_t)b * a.S + (row_ok ? q : 0);
      const size_t ld = (size_t)a.H * a.D;
      float* o32 = a.out32 + row * ld + (size_t)h * a.D;
      using T = typename std::conditional<F16, __half, __nv_bfloat16>::type;
      T* o16 = reinterpret_cast<T*>(a.out) + row * ld + (size_t)h * a.D;
#pragma unroll
      for (int c = 0; c < DP; c += 16) {
        uint32_t ov[16];
        tmem_ld16(o_tmem + c, ov);
        tmem_wait_ld();
        float f[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(ov[e]) * inv_l;
#pragma unroll
        for (int e = 0; e < 16; e += 8) {
          if (row_ok && c + e < a.D) {   // D is a multiple of 8: whole 8-column groups are in or out
            float4* d32 = reinterpret_cast<float4*>(o32 + c + e);
            d32[0] = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
            d32[1] = make_float4(f[e + 4], f[e + 5], f[e + 6], f[e + 7]);
            uint4 pk;
            if (F16) {
              pk = make_uint4(pack_f16x2(f[e], f[e + 1]), pack_f16x2(f[e + 2], f[e + 3]),
                              pack_f16x2(f[e + 4], f[e + 5]), pack_f16x2(f[e + 6], f[e + 7]));
            } else {
              pk = make_uint4(pack_bf16x2(f[e], f[e + 1]), pack_bf16x2(f[e + 2], f[e + 3]),
                              pack_bf16x2(f[e + 4], f[e + 5]), pack_bf16x2(f[e + 6], f[e + 7]));
            }
            *reinterpret_cast<uint4*>(o16 + c + e) = pk;
          }
        }
      }
      if (row_ok) a.lse[(size_t)bh * a.S + q] = m_run + __log2f(l_run);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

constexpr size_t kMaxSmem = 232448;   // 227 KB per CTA on sm_100

template <int DP, bool F16>
int launch_fwd(const CUtensorMap& tmap, const FwdArgs& a, cudaStream_t stream) {
  using C = FwdCfg<DP>;
  const size_t res_smem = C::kSmem + (size_t)row_bytes(a.S);
  const bool res = res_smem <= kMaxSmem;
  auto kern = res ? relpos_fwd_kernel<DP, F16, true> : relpos_fwd_kernel<DP, F16, false>;
  const size_t smem = res ? res_smem : C::kSmem;
  KRSI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((a.S + kQTiles * kTileRows - 1) / (kQTiles * kTileRows), a.B * a.H);
  kern<<<grid, kThreads, smem, stream>>>(tmap, a);
  KRSI_LAUNCH_CHECK();
  return KRSI_OK;
}

template <bool F16>
int dispatch_dp(int DP, const CUtensorMap& tmap, const FwdArgs& a, cudaStream_t s) {
  switch (DP) {
    case 32: return launch_fwd<32, F16>(tmap, a, s);
    case 64: return launch_fwd<64, F16>(tmap, a, s);
    case 80: return launch_fwd<80, F16>(tmap, a, s);
    case 96: return launch_fwd<96, F16>(tmap, a, s);
    case 128: return launch_fwd<128, F16>(tmap, a, s);
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
  FwdArgs a{pd, out, out32, lse, (int)B, (int)S, (int)H, (int)D, scale * 1.4426950408889634f,
            (int)((S + kBN - 1) / kBN), kSpinLimit};
  return dtype == KRSI_F16 ? dispatch_dp<true>(DP, tmap, a, stream) : dispatch_dp<false>(DP, tmap, a, stream);
}
