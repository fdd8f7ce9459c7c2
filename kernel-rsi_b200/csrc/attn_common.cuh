// attn_common.cuh - layout shared by the relpos-attention forward and backward kernels:
// how a head row of D elements (padded to DP, a multiple of 16) is split into TMA boxes /
// UMMA swizzle atoms, the qkv tensor map, and the host helpers that build it.
//
// A tile of R token rows x DP columns lives in shared memory as NCHUNK column blocks.  Block c
// covers columns [start_c, start_c + w_c) with w_c in {64, 32, 16} elements (128/64/32 bytes per
// row) and the matching 128B/64B/32B swizzle, stored row-major (R rows x w_c*2 bytes), so one
// block is one TMA box and a canonical UMMA layout for both K-major use (rows = M/N, columns =
// K) and MN-major use (rows = K, columns = M/N).  Columns D..DP-1 are outside the tensor map's
// extent and arrive as zeros (TMA out-of-bounds fill), which pads the contraction for D = 72.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "sm100.cuh"

namespace krsi {
namespace attn {

constexpr int kTileRows = 128;   // rows of every Q/K/V/dO tile (M of the UMMA)

template <int DP>
struct DLayout {
  static_assert(DP % 16 == 0 && DP >= 16 && DP <= 128, "DP must be a multiple of 16 in [16, 128]");
  static constexpr int kFull = DP / 64;              // 64-wide (128B swizzle) blocks
  static constexpr int kRem = DP % 64;               // 0, 16, 32 or 48
  static constexpr int kN32 = (kRem == 32 || kRem == 48) ? 1 : 0;
  static constexpr int kN16 = (kRem == 16 || kRem == 48) ? 1 : 0;
  static constexpr int NCHUNK = kFull + kN32 + kN16;
  __host__ __device__ static constexpr int width(int c) { return c < kFull ? 64 : (c == kFull && kN32) ? 32 : 16; }
  __host__ __device__ static constexpr int start(int c) { return c < kFull ? 64 * c : 64 * kFull + (c > kFull ? 32 : 0); }
  __host__ __device__ static constexpr uint32_t layout(int c) {
    return width(c) == 64 ? sm100::kSw128 : width(c) == 32 ? sm100::kSw64 : sm100::kSw32;
  }
  // byte offset of block c inside a tile of `rows` rows
  __host__ __device__ static constexpr uint32_t block_off(int c, int rows) {
    uint32_t o = 0;
    for (int i = 0; i < c; ++i) o += (uint32_t)rows * width(i) * 2;
    return o;
  }
  // chunk holding column `col` (a multiple of 16)
  __host__ __device__ static constexpr int chunk_of(int col) {
    for (int c = 0; c < NCHUNK; ++c)
      if (col < start(c) + width(c)) return c;
    return NCHUNK - 1;
  }
  static constexpr uint32_t tile_bytes(int rows) { return (uint32_t)rows * DP * 2; }
};

// K-major UMMA descriptor for the 16-column K slice starting at column `col` of a tile whose
// rows are M/N.  SBO = 8 rows of the block; LBO unused for swizzled K-major layouts.
template <int DP>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int rows, int col) {
  using L = DLayout<DP>;
  const int c = L::chunk_of(col);
  const uint32_t row_bytes = L::width(c) * 2;
  const uint32_t addr = tile_addr + L::block_off(c, rows) + (uint32_t)(col - L::start(c)) * 2;
  return sm100::smem_desc(addr, 16, 8 * row_bytes, L::layout(c));
}

// MN-major UMMA descriptor for block c of a tile whose rows are K, starting at K row `krow`
// (a multiple of 8).  SBO = 8 K-rows; LBO (stride between MN atoms) is unused because a block
// is exactly one swizzle atom wide.
template <int DP>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_addr, int rows, int c, int krow) {
  using L = DLayout<DP>;
  const uint32_t row_bytes = L::width(c) * 2;
  const uint32_t addr = tile_addr + L::block_off(c, rows) + (uint32_t)krow * row_bytes;
  return sm100::smem_desc(addr, (uint32_t)rows * row_bytes, 8 * row_bytes, L::layout(c));
}

// Loads a [kTileRows x DP] tile of section `sec` (0 = q, 1 = k, 2 = v; or the single section of
// a [B*S, H*D] tensor) for head h, token rows [row0, row0 + 128) of batch b, as NCHUNK boxes.
template <int DP>
__device__ __forceinline__ void load_tile(uint8_t* smem_tile, const CUtensorMap* m64, const CUtensorMap* m32,
                                          const CUtensorMap* m16, uint64_t* bar, int head_coord, int row0, int b) {
  using L = DLayout<DP>;
#pragma unroll
  for (int c = 0; c < L::NCHUNK; ++c) {
    const CUtensorMap* m = L::width(c) == 64 ? m64 : L::width(c) == 32 ? m32 : m16;
    sm100::tma_load_4d(smem_tile + L::block_off(c, kTileRows), m, bar, L::start(c), head_coord, row0, b);
  }
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D view (D, n_heads, S, B) of a token-major tensor with `row_stride` elements between
// tokens: element (d, hd, s, b) at base + ((b*S + s)*row_stride + hd*D + d).  Box = (box_w, 1,
// 128, 1) with the swizzle that matches box_w.  Columns >= D and rows >= S read as zero.
inline bool make_head_map(CUtensorMap* map, const void* base, int64_t row_stride, int64_t B, int64_t S,
                          int64_t n_heads, int64_t D, int box_w, bool f16) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n_heads, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)row_stride * 2, (cuuint64_t)(S * row_stride * 2)};
  cuuint32_t box[4] = {(cuuint32_t)box_w, 1, (cuuint32_t)kTileRows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMapSwizzle sw = box_w == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : box_w == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct HeadMaps {
  CUtensorMap m64, m32, m16;
};

// Builds the (up to three) box widths a DP needs; unused ones are left zeroed.
inline bool make_head_maps(HeadMaps* hm, int DP, const void* base, int64_t row_stride, int64_t B, int64_t S,
                           int64_t n_heads, int64_t D, bool f16) {
  memset(hm, 0, sizeof(*hm));
  const int rem = DP % 64;
  bool ok = true;
  if (DP >= 64) ok &= make_head_map(&hm->m64, base, row_stride, B, S, n_heads, D, 64, f16);
  if (rem == 32 || rem == 48) ok &= make_head_map(&hm->m32, base, row_stride, B, S, n_heads, D, 32, f16);
  if (rem == 16 || rem == 48) ok &= make_head_map(&hm->m16, base, row_stride, B, S, n_heads, D, 16, f16);
  return ok;
}

}  // namespace attn
}  // namespace krsi
