// attn_common.cuh - the shared-memory tile layout of the relpos-attention kernels, the qkv tensor
// maps that fill it, and descriptor helpers for the tcgen05 MMAs that read it.
//
// A tile of 128 token rows x DP columns (DP = D rounded up to 16) is stored as DP/16 column blocks.
// Block c holds columns [16c, 16c + 16) of every row, row-major with 32-byte rows (4 KB) and the
// 32-byte swizzle, and is filled by one TMA box.  This one layout serves every use:
//   * K-major operand (rows = M or N, columns = the contraction): the 16-column K slice kk of an
//     MMA is block kk, a canonical SW32 K-major matrix (SBO = 8 rows x 32 B).
//   * MN-major operand (rows = the contraction, columns = N): all DP/16 blocks together are DP/16
//     MN atoms of 16 columns, LBO = block stride, SBO = 8 rows x 32 B, so PV, dV, dK and dQ take a
//     single N = DP instruction per 16-row K step.
// Columns D..DP-1 and rows >= S lie outside the tensor map and arrive as zeros (TMA out-of-bounds
// fill): the contraction over D = 72 is padded to 80 without touching the neighbouring head.
// Measured on B200: SS M128 N128 K-major SW32 and TS M128 N80 MN-major SW32 both issue at full
// tensor rate from one thread when descriptors are precomputed (the issue loop stays tight).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <string.h>

#include "sm100.cuh"

namespace krsi {
namespace attn {

constexpr int kTileRows = 128;              // rows of every Q/K/V/dO tile (M of the UMMA)
constexpr uint32_t kBlockBytes = kTileRows * 32;   // one 16-column block of a tile

template <int DP>
struct Tile {
  static_assert(DP % 16 == 0 && DP >= 16 && DP <= 128, "DP must be a multiple of 16 in [16, 128]");
  static constexpr int kBlocks = DP / 16;
  static constexpr uint32_t kBytes = kBlocks * kBlockBytes;
};

// K-major descriptor of block 0 of a tile; K slice kk is this + kk * (kBlockBytes >> 4).
__device__ __forceinline__ uint64_t kmajor_base(uint32_t tile_addr) {
  return sm100::smem_desc(tile_addr, 16, 256, sm100::kSw32);
}
// MN-major descriptor (N = all columns) at K row 0; K rows [16k, 16k+16) are this + k * (512 >> 4).
__device__ __forceinline__ uint64_t mnmajor_base(uint32_t tile_addr) {
  return sm100::smem_desc(tile_addr, kBlockBytes, 256, sm100::kSw32);
}
constexpr uint64_t kKSliceStep = kBlockBytes >> 4;   // next 16 contraction columns (K-major)
constexpr uint64_t kKRowStep = (16 * 32) >> 4;       // next 16 contraction rows (MN-major)

// Loads a [128 x DP] tile of head coordinate `head_coord` (qkv: q = h, k = H + h, v = 2H + h; a
// [B*S, H*D] tensor: h), token rows [row0, row0 + 128) of batch b: DP/16 boxes of 16 columns.
template <int DP>
__device__ __forceinline__ void load_tile(uint8_t* smem_tile, const CUtensorMap* map, uint64_t* bar, int head_coord,
                                          int row0, int b) {
#pragma unroll
  for (int c = 0; c < Tile<DP>::kBlocks; ++c)
    sm100::tma_load_4d(smem_tile + c * kBlockBytes, map, bar, 16 * c, head_coord, row0, b);
}

// Fills dst[i] = src[i - pad] * mul for i in [0, n), zero where i - pad is outside [0, len).  Run by
// `nthr` cooperating threads (tid in [0, nthr)); the 16-byte-aligned interior of src is read with
// 128-bit loads, four in flight per thread, so a row of a few thousand floats takes one or two
// memory round trips.  dst may have any 4-byte alignment.  Source elements that would land at or
// past dst[n] are not read (len is clipped to n - pad).
__device__ __forceinline__ void fill_row(float* dst, int n, int pad, const float* __restrict__ src, int len, float mul,
                                         int tid, int nthr) {
  len = min(len, max(n - pad, 0));
  const int mis = (int)((reinterpret_cast<uintptr_t>(src) >> 2) & 3);
  const int a0 = mis ? min(4 - mis, len) : 0;         // first 16-byte aligned source index
  const int nvec = len > a0 ? (len - a0) / 4 : 0;
  const int a1 = a0 + 4 * nvec;                        // end of the vector interior
  const float4* src4 = reinterpret_cast<const float4*>(src + a0);
  for (int v0 = tid; v0 < nvec; v0 += 4 * nthr) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v0 + u * nthr < nvec) x[u] = __ldg(src4 + v0 + u * nthr);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v0 + u * nthr < nvec) {
        float* d = dst + pad + a0 + 4 * (v0 + u * nthr);
        d[0] = x[u].x * mul;
        d[1] = x[u].y * mul;
        d[2] = x[u].z * mul;
        d[3] = x[u].w * mul;
      }
  }
  // source edges and the zero pads
  for (int i = tid; i < n; i += nthr) {
    const int p = i - pad;
    if (p < 0 || p >= len) dst[i] = 0.f;
    else if (p < a0 || p >= a1) dst[i] = __ldg(src + p) * mul;
  }
}

// Fills dst[i] = src[top - i] * mul for i in [0, n), zero where top - i is outside [lo, hi] (a
// reversed window of src; lo >= 0 and hi must be valid source indices or lo > hi).  Same
// cooperative scheme as fill_row: the 16-byte-aligned interior of src[lo..hi] is read with 128-bit
// loads (four in flight per thread) and scattered in reverse order.
__device__ __forceinline__ void fill_row_rev(float* dst, int n, int top, const float* __restrict__ src, int lo, int hi,
                                             float mul, int tid, int nthr) {
  const int len = hi >= lo ? hi - lo + 1 : 0;
  const int mis = (int)((reinterpret_cast<uintptr_t>(src + lo) >> 2) & 3);
  const int a0 = lo + (mis ? min(4 - mis, len) : 0);   // first aligned source index
  const int nvec = lo + len > a0 ? (lo + len - a0) / 4 : 0;
  const int a1 = a0 + 4 * nvec;
  const float4* src4 = reinterpret_cast<const float4*>(src + a0);
  for (int v0 = tid; v0 < nvec; v0 += 4 * nthr) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v0 + u * nthr < nvec) x[u] = __ldg(src4 + v0 + u * nthr);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int m = a0 + 4 * (v0 + u * nthr);   // source index of x[u].x
      const int i = top - m;                      // its destination; m + 1.. go to i - 1..
      if (v0 + u * nthr < nvec) {
        if (i >= 0 && i < n) dst[i] = x[u].x * mul;
        if (i - 1 >= 0 && i - 1 < n) dst[i - 1] = x[u].y * mul;
        if (i - 2 >= 0 && i - 2 < n) dst[i - 2] = x[u].z * mul;
        if (i - 3 >= 0 && i - 3 < n) dst[i - 3] = x[u].w * mul;
      }
    }
  }
  for (int i = tid; i < n; i += nthr) {
    const int m = top - i;
    if (m < lo || m > hi) dst[i] = 0.f;
    else if (m < a0 || m >= a1) dst[i] = __ldg(src + m) * mul;
  }
}

// The two copies fill_row_rev(dst0, n, top, ...) and fill_row_rev(dst1, n, top - 1, ...) in one
// pass over the source (dst1[i] = dst0[i + 1]): one global round trip instead of two.
__device__ __forceinline__ void fill_row_rev2(float* dst0, float* dst1, int n, int top, const float* __restrict__ src,
                                              int lo, int hi, float mul, int tid, int nthr) {
  const int len = hi >= lo ? hi - lo + 1 : 0;
  const int mis = (int)((reinterpret_cast<uintptr_t>(src + lo) >> 2) & 3);
  const int a0 = lo + (mis ? min(4 - mis, len) : 0);   // first aligned source index
  const int nvec = lo + len > a0 ? (lo + len - a0) / 4 : 0;
  const int a1 = a0 + 4 * nvec;
  const float4* src4 = reinterpret_cast<const float4*>(src + a0);
  auto put = [&](int i, float v) {            // source element whose dst0 index is i
    if (i >= 0 && i < n) dst0[i] = v;
    if (i >= 1 && i - 1 < n) dst1[i - 1] = v;
  };
  for (int v0 = tid; v0 < nvec; v0 += 4 * nthr) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (v0 + u * nthr < nvec) x[u] = __ldg(src4 + v0 + u * nthr);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = top - (a0 + 4 * (v0 + u * nthr));
      if (v0 + u * nthr < nvec) {
        put(i, x[u].x * mul);
        put(i - 1, x[u].y * mul);
        put(i - 2, x[u].z * mul);
        put(i - 3, x[u].w * mul);
      }
    }
  }
  for (int i = tid; i < n; i += nthr) {
    const int m0 = top - i, m1 = top - 1 - i;
    if (m0 < lo || m0 > hi) dst0[i] = 0.f;
    else if (m0 < a0 || m0 >= a1) dst0[i] = __ldg(src + m0) * mul;
    if (m1 < lo || m1 > hi) dst1[i] = 0.f;
    else if (m1 < a0 || m1 >= a1) dst1[i] = __ldg(src + m1) * mul;
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

// 4-D view (D, n_heads, S, B) of a token-major tensor with `row_stride` elements between tokens:
// element (d, hd, s, b) at base + ((b*S + s)*row_stride + hd*D + d).  Box = (16, 1, 128, 1) with
// the 32-byte swizzle.  Columns >= D and rows >= S read as zero.
inline bool make_head_map(CUtensorMap* map, const void* base, int64_t row_stride, int64_t B, int64_t S,
                          int64_t n_heads, int64_t D, bool f16) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  memset(map, 0, sizeof(*map));
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n_heads, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)row_stride * 2, (cuuint64_t)(S * row_stride * 2)};
  cuuint32_t box[4] = {16, 1, (cuuint32_t)kTileRows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D view (D, n_heads, S, B) of a token-major 16-bit tensor like make_head_map, with box
// (D, 1, 128, 1) and no swizzle: a dense [128 rows x D] tile, for TMA stores of whole head rows.
// Rows >= S are outside the tensor and are not written.
inline bool make_head_rows_map(CUtensorMap* map, const void* base, int64_t row_stride, int64_t B, int64_t S,
                               int64_t n_heads, int64_t D, bool f16) {
  EncodeTiledFn enc = encode_fn();
  if (!enc || D > 256) return false;
  memset(map, 0, sizeof(*map));
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n_heads, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)row_stride * 2, (cuuint64_t)(S * row_stride * 2)};
  cuuint32_t box[4] = {(cuuint32_t)D, 1, (cuuint32_t)kTileRows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D fp32 view (D, S, B) of head `h` columns of a [B*S, n_heads*D] fp32 tensor, for the TMA
// reduce-add of a [128 rows x box_cols] tile: element (d, s, b) at base + ((b*S + s)*n_heads*D + d),
// the caller adds h*D (+ the part's first column) to the x coordinate.  Box = (box_cols, 128, 1), no
// swizzle (row-major tile with a box_cols*4-byte pitch; box_cols * 4 a multiple of 16).  Rows >= S
// are clipped, so a ragged last block writes nothing outside its batch.
inline bool make_rows_f32_map(CUtensorMap* map, float* base, int64_t B, int64_t S, int64_t n_heads, int64_t D,
                              int64_t box_cols) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  memset(map, 0, sizeof(*map));
  cuuint64_t dims[3] = {(cuuint64_t)(n_heads * D), (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(n_heads * D * 4), (cuuint64_t)(S * n_heads * D * 4)};
  if (box_cols <= 0 || box_cols > 256 || (box_cols * 4) % 16) return false;
  cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)kTileRows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace attn
}  // namespace krsi
