// t5_bias.cu - T5 bucketed relative position, on either side of the relpos attention op.
//
// T5 (HF T5Attention._relative_position_bucket / compute_bias, transformers
// models/t5/modeling_t5.py) maps the distance rel = key - query to one of `num_buckets` buckets and
// looks the bias up in a learned table [num_buckets, H]:
//   bidirectional: half the buckets per sign (rel > 0 adds num_buckets / 2), a = |rel|;
//   otherwise:     a = max(-rel, 0);
//   with n = the buckets per side and e = n / 2: bucket offset a for a < e, else
//   e + trunc(log(a / e) / log(max_distance / e) * (n - e)), capped at n - 1.
// The attention op takes that bias as a per-distance row pd[h, rel + S - 1] (relpos_attention.py:5,
// bias[h, i, j] = pd[h, j - i + S - 1]), so:
//   forward:  pd[h, t] = table[bucket(t - (S - 1)), h]                      (an expansion, [H, 2S-1])
//   backward: dtable[k, h] = sum of dpd[h, t] over the t with bucket(t - (S - 1)) = k
// Every bucket is a contiguous run of distances, so the backward is a segmented sum: one warp per
// (bucket, head) adds its run in a fixed order (deterministic, no atomics, no S x S scatter).
//
// The bucket of a large distance depends on a float log, which can tip at the exact bucket edges
// (a / e a power of max_distance / e).  The host therefore derives, once per call, the smallest
// distance of every large-distance bucket offset in double precision (edges land on their exact
// value, as torch's fp32 evaluation does there), and the kernels only compare integers.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace krsi {
namespace {

constexpr int kMaxBuckets = 256;

struct BucketMap {
  int n_side;             // buckets per side (num_buckets / 2 if bidirectional)
  int exact;              // n_side / 2: distances below it are their own bucket
  int bidir;
  int n_thr;              // large-distance thresholds: offset k >= 1 starts at thr[k - 1]
  int thr[kMaxBuckets];
};

__host__ __device__ inline int bucket_of(const BucketMap& m, int64_t rel) {
  int base = 0;
  int64_t a;
  if (m.bidir) {
    base = rel > 0 ? m.n_side : 0;
    a = rel < 0 ? -rel : rel;
  } else {
    a = rel < 0 ? -rel : 0;
  }
  if (a < m.exact) return base + (int)a;
  int k = 0;
  while (k < m.n_thr && a >= m.thr[k]) ++k;
  return base + m.exact + k;
}

// Smallest distance of each large-distance offset k = 1 .. n_side - exact - 1.
inline bool make_map(int num_buckets, int max_distance, int bidir, BucketMap* m) {
  const int n_side = bidir ? num_buckets / 2 : num_buckets;
  const int exact = n_side / 2;
  if (num_buckets < 2 || num_buckets > kMaxBuckets || exact < 1 || max_distance <= exact) return false;
  m->n_side = n_side;
  m->exact = exact;
  m->bidir = bidir;
  m->n_thr = n_side - exact - 1;
  const double scale = (double)(n_side - exact) / std::log((double)max_distance / exact);
  for (int k = 1; k <= m->n_thr; ++k) {
    // offset(a) = floor(log(a / exact) * scale) >= k  <=>  a >= exact * exp(k / scale)
    const double edge = exact * std::exp(k / scale);
    int64_t a = (int64_t)std::ceil(edge - 1e-9 * edge);
    if (a < exact) a = exact;
    m->thr[k - 1] = a > (int64_t)0x7fffffff ? 0x7fffffff : (int)a;
  }
  return true;
}

template <int DT>
__global__ void __launch_bounds__(256)
t5_bias_fwd_kernel(const typename Elem<DT>::T* __restrict__ table, float* __restrict__ pd, int64_t S, int H,
                   const __grid_constant__ BucketMap m) {
  pdl_enter();
  const int64_t n = 2 * S - 1;
  const int h = blockIdx.y;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int k = bucket_of(m, t - (S - 1));
    pd[(int64_t)h * n + t] = Elem<DT>::load(table[(int64_t)k * H + h]);
  }
}

// Distances a (>= 0) of bucket offset k on one side: [lo, hi), hi = INT64_MAX for the last offset.
__device__ __forceinline__ void offset_range(const BucketMap& m, int k, int64_t* lo, int64_t* hi) {
  const int64_t kInf = 0x7fffffffffffffffLL;
  if (k < m.exact) {
    *lo = k;
    *hi = k + 1;
  } else {
    const int j = k - m.exact;                  // 0 .. n_thr
    *lo = j == 0 ? m.exact : m.thr[j - 1];
    *hi = j < m.n_thr ? m.thr[j] : kInf;
  }
}

// One warp per (bucket, head).  A bucket is one run of distances on each side of rel = 0, found in
// closed form from the thresholds; the lanes add the run's dpd in strides of 32, in order, then a
// fixed butterfly adds the lanes (deterministic).
template <int DT>
__global__ void __launch_bounds__(256)
t5_bias_bwd_kernel(const float* __restrict__ dpd, typename Elem<DT>::T* __restrict__ dtable, int64_t S, int H,
                   int num_buckets, const __grid_constant__ BucketMap m) {
  pdl_enter();
  const int warp = (int)(blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32), lane = threadIdx.x % 32;
  if (warp >= num_buckets * H) return;
  const int k = warp / H, h = warp % H;
  const int64_t n = 2 * S - 1;
  const float* row = dpd + (int64_t)h * n;
  float s = 0.f;
  auto add_run = [&](int64_t t0, int64_t t1) {   // t in [t0, t1)
    for (int64_t t = t0 + lane; t < t1; t += 32) s += row[t];
  };
  int64_t lo, hi;
  if (m.bidir) {
    if (k < m.n_side) {                         // rel = -a <= 0: t = S - 1 - a
      offset_range(m, k, &lo, &hi);
      if (lo <= S - 1) add_run(S - 1 - min(hi - 1, S - 1), S - lo);
    } else {                                    // rel = a > 0: t = S - 1 + a
      offset_range(m, k - m.n_side, &lo, &hi);
      lo = max(lo, (int64_t)1);
      if (lo <= S - 1) add_run(S - 1 + lo, S - 1 + min(hi - 1, S - 1) + 1);
    }
  } else {
    offset_range(m, k, &lo, &hi);               // rel = -a <= 0
    if (lo <= S - 1) add_run(S - 1 - min(hi - 1, S - 1), S - lo);
    if (k == 0) add_run(S, n);                  // every rel > 0 is bucket 0
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) dtable[(int64_t)k * H + h] = Elem<DT>::store(s);
}

}  // namespace

int t5_bucket_of(int num_buckets, int max_distance, int bidirectional, int64_t rel, int* bucket) {
  BucketMap m;
  if (!make_map(num_buckets, max_distance, bidirectional, &m)) return KRSI_ERR_INVALID_ARGUMENT;
  *bucket = bucket_of(m, rel);
  return KRSI_OK;
}

}  // namespace krsi

using namespace krsi;

extern "C" int krsi_t5_bucket(int num_buckets, int max_distance, int bidirectional, int64_t rel, int* bucket) {
  KRSI_CHECK_ARG(bucket);
  return t5_bucket_of(num_buckets, max_distance, bidirectional, rel, bucket);
}

extern "C" int krsi_t5_bias_fwd(const void* table, float* pd, int64_t S, int64_t H, int num_buckets, int max_distance,
                                int bidirectional, int table_dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(S >= 0 && H > 0 && H <= 65535);
  if (table_dtype != KRSI_F32 && table_dtype != KRSI_BF16 && table_dtype != KRSI_F16) return KRSI_ERR_INVALID_ARGUMENT;
  BucketMap m;
  if (!make_map(num_buckets, max_distance, bidirectional, &m)) return KRSI_ERR_INVALID_ARGUMENT;
  if (S == 0) return KRSI_OK;
  KRSI_CHECK_ARG(table && pd);
  if (S > (1 << 30)) return KRSI_ERR_UNSUPPORTED;
  const int64_t n = 2 * S - 1;
  const dim3 grid((unsigned)std::min<int64_t>((n + 255) / 256, 1024), (unsigned)H);
#define KRSI_T5F(DT)                                                                                        \
  KRSI_CUDA_TRY(launch_pdl(t5_bias_fwd_kernel<DT>, grid, dim3(256), 0, stream,                              \
                           (const typename Elem<DT>::T*)table, pd, S, (int)H, m))
  if (table_dtype == KRSI_F32) KRSI_T5F(KRSI_F32);
  else if (table_dtype == KRSI_BF16) KRSI_T5F(KRSI_BF16);
  else KRSI_T5F(KRSI_F16);
#undef KRSI_T5F
  return KRSI_OK;
}

extern "C" int krsi_t5_bias_bwd(const float* dpd, void* dtable, int64_t S, int64_t H, int num_buckets,
                                int max_distance, int bidirectional, int table_dtype, cudaStream_t stream) {
  KRSI_CHECK_ARG(S >= 0 && H > 0 && H <= 65535);
  if (table_dtype != KRSI_F32 && table_dtype != KRSI_BF16 && table_dtype != KRSI_F16) return KRSI_ERR_INVALID_ARGUMENT;
  BucketMap m;
  if (!make_map(num_buckets, max_distance, bidirectional, &m)) return KRSI_ERR_INVALID_ARGUMENT;
  KRSI_CHECK_ARG(dtable);
  if (S == 0) {   // no distances: the table's gradient is zero
    KRSI_CUDA_TRY(cudaMemsetAsync(dtable, 0, (size_t)num_buckets * H * (table_dtype == KRSI_F32 ? 4 : 2), stream));
    return KRSI_OK;
  }
  KRSI_CHECK_ARG(dpd);
  if (S > (1 << 30)) return KRSI_ERR_UNSUPPORTED;
  const int64_t warps = (int64_t)num_buckets * H;
  const dim3 grid((unsigned)((warps + 7) / 8));
#define KRSI_T5B(DT)                                                                                        \
  KRSI_CUDA_TRY(launch_pdl(t5_bias_bwd_kernel<DT>, grid, dim3(256), 0, stream, dpd,                         \
                           (typename Elem<DT>::T*)dtable, S, (int)H, num_buckets, m))
  if (table_dtype == KRSI_F32) KRSI_T5B(KRSI_F32);
  else if (table_dtype == KRSI_BF16) KRSI_T5B(KRSI_BF16);
  else KRSI_T5B(KRSI_F16);
#undef KRSI_T5B
  return KRSI_OK;
}
