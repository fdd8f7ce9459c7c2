/*
 * krsi_b200.h - C ABI of the B200 (sm_100a) kernels behind kernel-rsi's library ops.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t, launches
 * asynchronously on that stream, never synchronises, never allocates device memory and
 * returns a krsi_status code (0 = success).  Callers own all buffers; kernels that need
 * scratch memory take a caller-provided workspace whose size is reported by the matching
 * *_workspace_size() query.  Calls run on the CUDA context current to the calling thread,
 * and the stream must belong to that context.
 *
 * Each function names the reference interface it replaces (file:line inside the
 * kernel-rsi project).  Tensor layouts are the reference's:
 *   - rows are contiguous, row-major ("x2d" [rows, n], "u" [rows, 2F]);
 *   - qkv is [B*S, 3*H*D] with row stride `qkv_row_stride` elements and column layout
 *     [3][H][D]; out/out32 are [B*S, H*D] contiguous; lse and delta are [B*H, S];
 *   - pd is the per-head, per-distance bias [H, 2S-1] fp32:
 *     bias[h, i, j] = pd[h, j - i + S - 1].
 */
#ifndef KRSI_B200_H
#define KRSI_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
typedef enum {
  KRSI_OK = 0,
  KRSI_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, stride or dtype combination   */
  KRSI_ERR_UNSUPPORTED = 2,      /* valid for the reference, not implemented here         */
  KRSI_ERR_MISALIGNED = 3,       /* pointer/stride alignment required by TMA or vector IO */
  KRSI_ERR_WORKSPACE = 4,        /* workspace pointer null or smaller than required       */
  KRSI_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed (launch, attribute) */
  KRSI_ERR_DEVICE_TIMEOUT = 6    /* a bounded device-side wait gave up (see status read)  */
} krsi_status;

/* Element types accepted by the entry points. */
typedef enum { KRSI_F32 = 0, KRSI_BF16 = 1, KRSI_F16 = 2 } krsi_dtype;

/* Human-readable text for a krsi_status value. */
const char* krsi_error_string(int status);

/* ABI version: major*10000 + minor*100 + patch. */
int krsi_abi_version(void);

/* Reads (and optionally clears) the device-side watchdog word of the current device:
 * 0 when no bounded wait ever gave up, else a KRSI_ERR_DEVICE_TIMEOUT code with the
 * waiting role in bits 8..15.  Synchronises the current device; not for hot paths. */
int krsi_device_status(int* status_out, int clear);

/* ---------------------------------------------------------------- RMSNorm
 * y = w * (x * rstd).to(w.dtype), rstd = 1/sqrt(mean(x^2) + eps), per row.
 * Replaces library/rmsnorm.py:54-59 (_fwd -> _rms_fwd, rmsnorm.py:22-31).
 * x, y: [rows, n] of x_dtype; w: [n] of w_dtype; rstd: [rows] fp32. */
int krsi_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd,
                     int64_t rows, int64_t n, float eps,
                     int x_dtype, int w_dtype, cudaStream_t stream);

/* Bytes of workspace krsi_rmsnorm_bwd needs (the per-block dw partial sums). */
int krsi_rmsnorm_bwd_workspace_size(int64_t rows, int64_t n, size_t* bytes);

/* dx = r*dn - x*r^3*mean(dn*x) with dn = (g*w) rounded to the promoted input type;
 * dw = sum over rows of g * (x*r).to(w.dtype), reduced deterministically in two stages.
 * Replaces library/rmsnorm.py:62-68 (_bwd -> _rms_bwd, rmsnorm.py:34-51, then dwp.sum(0) at :68).
 * g, x, dx: [rows, n] of x_dtype; w, dw: [n] of w_dtype; rstd: [rows] fp32. */
int krsi_rmsnorm_bwd(const void* g, const void* x, const void* w, const float* rstd,
                     void* dx, void* dw, void* workspace, size_t workspace_bytes,
                     int64_t rows, int64_t n, int x_dtype, int w_dtype, cudaStream_t stream);

/* The same backward with a second gradient of x added: dx = (the backward above) + gadd, rounded
 * once.  For a pre-norm residual block, where x also feeds the residual branch and autograd would
 * otherwise add the two gradients of x in a separate pass (read both, write the sum).  No
 * counterpart in the reference (its backward returns dx alone, rmsnorm.py:62-68).
 * gadd: [rows, n] of x_dtype (16-byte aligned when n is a multiple of the vector width). */
int krsi_rmsnorm_bwd_add(const void* g, const void* x, const void* w, const float* rstd, const void* gadd,
                         void* dx, void* dw, void* workspace, size_t workspace_bytes,
                         int64_t rows, int64_t n, int x_dtype, int w_dtype, cudaStream_t stream);

/* The same backward for callers that cannot allocate device memory (a host that owns all device
 * memory, or a loop that must not stall on cudaMalloc): the dw partial sums live in a fixed
 * device array inside this library (4 MiB per GPU that loads it, kept until the process exits)
 * instead of a caller workspace.  No counterpart in the reference (its backward allocates
 * through torch, rmsnorm.py:66).
 * Limit: (dw partial rows) x n <= 1,048,576 floats.  The partial-row count is
 * min(ceil(rows / 8), 296) when one warp handles a row (rows of up to 2048 fp32 or 4096
 * 16-bit elements, 16-byte aligned) and min(rows, 296) otherwise; for example rows = 2048,
 * n = 1152 uses 256 x 1152.  Larger problems return KRSI_ERR_UNSUPPORTED.
 * Every call looks up the array's address (cudaGetSymbolAddress) in the current context, so a
 * device reset never leaves a stale pointer; the first call on a device also loads the module,
 * so make it before any stream capture.  All calls share the array:
 * calls whose kernels overlap on the GPU (different streams, same device) race and corrupt dw.
 * Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
int krsi_rmsnorm_bwd_noalloc(const void* g, const void* x, const void* w, const float* rstd,
                             void* dx, void* dw, int64_t rows, int64_t n, int x_dtype, int w_dtype,
                             cudaStream_t stream);

/* ---------------------------------------------------------------- GEGLU
 * out = gelu_tanh(u[:, :F]).to(dtype) * u[:, F:].
 * Replaces library/geglu.py:55-61 (_fwd -> _geglu_fwd, geglu.py:27-35).
 * u: [rows, 2F]; out: [rows, F]; both of `dtype`. */
int krsi_geglu_fwd(const void* u, void* out, int64_t rows, int64_t F, int dtype,
                   cudaStream_t stream);

/* du = [d(gate) | d(value)] in one [rows, 2F] tensor.
 * Replaces library/geglu.py:64-68 (_bwd -> _geglu_bwd, geglu.py:38-52).
 * g: [rows, F]; u, du: [rows, 2F]; all of `dtype`. */
int krsi_geglu_bwd(const void* g, const void* u, void* du, int64_t rows, int64_t F,
                   int dtype, cudaStream_t stream);

/* The gate|value projection with GEGLU in its epilogue (tcgen05 GEMM, fp32 accumulate):
 *   u = x @ w^T (rounded to dtype), out = gelu_tanh(u[:, :F]).to(dtype) * u[:, F:]
 * with krsi_geglu_fwd's arithmetic on the rounded u, so out equals krsi_geglu_fwd(u) bit for bit.
 * Replaces the T5 feed-forward's `geglu(h @ wi.T)`: the projection followed by
 * library/geglu.py:104-108 (geglu -> _fwd, geglu.py:55-61 -> _geglu_fwd, geglu.py:27-35).
 * x: [rows, K]; w: [2F, K] (rows [0, F) gate, [F, 2F) value); u: [rows, 2F]; out: [rows, F];
 * all of `dtype` (BF16 or F16), contiguous, 16-byte aligned; K and F multiples of 8. */
int krsi_linear_geglu_fwd(const void* x, const void* w, void* u, void* out, int64_t rows,
                          int64_t K, int64_t F, int dtype, cudaStream_t stream);

/* The down projection's input gradient with GEGLU's backward in its epilogue (tcgen05 GEMM):
 *   g = dy @ w (fp32 accumulate, rounded to dtype; never written), du = geglu_bwd(g, u)
 * with krsi_geglu_bwd's arithmetic, so du equals krsi_geglu_bwd(g, u) bit for bit for the rounded g.
 * Replaces the backward of the T5 feed-forward's `geglu(h @ wi.T) @ wo.T` from the down projection's
 * input gradient through GEGLU: `dy @ wo` followed by library/geglu.py:64-68 (_bwd -> _geglu_bwd,
 * geglu.py:38-52).
 * dy: [rows, K]; w: [K, F] (the down projection's weight, nn.Linear layout); u: [rows, 2F] (the
 * gate|value projection's output); du: [rows, 2F]; all of `dtype` (BF16 or F16), contiguous,
 * 16-byte aligned; K and F multiples of 8. */
int krsi_linear_geglu_bwd(const void* dy, const void* w, const void* u, void* du, int64_t rows,
                          int64_t K, int64_t F, int dtype, cudaStream_t stream);

/* ---------------------------------------------------------------- relpos attention
 * Flash attention with an additive Toeplitz bias, non-causal:
 *   s2[i,j] = (q_i . k_j * scale + pd[h, j-i+S-1]) * log2(e),  p = softmax over j,
 *   out = p @ v  (bf16 or f16, [B*S, H*D]),  out32 = same in fp32,
 *   lse[b*H+h, i] = max_j s2 + log2(sum_j exp2(s2 - max))   (log2 domain).
 * Replaces library/relpos_attention.py:132-140 (_forward -> _fwd, relpos_attention.py:26-59).
 * D must be a multiple of 8 and <= 128; qkv_row_stride a multiple of 8; dtype BF16 or F16. */
int krsi_relpos_attn_fwd(const void* qkv, int64_t qkv_row_stride, const float* pd,
                         void* out, float* out32, float* lse,
                         int64_t B, int64_t S, int64_t H, int64_t D, float scale,
                         int dtype, cudaStream_t stream);

/* Bytes of workspace krsi_relpos_attn_bwd needs (delta, fp32 dQ accumulator,
 * per-tile dBias diagonal partials). */
int krsi_relpos_attn_bwd_workspace_size(int64_t B, int64_t S, int64_t H, int64_t D,
                                        size_t* bytes);

/* Gradients of the forward above for upstream gradient dout [B*S, H*D] (contiguous):
 *   dqkv [B*S, 3*H*D] (row stride dqkv_row_stride, same [3][H][D] column layout),
 *   dpd  [H, 2S-1] fp32 = sum over batch of the diagonal sums of dS (unscaled).
 * delta = rowsum(dout * out32) is computed from the fp32 copy of O.
 * Replaces library/relpos_attention.py:143-157 (_backward_impl -> _bwd_dkdv :62-94,
 * _bwd_dq :97-126 and the torch diagonal reduction :154-156). */
int krsi_relpos_attn_bwd(const void* dout, const void* qkv, int64_t qkv_row_stride,
                         const float* pd, const float* out32, const float* lse,
                         void* dqkv, int64_t dqkv_row_stride, float* dpd,
                         void* workspace, size_t workspace_bytes,
                         int64_t B, int64_t S, int64_t H, int64_t D, float scale,
                         int dtype, cudaStream_t stream);

/* ---------------------------------------------------------------- T5 bucketed relative position
 * The step either side of the attention op in a T5 model (its relative_attention_bias table).
 * T5's bucket of a distance rel = key - query (HF transformers T5Attention._relative_position_bucket,
 * models/t5/modeling_t5.py): with n = num_buckets / 2 if bidirectional (rel > 0 adds n) else
 * num_buckets, e = n / 2 and a = |rel| (bidirectional) or max(-rel, 0): bucket offset a for a < e,
 * else e + trunc(log(a / e) / log(max_distance / e) * (n - e)), capped at n - 1.
 * The reference's attention op takes the bias per distance (pd [H, 2S-1], relpos_attention.py:5);
 * the reference leaves the table -> pd step and its gradient to torch (an embedding lookup, and
 * an S x S scatter-add in its backward, LESSONS.md:35). */

/* Bucket of one distance (host-side, no device work): the map the kernels below use. */
int krsi_t5_bucket(int num_buckets, int max_distance, int bidirectional, int64_t rel, int* bucket);

/* pd[h, t] = table[bucket(t - (S - 1)), h] for t in [0, 2S - 1).
 * table: [num_buckets, H] of table_dtype (F32, BF16, F16); pd: [H, 2S - 1] fp32. */
int krsi_t5_bias_fwd(const void* table, float* pd, int64_t S, int64_t H, int num_buckets, int max_distance,
                     int bidirectional, int table_dtype, cudaStream_t stream);

/* dtable[k, h] = sum of dpd[h, t] over the distances t - (S - 1) in bucket k (a segmented sum in a
 * fixed order: deterministic), rounded to table_dtype.  dpd: [H, 2S - 1] fp32. */
int krsi_t5_bias_bwd(const float* dpd, void* dtable, int64_t S, int64_t H, int num_buckets, int max_distance,
                     int bidirectional, int table_dtype, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* KRSI_B200_H */
