/*
 * fxpr_b200.h -- C ABI of the B200-native fixed-point reduction (FxPR) hot path.
 *
 * Plain C: pointers, sizes and strides (in elements), no torch types. Every
 * entry point enqueues work on the CUDA stream passed as `stream` (a
 * cudaStream_t, NULL = legacy default stream), never synchronises, never
 * allocates, and returns FXPR_OK (0) or a negative error code; the message of
 * the last error on the calling thread is returned by fxpr_last_error().
 *
 * Numerics follow the reference plugin (Gursukh/Fixed-Point-Reductions-For-vLLM,
 * Triton kernels) bit for bit: F2X = scale by 2^frac_bits, clamp to
 * [-2^(b-1), 2^(b-1) - 2^s] (s = max(0, b - mantissa bits of the input float)),
 * round to nearest even, cast; X2F = int -> float (RNE) times 2^-frac_bits;
 * integer accumulation wraps at the accumulator width b in {16, 32, 64}.
 */
#ifndef FXPR_B200_H
#define FXPR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FXPR_ABI_VERSION 3

/* error codes */
#define FXPR_OK 0
#define FXPR_ERR_INVALID (-1)     /* bad argument (shape, dtype, bits, alignment) */
#define FXPR_ERR_UNSUPPORTED (-2) /* valid in the reference, not implemented here */
#define FXPR_ERR_CUDA (-3)        /* a CUDA launch/runtime call failed */

/* dtype codes */
#define FXPR_F16 0
#define FXPR_BF16 1
#define FXPR_F32 2
#define FXPR_F64 3
#define FXPR_I16 10
#define FXPR_I32 11
#define FXPR_I64 12

int fxpr_abi_version(void);
const char* fxpr_last_error(void);

/* Elementwise F2X of n contiguous floats (x_dtype F16/F32/F64; BF16 is
 * rejected like the reference's static_assert) into int_bits-wide integers.
 * Replaces fxpr_vllm/fixed_point_kernels/fixed_point.py:25-53 (float_to_fixed). */
int fxpr_float_to_fixed(const void* x, int x_dtype, void* q, int int_bits, int64_t n,
                        int frac_bits, void* stream);

/* Elementwise X2F of n contiguous int_bits-wide integers into y_dtype
 * (F16/F32/F64). Replaces fixed_point.py:56-69 (fixed_to_float). */
int fxpr_fixed_to_float(const void* q, int int_bits, void* y, int y_dtype, int64_t n,
                        int frac_bits, void* stream);

/* Fixed-point sum over the last dim of a [rows, cols] matrix (row stride in
 * elements): per-element F2X into int_bits, exact int64 sum, saturating clamp
 * to the int_bits range, X2F into fp32 out[rows]. x_dtype F16/BF16/F32/F64
 * (BF16 widened exactly to fp32). Semantics of tests/test_sum.py:13-29 (the
 * reference has no kernel for it). */
int fxpr_fxp_sum(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t row_stride,
                 float* out, int frac_bits, int int_bits, void* stream);

/* Workspace bytes needed by fxpr_gemm_fxp for this shape on the current
 * device (0 when no split-K is used). The workspace must be zero-filled
 * before its first use; every call leaves it zero-filled again. Calls that
 * share a workspace must be ordered on one stream. */
int64_t fxpr_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int int_bits);

/* Fixed-point GEMM C[M,N] = X2F(sum_k F2X(fp32(a[m,k]) * fp32(b[k,n]))).
 * a, b: F16/BF16/F32 with arbitrary strides (elements). out_kind 0: c is fp32
 * (the reference's output); out_kind 1: c holds the raw integer accumulator
 * (int32 for int_bits 16/32 -- only the low 16 bits matter for 16 --, int64
 * for 64), used before an integer tensor-parallel allreduce.
 * Replaces fxpr_vllm/library_ops.py:14-45 (fxpr::gemm_fxp) and
 * fixed_point_kernels/gemm.py:97-196. */
int fxpr_gemm_fxp(const void* a, int a_dtype, int64_t sam, int64_t sak, const void* b,
                  int b_dtype, int64_t sbk, int64_t sbn, void* c, int out_kind, int64_t scm,
                  int64_t scn, int64_t M, int64_t N, int64_t K, int frac_bits, int int_bits,
                  void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free fxpr_gemm_fxp for callers that cannot allocate device
 * memory (a serving engine with a fixed, pre-planned memory budget, or a
 * foreign-language binding with no device allocator). No counterpart in the
 * reference. The split-K scratch is a fixed 8 MiB array inside the library,
 * one per device; shapes needing more are rejected with FXPR_ERR_INVALID.
 * The first call on a device looks the array up (make it before any stream
 * capture); the lookup is safe to race from several host threads. Calls that
 * overlap on the GPU share the array and race. */
int fxpr_gemm_fxp_noalloc(const void* a, int a_dtype, int64_t sam, int64_t sak, const void* b,
                          int b_dtype, int64_t sbk, int64_t sbn, void* c, int out_kind,
                          int64_t scm, int64_t scn, int64_t M, int64_t N, int64_t K,
                          int frac_bits, int int_bits, void* stream);

/* Epilogue of a row-parallel linear layer after the integer allreduce:
 * out[m,n] = cast(X2F(acc[m,n]) + fp32(bias[n])) with acc int32 (int_bits 16:
 * low 16 bits, 32) or int64 (64); bias may be NULL; out_dtype F16/BF16/F32.
 * Replaces quantisation_config.py:181-187 (fixed_to_float + bias + cast). */
int fxpr_fixed_to_float_bias(const void* acc, int int_bits, int64_t M, int64_t N,
                             int64_t acc_row_stride, const void* bias, int bias_dtype, void* out,
                             int out_dtype, int64_t out_row_stride, int frac_bits, void* stream);

/* Fixed-point RMSNorm over rows of length `hidden` (rms_norm.py:10-60):
 * optional fused residual (x = x + residual in fp32; the sum is written back
 * to residual in residual's dtype; the fp32 sum is normalised), F2X of x^2,
 * integer row sum (int16 F2X summed in int32 like tl.sum), X2F,
 * rrms = 1/sqrt(max(S/hidden, 0) + eps) with the reference's fast divide and
 * square root, y = (x * w) * rrms in y_dtype. residual may be NULL.
 * Replaces library_ops.py:53-126 (fxpr::rms_norm_fxp, fxpr::rms_norm_fxp_residual). */
int fxpr_rms_norm_fxp(const void* x, int x_dtype, int64_t x_row_stride, const void* w,
                      int w_dtype, void* y, int y_dtype, int64_t y_row_stride, void* residual,
                      int res_dtype, int64_t res_row_stride, int64_t rows, int64_t hidden,
                      float eps, int frac_bits, int int_bits, void* stream);

/* Row-parallel linear epilogue fused with the residual RMSNorm: per row,
 * h = cast_act(X2F(acc) + fp32(bias)) (the linear layer's output, acc int32
 * for int_bits 16/32 -- low 16 bits for 16 -- or int64), v = fp32(h) +
 * fp32(residual) written back to residual in act_dtype, y = fixed-point
 * RMSNorm of v (as fxpr_rms_norm_fxp) in act_dtype. bias may be NULL.
 * Replaces the pair quantisation_config.py:181-187 (fixed_to_float + bias +
 * cast after the allreduce) and library_ops.py:88-126
 * (fxpr::rms_norm_fxp_residual) with one pass; same bits. */
int fxpr_fixed_to_float_add_rms_norm(const void* acc, int int_bits, int64_t acc_row_stride,
                                     const void* bias, int bias_dtype, void* residual, int act_dtype,
                                     int64_t res_row_stride, const void* w, int w_dtype, void* y,
                                     int64_t y_row_stride, int64_t rows, int64_t hidden, float eps,
                                     int frac_bits, void* stream);

/* Paged unified (prefill + decode) attention with fixed-point softmax
 * normaliser and PV accumulation and a bit-exact integer split-KV combine.
 * Replaces fixed_point_kernels/attention.py:398-489 (unified_attention_fxp)
 * and attention.py:18-395; strides are in elements. */
typedef struct fxpr_attention_params {
  const void* q;               /* [tokens, num_heads, head_dim] */
  int q_dtype;
  int64_t q_stride_tok, q_stride_head;
  const void* k_cache;         /* [blocks, page, num_kv_heads, head_dim] view */
  const void* v_cache;
  int kv_dtype;
  int64_t k_stride_blk, k_stride_slot, k_stride_head;
  int64_t v_stride_blk, v_stride_slot, v_stride_head;
  void* o;                     /* [tokens, num_heads, head_dim] */
  int o_dtype;
  int64_t o_stride_tok, o_stride_head;
  const int32_t* query_start_loc; /* [num_requests + 1] */
  const int32_t* seq_lens;        /* [num_requests] */
  const int32_t* block_table;     /* [num_requests, bt_stride] */
  int64_t bt_stride;
  int32_t block_table_cols;       /* columns of block_table */
  int32_t max_seq_len;            /* bound on seq_lens, 0 = block_table_cols * page_size */
  const float* alibi_slopes;      /* [num_heads], pre-scaled by 1/ln2, or NULL */
  int32_t num_requests, max_query_len, num_heads, num_kv_heads, head_dim, page_size;
  int32_t is_causal, window_size;
  float scale_log2;               /* softmax_scale * (1/ln2), rounded to fp32 */
  float logits_soft_cap;          /* logits_soft_cap * (1/ln2) as fp32; 0 = off */
  int32_t frac_bits, int_bits;    /* int_bits 32 or 64 */
  int32_t num_kv_splits;          /* performance knob; results do not depend on it */
  void* workspace;                /* optional scratch, 256-byte aligned, any contents;
                                     NULL = cluster path without scratch */
  int64_t workspace_bytes;
  int64_t num_blocks;             /* blocks in the paged cache (leading dim), 0 = unknown;
                                     with it, decode batches take the TMA page path and a
                                     block id outside [0, num_blocks) reads zeros */
} fxpr_attention_params;

int fxpr_unified_attention_fxp(const fxpr_attention_params* p, void* stream);

/* Workspace bytes that enable the chunked two-kernel path for this shape
 * (fixed chunks of keys, uniform work units; results identical to the
 * cluster path), or 0 when the shape uses the cluster path. Depends on
 * num_requests, max_query_len, head counts, head_dim, kv dtype and
 * max_seq_len (or block_table_cols * page_size). max_seq_len must bound
 * every seq_lens entry. Calls sharing a workspace must be ordered on one
 * stream. Same interface as fxpr_unified_attention_fxp (attention.py:398-489);
 * the reference has no workspace. */
int64_t fxpr_attention_workspace_bytes(const fxpr_attention_params* p);

/* Row-wise log-softmax with a fixed-point exp-sum (softmax.py:8-97): logits
 * rounded to fp16 before the max and exp, [rows, n] fp32 in/out. */
int fxpr_log_softmax_fxp(const float* x, int64_t x_row_stride, float* y, int64_t y_row_stride,
                         int64_t rows, int64_t n, int frac_bits, int int_bits, void* stream);

/* Test hook: evaluates on the device the fp32 primitives the kernels use
 * where the reference relies on the GPU compiler's rounding. op: 0 exp2(a),
 * 1 a / b (fast divide), 2 sqrt(a) (fast), 3 tanh(a), 4 exp(a), 5 log(a). */
int fxpr_probe_prims(int op, const float* a, const float* b, float* out, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FXPR_B200_H */
