/*
 * ak_b200.h -- C ABI of libak_b200.so, the sm_100a (B200) implementation of
 * AutoKernel's nine-operator kernel_fn contract.
 *
 * Conventions (all entry points):
 *   - Plain device pointers, element counts and element strides; no framework
 *     types.  `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Work is enqueued asynchronously on that stream.
 *   - The caller allocates every input, output and workspace buffer; the
 *     library never allocates device memory.
 *   - Return AK_OK (0) or a negative AK_ERR_* code; ak_last_error() returns a
 *     thread-local message for the last failure.  Nothing aborts or traps.
 *   - dtype is one of AK_F32 / AK_F16 / AK_BF16; arithmetic accumulates in
 *     fp32 (fp64 for cross-CTA sums), results are bitwise deterministic for a
 *     given device, shape and dtype.
 *
 * Each declaration names the reference interface it replaces.  Paths are
 * relative to the AutoKernel repository root.
 */
#ifndef AK_B200_H_
#define AK_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AK_API __attribute__((visibility("default")))
#else
#define AK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AK_VERSION 1

enum ak_dtype { AK_F32 = 0, AK_F16 = 1, AK_BF16 = 2 };

enum ak_status {
  AK_OK = 0,
  AK_ERR_ARG = -1,         /* null pointer, bad workspace, bad enum */
  AK_ERR_DTYPE = -2,       /* dtype not supported by this op */
  AK_ERR_SHAPE = -3,       /* inconsistent or out-of-range sizes */
  AK_ERR_ALIGN = -4,       /* alignment the op cannot handle */
  AK_ERR_LAUNCH = -5,      /* CUDA launch / driver error */
  AK_ERR_UNSUPPORTED = -6  /* feature not available on this device */
};

enum ak_activation { AK_ACT_SILU = 0, AK_ACT_GELU = 1, AK_ACT_RELU2 = 2 };

/* Codes written to the device status word by bounded spin-waits. */
#define AK_STATUS_TIMEOUT 1

/* ----------------------------------------------------------------- utilities */
AK_API const char* ak_last_error(void);
AK_API int ak_version(void);
/* Reads (and optionally clears) the device status word; synchronous. */
AK_API int ak_device_status(int clear);
AK_API int ak_sm_count(void);
/* Test hook: 1 routes matmul/MLP/attention through the SIMT kernels. */
AK_API void ak_set_force_simt(int on);

/* ----------------------------------------------------------------- row ops */

/* y = x / sqrt(mean(x^2, -1) + eps) * w over rows of length `cols`, with reference.py's
 * rounding: each of x*x, the mean, + eps, sqrt, x / rms and * w is rounded to the input
 * dtype (the mean's sum accumulates in fp32), so fp16 inputs with |x| > 256 overflow x*x
 * exactly as the reference does.
 * Replaces kernels/rmsnorm.py:45 kernel_fn(x, weight, eps) and
 * kernels/cuda/rmsnorm.py:171 (reference oracle reference.py:26-29). */
AK_API int ak_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t cols, int64_t ldx,
               int64_t ldy, float eps, int dtype, void* stream);

/* y = x * rsqrt(mean(x^2, -1) + eps) * w with every intermediate in fp32 and one rounding:
 * the RMSNorm of models/llama_7b.py:22-30 (RMSNorm.forward) without its 16-bit overflow of
 * x^2; used by the model path. */
AK_API int ak_rmsnorm_fp32(const void* x, const void* w, void* y, int64_t rows, int64_t cols,
                    int64_t ldx, int64_t ldy, float eps, int dtype, void* stream);

/* y = (x - mean) / sqrt(var + eps) * w + b over rows.
 * Replaces kernels/layernorm.py:65 kernel_fn(x, weight, bias, eps)
 * (reference.py:20-23). */
AK_API int ak_layernorm(const void* x, const void* w, const void* b, void* y, int64_t rows,
                 int64_t cols, int64_t ldx, int64_t ldy, float eps, int dtype, void* stream);

/* y = softmax(x, -1) over rows.  Replaces kernels/softmax.py:57 kernel_fn(x)
 * (reference.py:15-17). */
AK_API int ak_softmax(const void* x, void* y, int64_t rows, int64_t cols, int64_t ldx, int64_t ldy,
               int dtype, void* stream);

/* Interleaved-pair RoPE on contiguous x/y [rows, head_dim]; cos/sin are
 * contiguous [cs_rows, head_dim/2] and row r uses cos/sin row
 * (r / cs_div) % cs_rows.  cs_dtype is dtype or AK_F32.
 * Replaces kernels/rotary_embedding.py:75 kernel_fn(x, cos, sin)
 * (reference.py:63-69). */
AK_API int ak_rotary_embedding(const void* x, const void* cos, const void* sin, void* y, int64_t rows,
                        int64_t head_dim, int64_t cs_div, int64_t cs_rows, int dtype,
                        int cs_dtype, void* stream);

/* ----------------------------------------------------------------- reductions */

/* out[o, i] = sum_r x[o, r, i] for contiguous x viewed as [outer, n, inner].
 * Replaces kernels/reduce.py:51 kernel_fn(x, dim) (reference.py:72-74). */
AK_API int ak_reduce_sum(const void* x, void* out, int64_t outer, int64_t n, int64_t inner, int dtype,
                  int out_dtype, void* stream);

/* Bytes of workspace ak_reduce_sum_full needs on the current device. */
AK_API size_t ak_reduce_workspace_size(void);

/* Sum of all n elements of contiguous x.  Writes the fp64 total to *total
 * (device pointer, may be NULL) and, if out != NULL, the total cast to
 * out_dtype to *out.  The fp64 total is the per-rank partial that a sharded
 * caller all-reduces.  Same reference entry as ak_reduce_sum, for 1-D x. */
AK_API int ak_reduce_sum_full(const void* x, int64_t n, int dtype, double* total, void* out,
                       int out_dtype, void* workspace, size_t ws_bytes, void* stream);

/* Same result as ak_reduce_sum_full, for callers that cannot allocate device memory (they
 * run inside another framework's allocator or a host that forbids cudaMalloc after start-up).
 * No counterpart in the reference.  The per-CTA scratch lives in a 16 KiB array inside the
 * library (held by every GPU that loads it until exit); the first call on a device looks up
 * its address and should come before any stream capture.  Calls on one device share that
 * array: calls that overlap on the GPU race.  Fails with AK_ERR_SHAPE if the device needs more
 * than 2048 partial slots (4 per SM).  Allocates nothing. */
AK_API int ak_reduce_sum_full_noalloc(const void* x, int64_t n, int dtype, double* total,
                                      void* out, int out_dtype, void* stream);

/* *out = (out_dtype) *total (both device pointers). */
AK_API int ak_scalar_from_sum(const double* total, void* out, int out_dtype, void* stream);

/* Per-row cross entropy: row_loss[r] = logsumexp(logits[r]) - logits[r, t_r]
 * (0 where t_r == ignore_index).  row_max / row_target_logit (optional, may
 * be NULL) receive the row max and the gathered target logit as fp32; both
 * are exact copies of input values.  *bad_target (optional) is set to 1 if a
 * target is outside [0, vocab) and not ignore_index.
 * Replaces kernels/cross_entropy.py:70 kernel_fn(logits, targets)
 * (reference.py:58-60). */
AK_API int ak_cross_entropy_rows(const void* logits, const int64_t* targets, int64_t rows,
                          int64_t vocab, int64_t ld, int dtype, int64_t ignore_index,
                          float* row_loss, float* row_max, float* row_target_logit,
                          int* bad_target, void* stream);

/* Fixed-order fp64 sum of row_loss over non-ignored rows.  sum_count (device,
 * may be NULL) receives {sum, count}; out (may be NULL) receives sum/count in
 * out_dtype. */
AK_API int ak_cross_entropy_finalize(const float* row_loss, const int64_t* targets, int64_t rows,
                              int64_t ignore_index, double* sum_count, void* out,
                              int out_dtype, void* stream);

/* *out = sum_count[0] / sum_count[1] in out_dtype (after an all-reduce). */
AK_API int ak_mean_from_sum_count(const double* sum_count, void* out, int out_dtype, void* stream);

/* LM head fused with cross entropy: row_loss[r] = logsumexp(z_r) - z_r[t_r] for the logits
 * z = x @ w^T (x [rows, dim], w [vocab, dim] row-major, 16-bit), without storing z.  Each
 * logit is rounded to the dtype before it enters the loss, so row_max / row_target_logit
 * (optional) are bitwise those of ak_matmul followed by ak_cross_entropy_rows.  Rows with
 * t_r == ignore_index get loss 0; other targets outside [0, vocab) give NaN and set
 * *bad_target.  workspace: ak_linear_cross_entropy_workspace_size(rows, vocab) bytes
 * (per-row partials of each 256-column vocab tile).  Finish with ak_cross_entropy_finalize.
 * Replaces the output projection + loss of models/llama_7b.py:199-209 as evaluated by
 * reference.py:58-60 (cross_entropy_ref over the LM head's logits). */
AK_API size_t ak_linear_cross_entropy_workspace_size(int64_t rows, int64_t vocab);
AK_API int ak_linear_cross_entropy_rows(const void* x, const void* w, const int64_t* targets,
                                 int64_t rows, int64_t vocab, int64_t dim, int64_t ldx,
                                 int64_t ldw, int dtype, int64_t ignore_index, void* workspace,
                                 size_t ws_bytes, float* row_loss, float* row_max,
                                 float* row_target_logit, int* bad_target, void* stream);

/* ----------------------------------------------------------------- contractions */

/* C[M, N] = A[M, K] @ B where B is [K, N] row-major (b_kmajor = 0) or the
 * transpose of an [N, K] row-major matrix (b_kmajor = 1).  Leading
 * dimensions in elements.  Replaces kernels/matmul.py:62 kernel_fn(A, B) and
 * kernels/cuda/matmul.py:246 (reference.py:10-12). */
AK_API int ak_matmul(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
              int64_t lda, int64_t ldb, int64_t ldc, int b_kmajor, int dtype, void* stream);

/* C[M, N] = A @ B + R: ak_matmul with a residual [M, N] (leading dimension ldr) added in the
 * epilogue before rounding; R may alias C (in-place residual update, each element read then
 * written by the same thread).  Fuses the residual adds around the o-projection and the MLP
 * down projection of models/llama_7b.py:110-111 into the GEMM (fused neighbour of the path;
 * matmul semantics of reference.py:10-12). */
AK_API int ak_matmul_add(const void* A, const void* B, void* C, const void* R, int64_t M,
                         int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                         int64_t ldr, int b_kmajor, int dtype, void* stream);

/* out[M, N] = x[M, K] @ w[N, K]^T with rotary embedding applied in the GEMM epilogue to
 * output columns [0, rope_cols): interleaved (even, odd) pairs within head_dim-wide column
 * groups, position = row % T, fp32 cos/sin [T, head_dim / 2].  Fuses the fused q/k/v
 * projection with apply_rotary_emb (models/llama_7b.py:40-48, 67-71; RoPE math of
 * reference.py:63-69).  16-bit inputs, tensor-core path only (AK_ERR_UNSUPPORTED otherwise). */
AK_API int ak_linear_rope(const void* x, const void* w, void* out, int64_t M, int64_t N,
                          int64_t K, int64_t ldx, int64_t ldo, const float* cos,
                          const float* sin, int64_t T, int64_t head_dim, int64_t rope_cols,
                          int dtype, void* stream);

/* hidden[M, H] = act(x @ w_gate^T) * (x @ w_up^T) for contiguous x [M, D],
 * w_gate / w_up [H, D].  First stage of kernels/fused_mlp.py:102. */
AK_API int ak_mlp_gate_up(const void* x, const void* w_gate, const void* w_up, void* hidden, int64_t M,
                   int64_t D, int64_t H, int activation, int dtype, void* stream);

/* RMSNorm folded into the projections that read it (models/llama_7b.py:22-30 in front of
 * the q/k/v projections and the feed-forward): with the norm weight folded into the
 * projection weight (w' = w * diag(norm.weight)), RMSNorm(x) @ w^T equals (x @ w'^T) scaled
 * per row by 1 / sqrt(mean(x^2) + eps), so the normalised activations are never stored.  The
 * per-row mean comes from partial sums of squares ss[t][row] over 256-column tiles of x,
 * written by ak_row_sumsq or by the ss_out of the GEMM that produced x.
 *   ak_row_sumsq:        ss_out [ceil(cols / 256)][rows] for x [rows, cols] (16-bit).
 *   ak_linear_rms:       C = rowscale * (x @ w^T) [+ R] with x [M, K], w [N, K]; rs_in
 *                        (optional) the rs_tiles partials of x; ss_out (optional) receives
 *                        the partials [ceil(N / 256)][M] of the stored C (after + R), for the
 *                        next norm.  R may alias C (in-place residual update).  With cos
 *                        (optional) interleaved RoPE is applied to output columns
 *                        [0, rope_cols) before rounding, as in ak_linear_rope (position
 *                        row % T, fp32 cos/sin [T, head_dim / 2]).
 *   ak_mlp_gate_up_rms:  hidden = act(g) * u with g, u the row-scaled x @ w_gate^T,
 *                        x @ w_up^T (reference.py:45-55 rounding of the hidden).
 * 16-bit operands on the tensor-core path only (AK_ERR_ARG otherwise).  Fused neighbours of
 * the path: no single reference function; their parts are reference.py:26-29 / :10-12 /
 * :45-55. */
AK_API int ak_row_sumsq(const void* x, int64_t rows, int64_t cols, int64_t ld, int dtype,
                 float* ss_out, void* stream);
AK_API int ak_linear_rms(const void* x, const void* w, void* C, const void* R, int64_t M,
                  int64_t N, int64_t K, int64_t ldx, int64_t ldc, int64_t ldr,
                  const float* rs_in, int rs_tiles, float eps, float* ss_out, const float* cos,
                  const float* sin, int64_t T, int64_t head_dim, int64_t rope_cols, int dtype,
                  void* stream);
AK_API int ak_mlp_gate_up_rms(const void* x, const void* w_gate, const void* w_up, void* hidden,
                       int64_t M, int64_t D, int64_t H, const float* rs_in, int rs_tiles,
                       float eps, int activation, int dtype, void* stream);

/* out[M, D] = (act(x @ w_gate^T) * (x @ w_up^T)) @ w_down^T with w_down
 * [D, H]; `hidden` is caller workspace of M*H elements of dtype.
 * Replaces kernels/fused_mlp.py:102 kernel_fn(x, w_gate, w_up, w_down,
 * activation) (reference.py:45-55). */
AK_API int ak_fused_mlp(const void* x, const void* w_gate, const void* w_up, const void* w_down,
                 void* hidden, void* out, int64_t M, int64_t D, int64_t H, int activation,
                 int dtype, void* stream);

/* O = softmax(Q K^T * sm_scale [+ causal mask]) V for contiguous Q/O
 * [batch_heads, Sq, D] and K/V [batch_heads, Sk, D].  The causal mask hides
 * key j from query i when j > i (top-left aligned, like
 * torch.triu(ones(Sq, Sk), 1)).  Replaces kernels/flash_attention.py:130
 * kernel_fn(Q, K, V, causal, sm_scale) (reference.py:32-42). */
AK_API int ak_flash_attention(const void* Q, const void* K, const void* V, void* O,
                       int64_t batch_heads, int64_t Sq, int64_t Sk, int64_t D, int causal,
                       float sm_scale, int dtype, void* stream);

/* Attention on strided views: Q/O [B, H, Sq, D], K/V [B, Hkv, Sk, D] given by element
 * strides {batch, head, seq} (last dim contiguous), so [B, T, H, D] projection outputs are read
 * and written in place.  Query head h uses key/value head h / (H / Hkv) (grouped-query
 * attention).  Tensor-core path only: 16-bit dtypes, D in {64, 128}, strides multiples of 8
 * elements; otherwise AK_ERR_UNSUPPORTED.  Same math as ak_flash_attention
 * (kernels/flash_attention.py:130, reference.py:32-42; the GQA head mapping follows
 * models/llama_7b.py:78-80 repeat_interleave). */
AK_API int ak_flash_attention_strided(const void* Q, const void* K, const void* V, void* O,
                                      int64_t B, int64_t H, int64_t Hkv, int64_t Sq, int64_t Sk,
                                      int64_t D, const int64_t* q_strides,
                                      const int64_t* k_strides, const int64_t* v_strides,
                                      const int64_t* o_strides, int causal, float sm_scale,
                                      int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AK_B200_H_ */
