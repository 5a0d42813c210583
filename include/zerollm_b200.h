/*
 * zerollm_b200.h -- C ABI of the B200 (sm_100a) training-step library.
 *
 * Plain pointers and sizes only.  Every pointer argument is a DEVICE pointer
 * owned by the caller unless stated otherwise; no entry point allocates
 * device memory except zl_model_create / zl_model_attach_nccl (which own an
 * arena, like the reference's layers own their buffers).  Every entry point
 * returns a zl_status; zl_last_error() gives the message of the last failure
 * on the calling thread.  `stream` is a cudaStream_t (NULL = legacy stream).
 *
 * Reference interfaces replaced are cited as path:line inside buladuo/ZeroLLM.
 * The reference's own error convention (config.hpp:55-66: launch failures
 * throw std::runtime_error, bad sizes throw std::invalid_argument, some ops
 * silently return on size <= 0) is reproduced by the C++ wrappers in
 * zerollm_b200/csrc/api/; at this layer it maps to ZL_EINVAL / ZL_ECUDA /
 * ZL_OK-without-work respectively.
 */
#ifndef ZEROLLM_B200_H
#define ZEROLLM_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  ZL_OK = 0,
  ZL_EINVAL = 1,      /* bad sizes / null pointers (reference: std::invalid_argument) */
  ZL_ECUDA = 2,       /* CUDA launch or runtime error (reference: CHECK -> runtime_error) */
  ZL_ETIMEOUT = 3,    /* a bounded device wait or a collective timed out */
  ZL_ENCCL = 4,       /* NCCL error */
  ZL_ENOMEM = 5,      /* arena allocation failed */
  ZL_EUNSUPPORTED = 6,/* shape/layout outside what the kernel supports */
  ZL_ESTATE = 7,      /* call order violated (e.g. backward before forward) */
  ZL_EIO = 8          /* checkpoint file missing, short or unwritable (reference: runtime_error) */
} zl_status;

typedef void *zl_stream;
typedef uint16_t zl_bf16; /* raw bfloat16 bits */

const char *zl_last_error(void);
/* Reads (and clears) the device-side error word set by bounded waits. */
zl_status zl_device_error(int *code_out);
/* Library version string. */
const char *zl_version(void);

/* ===================================================================== */
/* Kernel API (fp32), one entry point per reference host launcher.        */
/* GEMMs whose reduction length is a multiple of 4 run on tcgen05         */
/* kind::tf32 (MN-major operands through a K-major copy in stream-ordered  */
/* scratch memory); other shapes use a SIMT fp32 kernel.                   */
/* ===================================================================== */
/* src/kernel/cuda/matmul.cuh:20 matmul and :68 matmul_tiled: C[M,N] = A[M,K] B[K,N] */
zl_status zl_matmul_f32(const float *A, const float *B, float *C, int M, int N, int K, zl_stream stream);
/* matmul.cuh:36 matmul_transposed_A_T_B and :99 (tiled): C[K,N] = A[M,K]^T B[M,N] (overwrites C) */
zl_status zl_matmul_at_b_f32(const float *A, const float *B, float *C, int M, int N, int K, zl_stream stream);
/* matmul.cuh:52 matmul_transposed_A_B_T and :83 (tiled): C[M,N] = A[M,K] B[N,K]^T */
zl_status zl_matmul_a_bt_f32(const float *A, const float *B, float *C, int M, int N, int K, zl_stream stream);
/* linear.cuh:21-30 linear_forward: out = in W^T (+ b) */
zl_status zl_linear_forward_f32(const float *input, const float *weight, const float *bias, float *output,
                                int64_t M, int64_t K, int64_t N, int use_bias, zl_stream stream);
/* linear.cuh:48-59 linear_backward: dX = dY W, dW = dY^T X (overwritten), dB += colsum(dY) */
zl_status zl_linear_backward_f32(const float *d_output, const float *input, const float *weight,
                                 float *d_input, float *d_weight, float *d_bias, int64_t M, int64_t K,
                                 int64_t N, int use_bias, zl_stream stream);
/* mha.cuh:18-24 mha_forward: causal/masked MHA, probabilities written to attention_scores [B,H,S,S]
 * (may be NULL: then only attn_output is produced). mask is [S,S] bool (1 = keep) or NULL. */
zl_status zl_mha_forward_f32(const float *Q, const float *K, const float *V, float *attn_output,
                             float *attention_scores, const uint8_t *mask, int64_t batch, int64_t seq_len,
                             int64_t num_heads, int64_t head_dim, int is_causal, zl_stream stream);
/* mha.cuh:38-48 mha_backward from stored probabilities.  reference_semantics=1 reproduces
 * mha.cu:284-295 exactly (dQ, dK without the 1/sqrt(Dh) factor); 0 gives the true gradient. */
zl_status zl_mha_backward_f32(const float *d_attn_output, const float *Q, const float *K, const float *V,
                              const float *attention_scores, const uint8_t *mask, float *d_Q, float *d_K,
                              float *d_V, int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim,
                              int is_causal, int reference_semantics, zl_stream stream);
/* layernorm.cuh:22-32 cuda_layernorm_forward (mean/rstd may be NULL) */
zl_status zl_layernorm_forward_f32(const float *input, const float *gamma, const float *beta, float *output,
                                   float *mean, float *rstd, int64_t M, int64_t N, float eps,
                                   zl_stream stream);
/* layernorm.cuh:50-61 cuda_layernorm_backward (d_gamma, d_beta accumulated) */
zl_status zl_layernorm_backward_f32(const float *input, const float *d_output, const float *gamma,
                                    const float *mean, const float *rstd, float *d_input, float *d_gamma,
                                    float *d_beta, int64_t M, int64_t N, zl_stream stream);
/* RMSNorm (no reference kernel; the BASELINE topology's norm): y = x rstd g */
zl_status zl_rmsnorm_forward_f32(const float *input, const float *gamma, float *output, float *rstd,
                                 int64_t M, int64_t N, float eps, zl_stream stream);
zl_status zl_rmsnorm_backward_f32(const float *input, const float *d_output, const float *gamma,
                                  const float *rstd, float *d_input, float *d_gamma, int64_t M, int64_t N,
                                  zl_stream stream);
/* softmax.cuh:17-18 softmax (row-wise) */
zl_status zl_softmax_f32(const float *input, float *output, int M, int N, zl_stream stream);
/* cross_entropy.cuh:16-21 cross_entropy_backward_kernel: d = (p - onehot)/rows */
zl_status zl_cross_entropy_backward_f32(float *d_logits, const float *softmax_output, const int32_t *targets,
                                        int batch, int num_classes, zl_stream stream);
/* cross_entropy.cpp:23-79 CrossEntropyLoss::forward, on the device (no D2H of the
 * probabilities): *loss_out = mean_r -log(max(p[r,t_r], eps)) over all rows. */
zl_status zl_cross_entropy_forward_f32(const float *softmax_output, const int32_t *targets, int batch,
                                       int num_classes, float eps, float *loss_out, zl_stream stream);
/* embedding.cuh:23-33 cuda_embedding_forward<float,int> (invalid ids / positions leave rows untouched) */
zl_status zl_embedding_forward_f32(const int32_t *input, const float *embedding_table,
                                   const float *pos_encoding_table, float *output, int batch, int seq_len,
                                   int embed_dim, int vocab_size, int max_seq_len, zl_stream stream);
/* embedding.cuh:48-57 cuda_embedding_backward<float,int> (accumulates; skips invalid ids) */
zl_status zl_embedding_backward_f32(const int32_t *input, const float *d_output, float *d_embedding_table,
                                    int batch, int seq_len, int embed_dim, int vocab_size, zl_stream stream);
/* add.cuh:17,31 */
zl_status zl_add_f32(const float *a, const float *b, float *output, int size, zl_stream stream);
zl_status zl_add_inplace_f32(float *a, const float *b, int size, zl_stream stream);
/* relu.cuh:16,31 */
zl_status zl_relu_forward_f32(const float *input, float *output, int size, zl_stream stream);
zl_status zl_relu_backward_f32(const float *input, const float *grad_output, float *grad_input, int size,
                               zl_stream stream);
/* transpose.cuh:17-19 */
zl_status zl_transpose_f32(const float *input, float *output, int rows, int cols, zl_stream stream);
/* adamw.cuh:28-41, adam.cuh:23-35, sgd.cuh:23-31 (sizes as int64 here) */
zl_status zl_adamw_step_f32(float *params, const float *grads, float *m, float *v, int64_t size,
                            float learning_rate, float weight_decay, float beta1, float beta2, float eps,
                            float bias_correction1, float bias_correction2, zl_stream stream);
zl_status zl_adam_step_f32(float *params, const float *grads, float *m, float *v, int64_t size,
                           float learning_rate, float beta1, float beta2, float eps, float bias_correction1,
                           float bias_correction2, zl_stream stream);
zl_status zl_sgd_step_f32(float *params, const float *grads, float *velocity, int64_t size,
                          float learning_rate, float momentum, float weight_decay, zl_stream stream);

/* ===================================================================== */
/* bf16 training-path kernels (no reference counterpart: the fused        */
/* B200 forms of the ops above, used by the model step).                  */
/* ===================================================================== */
/* GEMM epilogue flags */
enum {
  ZL_EPI_BIAS = 1,       /* + bias[n] (fp32) */
  ZL_EPI_RELU = 2,       /* max(0, .) */
  ZL_EPI_RESIDUAL = 4,   /* + residual[m,n] (bf16, same layout as D) */
  ZL_EPI_RELU_MASK = 8,  /* * (aux[m,n] > 0), aux bf16 (ReLU backward) */
  ZL_EPI_ROPE = 16,      /* rotate interleaved pairs of columns [0, rope_cols) (q and k) */
  ZL_EPI_ACCUM = 64,     /* fp32 output: D += result instead of D = result */
  ZL_EPI_OUT_F32 = 128   /* output fp32 instead of bf16 */
};
/* Operand layouts: A_KMAJOR means A is stored [M, K] (K contiguous); otherwise [K, M].
 * B_KMAJOR means B is stored [N, K]; otherwise [K, N].  D is [M, N] row-major. */
enum { ZL_A_KMAJOR = 1, ZL_B_KMAJOR = 2 };
typedef struct {
  const float *bias;        /* [N] */
  const zl_bf16 *residual;  /* [M, N] */
  const zl_bf16 *aux;       /* [M, N] relu mask source */
  const float *rope_cos;    /* [seq, head_dim/2], or [head_dim/2, seq] when rope_pair_major */
  const float *rope_sin;
  int rope_cols;            /* columns [0, rope_cols) are rotated (2*d for q|k of a qkv row) */
  int rope_seq;             /* position of row m is m % rope_seq */
  int head_dim;
  int rope_pair_major;      /* 1: tables stored pair-major, which the epilogue reads with coalesced
                               loads (32 consecutive rows = 32 consecutive positions per load) */
} zl_epilogue;
/* D[M,N] = sum_k A(m,k) B(n,k), bf16 operands, fp32 accumulate in TMEM, fused epilogue.
 * `workspace` (fp32, >= zl_gemm_workspace_floats(...) elements, may be NULL when that is 0)
 * holds split-K partial sums. */
zl_status zl_gemm_bf16(const zl_bf16 *A, const zl_bf16 *B, void *D, int M, int N, int K, int layout,
                       int epi_flags, const zl_epilogue *epi, float *workspace, zl_stream stream);
int64_t zl_gemm_workspace_floats(int M, int N, int K, int layout, int epi_flags);
/* zl_gemm_bf16 for a bf16 output D that also adds D's column sums into colsum (fp32 [N], accumulated
 * with atomics, so the order of the additions is not fixed): a bias gradient computed by the product
 * that produces its input, as the model's FF1 bias gradient from the ReLU-masked dF product.  The
 * reference computes bias gradients with a separate kernel (linear.cu:59-69); this entry has no
 * counterpart there.  The sums are of the bf16-rounded stored values.  When the product does not
 * take the pipelined bf16 epilogue (N not a multiple of 32, A MN-major, split-K), a column-sum pass
 * over D runs after it.  ZL_EINVAL for fp32 outputs. */
zl_status zl_gemm_bf16_colsum(const zl_bf16 *A, const zl_bf16 *B, void *D, int M, int N, int K, int layout,
                              int epi_flags, const zl_epilogue *epi, float *workspace, float *colsum,
                              zl_stream stream);
/* zl_gemm_bf16 with the ReLU mask kept as bits ([M][N/32] uint32 words, bit j of word w of a row =
 * column 32 w + j; N a multiple of 32, bf16 output, A K-major): bits_out (may be NULL) receives
 * (stored output > 0) of every element, as the FF1 product's ReLU output f; bits_in (may be NULL) masks
 * a ZL_EPI_RELU_MASK product in place of epi->aux, so that the ReLU backward reads N/8 bytes per row
 * instead of the 2 N bytes of f.  No counterpart in the reference (relu.cu:14-43 reads the saved
 * input).  ZL_EINVAL for other outputs or shapes; the product runs unsplit. */
zl_status zl_gemm_bf16_relu_bits(const zl_bf16 *A, const zl_bf16 *B, void *D, int M, int N, int K, int layout,
                                 int epi_flags, const zl_epilogue *epi, float *workspace, uint32_t *bits_out,
                                 const uint32_t *bits_in, zl_stream stream);
/* zl_gemm_bf16 whose persistent CTAs draw their work units (output tiles x split-K slices) at run
 * time from `unit_counters` (one int32 in device memory, 4-byte aligned, zero before the first call)
 * instead of taking them round-robin: a CTA that starts late, because another kernel (an all-reduce
 * on a side stream, say) still holds its SM, takes fewer units instead of holding back the end of
 * the product.  The CTA that draws a launch's last value puts the counter back to zero, so
 * consecutive calls in one stream can share it; calls that may run at the same time (other
 * streams) must each have their own.  The result is the one zl_gemm_bf16 gives.  No counterpart in the reference, whose GEMMs
 * launch one thread block per output tile (matmul.cu:227-230, 257-260). */
zl_status zl_gemm_bf16_sched(const zl_bf16 *A, const zl_bf16 *B, void *D, int M, int N, int K, int layout,
                             int epi_flags, const zl_epilogue *epi, float *workspace, int *unit_counters,
                             zl_stream stream);
/* Causal flash attention over a packed qkv buffer [B*S, 3*H*Dh] (q | k | v), output o [B*S, H*Dh],
 * lse [B, H, S] (natural log of the row sums of exp(scale * q.k)). */
zl_status zl_attention_forward_bf16(const zl_bf16 *qkv, zl_bf16 *o, float *lse, int batch, int seq_len,
                                    int num_heads, int head_dim, zl_stream stream);
/* Backward: d_qkv [B*S, 3*H*Dh] receives dq | dk | dv.  `workspace` fp32 of
 * zl_attention_workspace_floats() elements (dq accumulation, row dot products and the counter from
 * which the kernel's CTAs draw work units at run time, so one workspace serves one call in flight at
 * a time); o, d_o and workspace 16-byte aligned.
 * rope_cos/rope_sin ([seq, head_dim/2], may be NULL, 16-byte aligned): dq and dk are rotated
 * back by the inverse of the interleaved-pair RoPE applied to q and k in the forward. */
zl_status zl_attention_backward_bf16(const zl_bf16 *qkv, const zl_bf16 *o, const zl_bf16 *d_o,
                                     const float *lse, zl_bf16 *d_qkv, float *workspace, int batch,
                                     int seq_len, int num_heads, int head_dim, const float *rope_cos,
                                     const float *rope_sin, zl_stream stream);
int64_t zl_attention_workspace_floats(int batch, int seq_len, int num_heads, int head_dim);
/* ===================================================================== */
/* __nv_bfloat16 instances of the reference's kernel templates            */
/* (the reference instantiates them for float only: linear.cu:173,183,     */
/* mha.cu:332,340, layernorm.cu, softmax.cu, add.cu, relu.cu, adamw.cu).   */
/* Storage is bf16, arithmetic fp32; sizes are checked as in the f32 forms. */
/* ===================================================================== */
/* linear.cuh:21-30 in bf16: Y[M,N] = X[M,K] W[N,K]^T (+ b) on the tcgen05 GEMM (no split-K
 * workspace).  K and N multiples of 8, rows 16-byte aligned (ZL_EUNSUPPORTED otherwise). */
zl_status zl_linear_forward_bf16(const zl_bf16 *input, const zl_bf16 *weight, const zl_bf16 *bias,
                                 zl_bf16 *output, int64_t M, int64_t K, int64_t N, int use_bias,
                                 zl_stream stream);
/* linear.cuh:48-59 in bf16: dX = dY W and dW = dY^T X overwrite (tcgen05 GEMM), dB += column sums
 * of dY (fp32 sums, one rounding to bf16).  M, K and N multiples of 8. */
zl_status zl_linear_backward_bf16(const zl_bf16 *d_output, const zl_bf16 *input, const zl_bf16 *weight,
                                  zl_bf16 *d_input, zl_bf16 *d_weight, zl_bf16 *d_bias, int64_t M, int64_t K,
                                  int64_t N, int use_bias, zl_stream stream);
/* mha.cuh:18-24 in bf16, on the tcgen05 flash-attention kernels: Q, K, V, attn_output [B*S, H*Dh]
 * (separate tensors, 16-byte aligned).  Causal, no mask, head_dim 64 or 128, seq_len a multiple of
 * 128 (ZL_EUNSUPPORTED otherwise).  The probability matrix is never formed: `state` (the reference
 * API's attention_scores buffer, state_bytes long, 256-byte aligned) receives what the backward needs
 * instead -- the per-row log-sum-exp and a copy of attn_output -- and the backward uses the rest of
 * it as scratch; zl_mha_state_bytes_bf16() bytes are needed (ZL_EINVAL with the count otherwise).
 * B*H*S*S bf16 elements are enough when seq_len >= 3 * head_dim + 6. */
zl_status zl_mha_forward_bf16(const zl_bf16 *Q, const zl_bf16 *K, const zl_bf16 *V, zl_bf16 *attn_output,
                              void *state, size_t state_bytes, const uint8_t *mask, int64_t batch,
                              int64_t seq_len, int64_t num_heads, int64_t head_dim, int is_causal,
                              zl_stream stream);
/* mha.cuh:38-48 in bf16: d_Q, d_K, d_V from d_attn_output and the forward's `state`.
 * reference_semantics = 1 leaves out the 1/sqrt(head_dim) factor of dQ and dK as mha.cu:284-295
 * does; 0 gives the true gradient. */
zl_status zl_mha_backward_bf16(const zl_bf16 *d_attn_output, const zl_bf16 *Q, const zl_bf16 *K,
                               const zl_bf16 *V, void *state, size_t state_bytes, const uint8_t *mask,
                               zl_bf16 *d_Q, zl_bf16 *d_K, zl_bf16 *d_V, int64_t batch, int64_t seq_len,
                               int64_t num_heads, int64_t head_dim, int is_causal, int reference_semantics,
                               zl_stream stream);
size_t zl_mha_state_bytes_bf16(int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim);
/* layernorm.cuh:22-61 in bf16 (gamma, beta, mean, rstd bf16; d_gamma / d_beta accumulate) */
zl_status zl_layernorm_forward_bf16(const zl_bf16 *input, const zl_bf16 *gamma, const zl_bf16 *beta,
                                    zl_bf16 *output, zl_bf16 *mean, zl_bf16 *rstd, int64_t M, int64_t N,
                                    float eps, zl_stream stream);
zl_status zl_layernorm_backward_bf16(const zl_bf16 *input, const zl_bf16 *d_output, const zl_bf16 *gamma,
                                     const zl_bf16 *mean, const zl_bf16 *rstd, zl_bf16 *d_input,
                                     zl_bf16 *d_gamma, zl_bf16 *d_beta, int64_t M, int64_t N, zl_stream stream);
/* softmax.cuh:17-18, add.cuh:17-31, relu.cuh:16-31, adamw.cuh:28-41 in bf16 */
zl_status zl_softmax_bf16(const zl_bf16 *input, zl_bf16 *output, int M, int N, zl_stream stream);
zl_status zl_add_bf16(const zl_bf16 *a, const zl_bf16 *b, zl_bf16 *output, int size, zl_stream stream);
zl_status zl_add_inplace_bf16(zl_bf16 *a, const zl_bf16 *b, int size, zl_stream stream);
zl_status zl_relu_forward_bf16(const zl_bf16 *input, zl_bf16 *output, int size, zl_stream stream);
zl_status zl_relu_backward_bf16(const zl_bf16 *input, const zl_bf16 *grad_output, zl_bf16 *grad_input, int size,
                                zl_stream stream);
zl_status zl_adamw_step_bf16(zl_bf16 *params, const zl_bf16 *grads, zl_bf16 *m, zl_bf16 *v, int64_t size,
                             float learning_rate, float weight_decay, float beta1, float beta2, float eps,
                             float bias_correction1, float bias_correction2, zl_stream stream);

/* Norms on bf16 rows with fp32 statistics.  kind: 0 LayerNorm (mean/rstd), 1 RMSNorm (rstd only).
 * x and y must be 16-byte aligned (ZL_EINVAL otherwise). */
zl_status zl_norm_forward_bf16(int kind, const zl_bf16 *x, const float *gamma, const float *beta, zl_bf16 *y,
                               float *mean, float *rstd, int64_t M, int N, float eps, zl_stream stream);
/* dx = norm backward (bf16) of the full upstream gradient dy; dgamma/dbeta accumulated (fp32).
 * `workspace` fp32 >= 2*N*zl_norm_bwd_blocks(M). */
zl_status zl_norm_backward_bf16(int kind, const zl_bf16 *x, const zl_bf16 *dy, const float *gamma,
                                const float *mean, const float *rstd, zl_bf16 *dx, float *dgamma,
                                float *dbeta, float *workspace, int64_t M, int N, zl_stream stream);
int zl_norm_bwd_blocks(int64_t M);
/* Token embedding for the model: x[t] = bf16(table[id] (+ pos[t % S])); invalid ids give a zero row.
 * table, pos and out must be 16-byte aligned (ZL_EINVAL otherwise). */
zl_status zl_embedding_forward_bf16(const int32_t *ids, const float *table, const float *pos, zl_bf16 *out,
                                    int64_t T, int seq_len, int dim, int vocab, zl_stream stream);
/* dtable[id] += dx[t] (fp32 atomics; invalid ids skipped); dx and dtable 16-byte aligned. */
zl_status zl_embedding_backward_bf16(const int32_t *ids, const zl_bf16 *dx, float *dtable, int64_t T, int dim,
                                     int vocab, zl_stream stream);
/* Fused cross-entropy on bf16 logits [rows, V]: loss_rows[r] = min(lse - x_t, -log(eps)) (0 for invalid
 * targets), d_logits = (softmax - onehot) * grad_scale written over `logits` in place (bf16).
 * *loss_out = sum(loss_rows) / rows (deterministic two-stage reduction). */
zl_status zl_cross_entropy_fused_bf16(zl_bf16 *logits, const int32_t *targets, int rows, int vocab,
                                      float eps, float grad_scale, float *loss_rows, float *loss_out,
                                      zl_stream stream);
/* Column sums of a bf16 [M, N] matrix accumulated into db (fp32): bias gradients.  N a multiple of 8
 * (ZL_EUNSUPPORTED otherwise); dy 16-byte aligned (ZL_EINVAL otherwise). */
zl_status zl_colsum_bf16(const zl_bf16 *dy, float *db, float *workspace, int64_t M, int N, zl_stream stream);
int64_t zl_colsum_workspace_floats(int64_t M, int N);
/* zl_colsum_bf16 without a workspace argument (no counterpart in the reference, whose bias
 * gradients come from its own kernels).  It is for callers that cannot hand over device
 * memory: code that must not call cudaMalloc/cudaFree because they can synchronise the whole
 * device and stall work on other streams, and plugins whose host framework owns every device
 * allocation.  The partial sums go to a fixed 4 MiB device array inside the library
 * (zl_colsum_noalloc_max_floats() floats); the call allocates nothing.  Sizes whose
 * zl_colsum_workspace_floats(M, N) exceeds that maximum return ZL_EINVAL with a message
 * (e.g. M <= 32768 fits at N = 2048; at N <= 880 every M fits).  N must be a multiple of 8
 * (ZL_EUNSUPPORTED otherwise), like zl_colsum_bf16.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) and keeps it for the life of the process;
 * make that first call before any stream capture.  A device reset (cudaDeviceReset) after the
 * first call is not supported: the kept address would no longer name the array.  Calls on one
 * device share the array: calls that overlap on the GPU (two streams, or two host threads)
 * race and give wrong sums, so order them on one stream. */
zl_status zl_colsum_bf16_noalloc(const zl_bf16 *dy, float *db, int64_t M, int N, zl_stream stream);
int64_t zl_colsum_noalloc_max_floats(void);
/* Flat AdamW over the whole parameter arena (adamw.cu:26-73 per element) with the gradient
 * multiplied by grad_scale (1/world for data parallelism), writing a bf16 shadow of the
 * updated parameters (may be NULL). */
zl_status zl_adamw_flat(float *params, const float *grads, float *m, float *v, zl_bf16 *params_bf16,
                        int64_t n, float lr, float weight_decay, float beta1, float beta2, float eps,
                        float bias_correction1, float bias_correction2, float grad_scale, zl_stream stream);
/* fp32 -> bf16 conversion (parameter shadow refresh). */
zl_status zl_f32_to_bf16(const float *x, zl_bf16 *y, int64_t n, zl_stream stream);

/* ===================================================================== */
/* Model: Layer -> Model -> Loss -> Optimizer API on one arena            */
/* (src/model/zerollm.hpp:51-130, src/layer/*, src/loss/cross_entropy.cpp, */
/* src/optimizer/adamw.cpp, src/distributed/abstract_backend.hpp:13-27)    */
/* ===================================================================== */
typedef struct {
  int vocab_size, embed_dim, num_layers, num_heads, ff_hidden_dim, max_seq_len; /* zerollm_config.hpp:10-17 */
  int norm;        /* 0 LayerNorm (reference), 1 RMSNorm */
  int pos;         /* 0 sinusoid absolute (reference embedding.cpp:107-126), 1 RoPE */
  int tied;        /* 1 = head tied to the token embedding (reference zerollm.cpp:150-178) */
  int bias;        /* 1 = biases on every Linear (reference) */
  float eps;       /* norm epsilon (reference 1e-5) */
  float rope_base; /* 10000 */
} zl_model_config;

typedef struct {
  float beta1, beta2, eps, weight_decay; /* optimizer.hpp:51-117 createAdamW */
} zl_adamw_config;

typedef struct zl_model zl_model;

/* Creates the model on the current device with an arena sized for batch*seq <= max_tokens.
 * Weights: N(0, init_std) from `seed` for matrices and the embedding, zero biases/betas,
 * unit gammas, in the canonical layout (zl_model_param_layout). */
zl_status zl_model_create(const zl_model_config *cfg, int64_t max_tokens, uint64_t seed, float init_std,
                          zl_model **out);
zl_status zl_model_destroy(zl_model *m);
/* Canonical parameter layout (reverse forward order); returns the tensor count in *count. */
zl_status zl_model_param_layout(const zl_model_config *cfg, int64_t *offsets, int64_t *sizes, int *kinds,
                                int max_n, int *count, int64_t *total);
zl_status zl_model_num_params(zl_model *m, int64_t *n);
/* Device pointers of the flat arenas (fp32 params, fp32 grads, AdamW m, v). */
zl_status zl_model_buffers(zl_model *m, float **params, float **grads, float **adam_m, float **adam_v);
/* After the caller writes params directly: refresh the bf16 shadow. */
zl_status zl_model_params_updated(zl_model *m, zl_stream stream);
/* Checkpoints in the reference's directory layout (src/utils/serializer.hpp:24-56,
 * src/model/zerollm.cpp:334-425 and the layers' save/load, e.g. src/layer/linear.cpp:215-250):
 *   dir/config.bin   the reference's ZeroLLMConfig (six int32, bool with_grad, three zero bytes)
 *   dir/embedding/weights/table.bin
 *   dir/decoder/layer_<i>/self_attn/{q,k,v,out}_proj/weights/{weight,bias}.bin
 *   dir/decoder/layer_<i>/{ln1,ln2}/weights/{gamma,beta}.bin
 *   dir/decoder/layer_<i>/ff/{ff1,ff2}/weights/{weight,bias}.bin
 *   dir/output_ln/weights/{gamma,beta}.bin
 * each a raw fp32 array (Linear weights [out, in] row-major).  Topologies the reference does not
 * have add: RMSNorm writes gamma.bin only, an untied head writes head/weights/weight.bin, a model
 * without biases writes no bias.bin, and dir/zerollm_b200.txt records norm / pos / tied / bias.
 * with_optimizer also writes optimizer/adamw_m.bin and optimizer/adamw_v.bin (the flat parameter
 * arena order of zl_model_param_layout) and optimizer/state.bin (int32 step count); the reference
 * saves no optimizer state.  Load checks config.bin (embed_dim, num_layers and vocab_size must
 * match, as the reference does) and every file's size, then refreshes the bf16 shadow. */
zl_status zl_model_save(zl_model *m, const char *dir, int with_optimizer);
zl_status zl_model_load(zl_model *m, const char *dir, int with_optimizer);
/* The tensor files of a configuration's checkpoint, one line per file:
 * "<relative path> <arena offset> <float count>\n", into buf (NUL-terminated when it fits);
 * *len receives the bytes needed (excluding the NUL). */
zl_status zl_checkpoint_manifest(const zl_model_config *cfg, char *buf, int64_t cap, int64_t *len);
zl_status zl_model_set_optimizer(zl_model *m, const zl_adamw_config *opt);
/* One training step: zero_grad -> forward -> fused CE -> backward -> [bucketed all-reduce] -> AdamW.
 * ids/targets are device int32 [batch*seq]; *loss_out (device fp32) receives the mean loss of this
 * rank's batch.  update=0 skips AdamW (gradients stay in the grad arena). */
zl_status zl_model_train_step(zl_model *m, const int32_t *ids, const int32_t *targets, int batch, int seq_len,
                              float lr, int update, float *loss_out, zl_stream stream);
/* Step as a CUDA graph (default on, single process): the second call with the same ids/targets/loss
 * pointers and shape captures zero_grad -> forward -> CE -> backward into a graph that later calls replay
 * (AdamW stays a separate launch so lr may change).  0 disables. */
zl_status zl_model_set_graph(zl_model *m, int enabled);
/* In-step kernel timing (no reference counterpart; a measurement aid).  When enabled, the step
 * records timing events just before and after each layer's attention forward kernel and the
 * attention backward's main kernel (event nodes of the captured step graph).
 * zl_model_kernel_times returns their mean duration per launch over the layers, in ms, for the most
 * recent step (it waits for that step's events); ZL_ESTATE when timing is off or no step ran. */
zl_status zl_model_set_kernel_timing(zl_model *m, int enabled);
zl_status zl_model_kernel_times(zl_model *m, float *attn_fwd_ms, float *attn_bwd_ms);
/* With kernel timing on: the latest step's duration (zero_grad to the end of the step, AdamW not
 * included) and the part of it after the last backward kernel, i.e. the time the step waited for the
 * gradient all-reduces still running on the side stream (0 without a communicator).  No reference
 * counterpart (a measurement aid). */
zl_status zl_model_step_times(zl_model *model, float *step_ms, float *exposed_exchange_ms);
/* Reference-API pieces: forward to fp32 logits [batch*seq, V] (zerollm.cpp:101-195) ... */
zl_status zl_model_forward(zl_model *m, const int32_t *ids, int batch, int seq_len, float *logits,
                           zl_stream stream);
/* ... and backward from fp32 d_logits (zerollm.cpp:197-323); gradients accumulate into the arena. */
zl_status zl_model_backward(zl_model *m, const int32_t *ids, const float *d_logits, int batch, int seq_len,
                            zl_stream stream);
zl_status zl_model_zero_grad(zl_model *m, zl_stream stream);
/* AdamW over every parameter (zerollm.cpp:450-463 -> adamw.cpp:12-53 per tensor). */
zl_status zl_model_step(zl_model *m, float lr, zl_stream stream);
/* Number of kernels the last train step launched (for accounting). */
zl_status zl_model_last_launches(zl_model *m, int *count);

/* ---- data parallelism over NCCL (gpu_backend.cpp:66-124, train_zerollm_dp.cpp:335-420) ---- */
/* 128-byte NCCL unique id, created on rank 0 and shared by the caller (any host transport). */
zl_status zl_nccl_unique_id(void *id_out, size_t id_bytes);
/* Creates the communicator and the bucket plan (bucket_bytes of fp32 gradients per all-reduce).
 * Parameters are broadcast from rank 0.  After this, zl_model_train_step all-reduces gradient
 * buckets on a side stream as soon as their last producer finishes and folds 1/world into AdamW. */
zl_status zl_model_attach_nccl(zl_model *m, const void *id, int rank, int world, int64_t bucket_bytes);
/* Bucket plan (host-side, no GPU needed): splits [0,total) floats at tensor boundaries into buckets
 * of at most bucket_floats (a tensor larger than a bucket is split); returns bucket starts.  The
 * buckets are formed from the end of the arena, where backward finishes, and taper there: the last
 * holds at most bucket_floats / 8, the one before it twice that, and so on up to bucket_floats (a
 * single tensor larger than its share gets a bucket of its own), so that little is left to
 * all-reduce after the step's last gradient is written. */
zl_status zl_bucket_plan(const int64_t *tensor_offsets, const int64_t *tensor_sizes, int n_tensors,
                         int64_t bucket_floats, int64_t *starts, int64_t *lens, int max_buckets,
                         int *n_buckets);
/* ---- communicator behind the reference's distributed backend (abstract_backend.hpp:13-27,
 *      gpu_backend.cpp:66-130), MPI-free.  dtype follows dist_types.hpp DataType order
 *      (0 f32, 1 f16, 2 bf16, 3 i32, 4 i64); op follows ReduceOp (0 sum, 1 prod, 2 min, 3 max, 4 avg). */
/* ===================================================================== */
/* Token data pipeline: LLMDataLoader (src/runtime/dataloader.cpp:35-149) */
/* ===================================================================== */
/* Stories are one int32 token array with offsets: story i = tokens[offsets[i], offsets[i+1]).
 * Samples: for every non-empty story, start positions 0, S, 2S, ... below len + 1
 * (dataloader.cpp:57-66).  token(story, p) = story[p] for p < len, eos_id at p == len, pad_id after
 * (:109-119); a sample's inputs are tokens [start, start + S) and its targets [start + 1, start + S + 1)
 * (:138-142).  shuffle != 0 reorders the samples with a generator seeded by `seed`, again at every
 * reset (the reference seeds it from std::random_device); 0 keeps story order.  The loader keeps its
 * own copy of the tokens. */
typedef struct zl_loader zl_loader;
zl_status zl_loader_create(const int32_t *tokens, const int64_t *offsets, int64_t n_stories, int batch, int seq_len,
                           int32_t eos_id, int32_t pad_id, int shuffle, uint64_t seed, zl_loader **out);
zl_status zl_loader_destroy(zl_loader *l);
/* New epoch: stops the device feed, rewinds, reshuffles (dataloader.cpp:17-21). */
zl_status zl_loader_reset(zl_loader *l);
zl_status zl_loader_info(zl_loader *l, int64_t *samples, int64_t *batches);
/* Next batch into host buffers of batch * seq_len int32 each; *count = samples in it (the last batch
 * of an epoch may be short, 0 once the epoch is over). */
zl_status zl_loader_next(zl_loader *l, int32_t *ids, int32_t *targets, int *count);
/* Device feed: a host thread assembles the following batches into `depth` pinned buffers;
 * zl_loader_next_device enqueues the copy of the next one into device ids / targets on `stream`
 * (count as above) and recycles the pinned buffer once that copy has completed. */
zl_status zl_loader_start(zl_loader *l, int depth);
zl_status zl_loader_next_device(zl_loader *l, int32_t *d_ids, int32_t *d_targets, int *count, zl_stream stream);

typedef struct zl_comm zl_comm;
/* Non-blocking NCCL init from a 128-byte id with a host deadline (ZL_ETIMEOUT, communicator aborted). */
zl_status zl_comm_create(const void *id, int rank, int world, double timeout_s, zl_comm **out);
/* Rank 0 writes a fresh id to `path`; the other ranks wait for it (bounded by timeout_s). */
zl_status zl_comm_create_from_file(const char *path, int rank, int world, double timeout_s, zl_comm **out);
zl_status zl_comm_destroy(zl_comm *c);
zl_status zl_comm_all_reduce(zl_comm *c, void *buffer, size_t count, int dtype, int op, zl_stream stream);
zl_status zl_comm_broadcast(zl_comm *c, void *buffer, size_t count, int dtype, int root, zl_stream stream);
zl_status zl_comm_all_gather(zl_comm *c, const void *sendbuf, void *recvbuf, size_t count, int dtype,
                             zl_stream stream);
/* Bounded wait for the stream's collectives; on an NCCL error or a timeout the communicator is
 * aborted and ZL_ENCCL / ZL_ETIMEOUT returned, so a lost peer cannot hang the caller. */
zl_status zl_comm_check(zl_comm *c, zl_stream stream, double timeout_s);
zl_status zl_comm_rank(zl_comm *c, int *rank, int *world);
/* 64-bit checksum of the fp32 parameter arena (bit pattern), for cross-rank equality checks. */
zl_status zl_model_param_checksum(zl_model *m, uint64_t *out, zl_stream stream);

#ifdef __cplusplus
}
#endif
#endif
