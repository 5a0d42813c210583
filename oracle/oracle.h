/*
 * oracle.h -- CPU restatement of ZeroLLM's training-step arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: the tests, the
 * smoke entry point and the CPU-baseline leg of bench.py call it to produce
 * expected values.  Nothing in the product (zerollm_b200/) links, loads or
 * calls it.
 *
 * Every kernel-level function restates one reference CUDA kernel of
 * buladuo/ZeroLLM (paths relative to the reference project root) with the
 * same per-element fp32 accumulation order, so that results can be compared
 * against the reference's own kernels.  Functions without a reference
 * counterpart (RMSNorm, RoPE, fused cross-entropy, the whole-step model in
 * the BASELINE topology) restate the standard published definitions; their
 * conventions are written next to each declaration.
 */
#ifndef ZEROLLM_ORACLE_H
#define ZEROLLM_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- seeded inputs ---------------------------------------- */
/* splitmix64 stream; uniform ids by rejection; normals by Box-Muller on
 * 53-bit uniforms computed in double and rounded to float. */
uint64_t orc_splitmix64(uint64_t *state);
void orc_fill_normal(float *out, int64_t n, uint64_t seed, float mean, float std);
void orc_fill_uniform_ids(int32_t *out, int64_t n, uint64_t seed, int32_t vocab);

/* ---------------- reference kernels (src/kernel/cuda) ------------------- */
/* matmul.cu:51-96  C[M,N] = A[M,K] B[K,N]; k ascending, one fp32 accumulator */
void orc_matmul(const float *A, const float *B, float *C, int M, int N, int K);
/* matmul.cu:150-218  C[K,N] = A[M,K]^T B[M,N]; reduction over M ascending; overwrites C */
void orc_matmul_at_b(const float *A, const float *B, float *C, int M, int N, int K);
/* matmul.cu:100-146  C[M,N] = A[M,K] B[N,K]^T */
void orc_matmul_a_bt(const float *A, const float *B, float *C, int M, int N, int K);
/* linear.cu:72-95 */
void orc_linear_forward(const float *in, const float *W, const float *b, float *out,
                        int64_t M, int64_t K, int64_t N, int use_bias);
/* linear.cu:98-170: dX, dW overwritten; dB accumulated */
void orc_linear_backward(const float *dY, const float *X, const float *W, float *dX,
                         float *dW, float *dB, int64_t M, int64_t K, int64_t N, int use_bias);
/* mha.cu:18-122.  scores [B,H,S,S] receives the probabilities. */
void orc_mha_forward(const float *Q, const float *K, const float *V, float *out,
                     float *scores, const uint8_t *mask, int64_t B, int64_t S,
                     int64_t H, int64_t Dh, int causal);
/* mha.cu:164-299.  apply_scale=0 reproduces the reference exactly (dQ, dK
 * without the 1/sqrt(Dh) factor); apply_scale=1 is the mathematically
 * correct gradient. */
void orc_mha_backward(const float *dO, const float *Q, const float *K, const float *V,
                      const float *P, const uint8_t *mask, float *dQ, float *dK, float *dV,
                      int64_t B, int64_t S, int64_t H, int64_t Dh, int causal,
                      int apply_scale);
/* layernorm.cu:6-76 (biased variance, 1/sqrt) */
void orc_layernorm_forward(const float *x, const float *g, const float *b, float *y,
                           float *mean, float *rstd, int64_t M, int64_t N, float eps);
/* layernorm.cu:79-165 (d_gamma, d_beta accumulated) */
void orc_layernorm_backward(const float *x, const float *dy, const float *g,
                            const float *mean, const float *rstd, float *dx,
                            float *dg, float *db, int64_t M, int64_t N);
/* softmax.cu:12-65 */
void orc_softmax(const float *in, float *out, int M, int N);
/* cross_entropy.cpp:23-79: mean over ALL rows of -log(max(p[t], eps));
 * rows with an invalid target add 0 but still count. */
float orc_ce_forward(const float *probs, const int32_t *targets, int rows, int classes, float eps);
/* cross_entropy.cu:5-31 */
void orc_ce_backward(float *dlogits, const float *probs, const int32_t *targets, int rows, int classes);
/* embedding.cu:6-30 (skips rows with s>=max_seq_len or id outside [0,V)) */
void orc_embedding_forward(const int32_t *ids, const float *table, const float *pos,
                           float *out, int B, int S, int D, int V, int max_seq_len);
/* embedding.cu:33-53 (accumulates, skips invalid ids) */
void orc_embedding_backward(const int32_t *ids, const float *dout, float *dtable,
                            int B, int S, int D, int V);
/* add.cu, relu.cu, transpose.cu */
void orc_add(const float *a, const float *b, float *out, int64_t n);
void orc_add_inplace(float *a, const float *b, int64_t n);
void orc_relu_forward(const float *x, float *y, int64_t n);
void orc_relu_backward(const float *x, const float *gy, float *gx, int64_t n);
void orc_transpose(const float *in, float *out, int rows, int cols);
/* adamw.cu:9-75, adam.cu:13-57, sgd.cu:14-57 */
void orc_adamw(float *p, const float *g, float *m, float *v, int64_t n, float lr, float wd,
               float b1, float b2, float eps, float bc1, float bc2);
void orc_adam(float *p, const float *g, float *m, float *v, int64_t n, float lr,
              float b1, float b2, float eps, float bc1, float bc2);
void orc_sgd(float *p, const float *g, float *vel, int64_t n, float lr, float momentum, float wd);

/* sinusoid table of embedding.cpp:107-126 (PE(pos,2i)=sin, PE(pos,2i+1)=cos) */
void orc_sinusoid_table(float *out, int max_seq_len, int D);

/* ---------------- definitions with no reference kernel ------------------ */
/* RMSNorm: rstd = 1/sqrt(mean(x^2)+eps), y = x*rstd*g.  bwd accumulates dg. */
void orc_rmsnorm_forward(const float *x, const float *g, float *y, float *rstd,
                         int64_t M, int64_t N, float eps);
void orc_rmsnorm_backward(const float *x, const float *dy, const float *g, const float *rstd,
                          float *dx, float *dg, int64_t M, int64_t N);
/* RoPE table: cos/sin [S, Dh/2], theta_i = pos * base^(-2i/Dh), computed in
 * double and rounded to float. */
void orc_rope_table(float *cos_t, float *sin_t, int S, int Dh, double base);
/* Interleaved-pair rotation of x [T, H*Dh] (row t has position t % S), in
 * place.  inverse=1 applies the transpose rotation (used for gradients). */
void orc_rope_apply(float *x, int64_t T, int S, int H, int Dh, int row_stride,
                    const float *cos_t, const float *sin_t, int inverse);
/* Causal attention with the 1/sqrt(Dh) scale, q/k/v rows of stride ld
 * (head h at column h*Dh).  lse [B,H,S] = row log-sum-exp of scaled scores. */
void orc_attention_forward(const float *q, const float *k, const float *v, int ld,
                           float *o, int ldo, float *lse, int B, int S, int H, int Dh);
void orc_attention_backward(const float *q, const float *k, const float *v, int ld,
                            const float *o, const float *dO, int ldo, const float *lse,
                            float *dq, float *dk, float *dv, int ldd,
                            int B, int S, int H, int Dh);
/* Fused cross-entropy from logits: per-row loss = min(lse - x_t, -log(eps))
 * (the reference's probability clamp), mean over all rows; dlogits =
 * (softmax - onehot)/rows.  Returns the loss. */
float orc_ce_fused(const float *logits, const int32_t *targets, float *dlogits,
                   int rows, int classes, float eps);

/* ---------------- whole training step ----------------------------------- */
/* bf16 storage emulation (see oracle.c): 1 rounds every tensor the B200 path
 * stores in bf16 at the same point of the step; 0 (default) is plain fp32. */
void orc_set_bf16_emulation(int on);
typedef struct {
    int vocab, dim, layers, heads, ffn, max_seq;
    int norm;      /* 0 = LayerNorm (reference), 1 = RMSNorm */
    int pos;       /* 0 = sinusoid absolute (reference), 1 = RoPE */
    int tied;      /* 1 = output head tied to the token embedding */
    int bias;      /* 1 = biases on every Linear */
    float eps;     /* norm epsilon */
    float rope_base;
} orc_model_cfg;

/* Canonical flat parameter layout, identical to the product's arena.
 * Tensors are listed in REVERSE forward order (the order backward finishes
 * them): head (untied only), norm_out, layers L-1..0 each as
 * [norm2.g, norm2.b?, w2, b2?, w1, b1?, norm1.g, norm1.b?, wo, bo?, wqkv, bqkv?],
 * then tok_emb.  Fills up to max_n offsets/sizes; returns the tensor count
 * and writes the total element count. */
/* OpenMP team size for later calls (n <= 0: query only); returns the size in force. */
int orc_set_threads(int n);
int orc_param_layout(const orc_model_cfg *cfg, int64_t *offsets, int64_t *sizes,
                     int *kinds, int max_n, int64_t *total);
/* N(0, init_std) for matrices and the embedding (tensor i seeded with
 * seed ^ (0xD1B54A32D192ED03 * (i+1)) where i is the index in the layout
 * above), 0 for biases/betas, 1 for gammas. */
void orc_init_params(const orc_model_cfg *cfg, float *params, uint64_t seed, float init_std);

typedef struct {
    float lr, beta1, beta2, eps, weight_decay;
    int step;          /* 1-based AdamW step t (bias corrections use powf) */
    float grad_scale;  /* multiplies every gradient inside AdamW (1/world for DP) */
} orc_adamw_cfg;

/* One fp32 training step: forward, fused CE loss, backward, AdamW.
 * grads (same layout as params) is overwritten with the gradients of this
 * batch.  When opt is NULL the parameters are not updated.  m, v hold the
 * AdamW moments (zero before step 1).  Returns the loss.
 * If logits_out is non-NULL it receives the [B*S, V] logits. */
float orc_train_step(const orc_model_cfg *cfg, float *params, float *grads, float *m, float *v,
                     const int32_t *ids, const int32_t *targets, int B, int S,
                     const orc_adamw_cfg *opt, float *logits_out);

#ifdef __cplusplus
}
#endif
#endif
