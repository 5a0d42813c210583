/*
 * oracle.c -- CPU restatement of ZeroLLM's training-step arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  Only tests/, the smoke entry point
 * and bench.py's CPU-baseline leg load this library; the product never does.
 *
 * Kernel-level functions follow the reference CUDA kernels of
 * buladuo/ZeroLLM line by line (file:line cited per function) and keep their
 * per-element fp32 accumulation order.  Parallelism (OpenMP) is only ever
 * across independent outputs, so results do not depend on the thread count.
 */
#include "oracle.h"
#include <math.h>
#include <float.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define MIN(a, b) ((a) < (b) ? (a) : (b))

/* bf16 storage emulation for the whole-step oracle: when on, every tensor the
 * B200 path stores in bf16 (weights used by GEMMs, forward activations, the
 * logits and backward activation gradients) is rounded to bf16 (round to
 * nearest even) at the same point, and the attention forward follows the
 * blockwise online-softmax order with bf16 probabilities.  Arithmetic stays
 * fp32.  Off by default (plain fp32 reference semantics). */
static int g_bf16 = 0;
void orc_set_bf16_emulation(int on) { g_bf16 = on; }

/* OpenMP team size for every later parallel region of this library (callers set it explicitly:
 * a launcher such as torchrun exports OMP_NUM_THREADS=1 to each rank).  Returns the size now in
 * force; n <= 0 only queries it. */
int orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

static inline float bf16r(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return x; /* inf / nan */
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float y;
    memcpy(&y, &u, 4);
    return y;
}
static void round_bf16(float *x, int64_t n) {
    if (!g_bf16) return;
#pragma omp parallel for
    for (int64_t i = 0; i < n; ++i) x[i] = bf16r(x[i]);
}

/* ======================================================================= */
/* seeded inputs                                                            */
/* ======================================================================= */
uint64_t orc_splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void orc_fill_normal(float *out, int64_t n, uint64_t seed, float mean, float std) {
    uint64_t s = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = 0; i < n; i += 2) {
        double u1 = ((double)(orc_splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(orc_splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        out[i] = (float)(mean + std * r * cos(two_pi * u2));
        if (i + 1 < n) out[i + 1] = (float)(mean + std * r * sin(two_pi * u2));
    }
}

void orc_fill_uniform_ids(int32_t *out, int64_t n, uint64_t seed, int32_t vocab) {
    uint64_t s = seed;
    uint64_t V = (uint64_t)vocab;
    uint64_t limit = UINT64_MAX - (UINT64_MAX % V) ; /* accept x < limit */
    for (int64_t i = 0; i < n; ++i) {
        uint64_t x;
        do { x = orc_splitmix64(&s); } while (x >= limit);
        out[i] = (int32_t)(x % V);
    }
}

/* ======================================================================= */
/* GEMM helpers: every output element accumulates its reduction index in   */
/* ascending order with one fp32 accumulator and fused multiply-add, the   */
/* order of the reference's SIMT kernels (matmul.cu:85-87, :135-137,       */
/* :208-210).  Vectorisation is across independent outputs only.          */
/* ======================================================================= */
#define BI 16
#define BJ 128

/* C[M,N] = A[M,K] * B[K,N] */
static void gemm_nn(const float *A, int64_t lda, const float *B, int64_t ldb,
                    float *C, int64_t ldc, int64_t M, int64_t N, int64_t K) {
    int64_t nbi = (M + BI - 1) / BI, nbj = (N + BJ - 1) / BJ;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t blk = 0; blk < nbi * nbj; ++blk) {
        int64_t i0 = (blk / nbj) * BI, j0 = (blk % nbj) * BJ;
        int ni = (int)MIN(BI, M - i0), nj = (int)MIN(BJ, N - j0);
        float acc[BI][BJ];
        for (int ii = 0; ii < BI; ++ii)
            for (int jj = 0; jj < BJ; ++jj) acc[ii][jj] = 0.f;
        for (int64_t k = 0; k < K; ++k) {
            const float *brow = B + k * ldb + j0;
            for (int ii = 0; ii < ni; ++ii) {
                float a = A[(i0 + ii) * lda + k];
#pragma omp simd
                for (int jj = 0; jj < nj; ++jj) acc[ii][jj] = fmaf(a, brow[jj], acc[ii][jj]);
            }
        }
        for (int ii = 0; ii < ni; ++ii)
            memcpy(C + (i0 + ii) * ldc + j0, acc[ii], (size_t)nj * sizeof(float));
    }
}

/* C[Kc,N] = A[M,Kc]^T * B[M,N]  (reduction over M) */
static void gemm_tn(const float *A, int64_t lda, const float *B, int64_t ldb,
                    float *C, int64_t ldc, int64_t M, int64_t N, int64_t Kc) {
    int64_t nbi = (Kc + BI - 1) / BI, nbj = (N + BJ - 1) / BJ;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t blk = 0; blk < nbi * nbj; ++blk) {
        int64_t k0 = (blk / nbj) * BI, j0 = (blk % nbj) * BJ;
        int nk = (int)MIN(BI, Kc - k0), nj = (int)MIN(BJ, N - j0);
        float acc[BI][BJ];
        for (int ii = 0; ii < BI; ++ii)
            for (int jj = 0; jj < BJ; ++jj) acc[ii][jj] = 0.f;
        for (int64_t m = 0; m < M; ++m) {
            const float *brow = B + m * ldb + j0;
            const float *arow = A + m * lda + k0;
            for (int kk = 0; kk < nk; ++kk) {
                float a = arow[kk];
#pragma omp simd
                for (int jj = 0; jj < nj; ++jj) acc[kk][jj] = fmaf(a, brow[jj], acc[kk][jj]);
            }
        }
        for (int kk = 0; kk < nk; ++kk)
            memcpy(C + (k0 + kk) * ldc + j0, acc[kk], (size_t)nj * sizeof(float));
    }
}

/* C[M,N] = A[M,K] * B[N,K]^T  (B transposed into a scratch copy first) */
static void gemm_nt(const float *A, int64_t lda, const float *B, int64_t ldb,
                    float *C, int64_t ldc, int64_t M, int64_t N, int64_t K) {
    float *Bt = (float *)malloc((size_t)K * N * sizeof(float));
#pragma omp parallel for
    for (int64_t k = 0; k < K; ++k)
        for (int64_t n = 0; n < N; ++n) Bt[k * N + n] = B[n * ldb + k];
    gemm_nn(A, lda, Bt, N, C, ldc, M, N, K);
    free(Bt);
}

/* ======================================================================= */
/* reference kernels                                                        */
/* ======================================================================= */
void orc_matmul(const float *A, const float *B, float *C, int M, int N, int K) {
    gemm_nn(A, K, B, N, C, N, M, N, K); /* matmul.cu:51-96 */
}
void orc_matmul_at_b(const float *A, const float *B, float *C, int M, int N, int K) {
    gemm_tn(A, K, B, N, C, N, M, N, K); /* matmul.cu:150-218 */
}
void orc_matmul_a_bt(const float *A, const float *B, float *C, int M, int N, int K) {
    gemm_nt(A, K, B, K, C, N, M, N, K); /* matmul.cu:100-146 */
}

/* linear.cu:72-95: GEMM, then add_bias_kernel (linear.cu:18-27) */
void orc_linear_forward(const float *in, const float *W, const float *b, float *out,
                        int64_t M, int64_t K, int64_t N, int use_bias) {
    gemm_nt(in, K, W, K, out, N, M, N, K);
    if (use_bias && b) {
#pragma omp parallel for
        for (int64_t i = 0; i < M; ++i)
            for (int64_t n = 0; n < N; ++n) out[i * N + n] += b[n];
    }
}

/* linear.cu:98-170 */
void orc_linear_backward(const float *dY, const float *X, const float *W, float *dX,
                         float *dW, float *dB, int64_t M, int64_t K, int64_t N, int use_bias) {
    if (dX) gemm_nn(dY, N, W, K, dX, K, M, K, N);        /* matmul_tiled(dY, W) :119 */
    if (dW) gemm_tn(dY, N, X, K, dW, K, M, K, N);        /* A_T_B(dY, X) :150-158 */
    if (use_bias && dB) {                                /* compute_bias_grad_kernel :59-69 */
#pragma omp parallel for
        for (int64_t n = 0; n < N; ++n) {
            float g = 0.f;
            for (int64_t i = 0; i < M; ++i) g += dY[i * N + n];
            dB[n] += g;
        }
    }
}

/* mha.cu:18-122 */
void orc_mha_forward(const float *Q, const float *K, const float *V, float *out,
                     float *scores, const uint8_t *mask, int64_t B, int64_t S,
                     int64_t H, int64_t Dh, int causal) {
    int64_t E = H * Dh;
    const float scale = 1.0f / sqrtf((float)Dh);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h) {
            const float *Qb = Q + b * S * E + h * Dh;
            const float *Kb = K + b * S * E + h * Dh;
            const float *Vb = V + b * S * E + h * Dh;
            float *sc = scores + (b * H + h) * S * S;
            for (int64_t i = 0; i < S; ++i) {
                float row_max = -FLT_MAX;
                for (int64_t j = 0; j < S; ++j) {
                    if (causal && j > i) { sc[i * S + j] = -FLT_MAX; continue; }
                    if (mask && !mask[i * S + j]) { sc[i * S + j] = -FLT_MAX; continue; }
                    float dot = 0.f;
                    for (int64_t d = 0; d < Dh; ++d) dot = fmaf(Qb[i * E + d], Kb[j * E + d], dot);
                    float s = dot * scale;
                    sc[i * S + j] = s;
                    if (s > row_max) row_max = s;
                }
                float row_sum = 0.f;
                for (int64_t j = 0; j < S; ++j) {
                    float s = sc[i * S + j];
                    if (s == -FLT_MAX) sc[i * S + j] = 0.f;
                    else { float e = expf(s - row_max); sc[i * S + j] = e; row_sum += e; }
                }
                if (row_sum == 0.f) row_sum = 1e-20f;
                for (int64_t j = 0; j < S; ++j) sc[i * S + j] = sc[i * S + j] / row_sum;
                for (int64_t d = 0; d < Dh; ++d) {
                    float o = 0.f;
                    for (int64_t j = 0; j < S; ++j) {
                        float p = sc[i * S + j];
                        if (p == 0.f) continue;
                        o = fmaf(p, Vb[j * E + d], o);
                    }
                    out[(b * S + i) * E + h * Dh + d] = o;
                }
            }
        }
}

/* mha.cu:164-299 (dQ/dK accumulation done serially; the reference's
 * atomics make its summation order unspecified) */
void orc_mha_backward(const float *dO, const float *Q, const float *K, const float *V,
                      const float *P, const uint8_t *mask, float *dQ, float *dK, float *dV,
                      int64_t B, int64_t S, int64_t H, int64_t Dh, int causal,
                      int apply_scale) {
    int64_t E = H * Dh;
    const float scale = apply_scale ? 1.0f / sqrtf((float)Dh) : 1.0f;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h) {
            const float *Qb = Q + b * S * E + h * Dh, *Kb = K + b * S * E + h * Dh;
            const float *Vb = V + b * S * E + h * Dh, *dOb = dO + b * S * E + h * Dh;
            float *dQb = dQ + b * S * E + h * Dh, *dKb = dK + b * S * E + h * Dh;
            float *dVb = dV + b * S * E + h * Dh;
            const float *Pb = P + (b * H + h) * S * S;
            for (int64_t t = 0; t < S; ++t)
                for (int64_t d = 0; d < Dh; ++d) { dQb[t * E + d] = 0; dKb[t * E + d] = 0; dVb[t * E + d] = 0; }
            for (int64_t j = 0; j < S; ++j)
                for (int64_t d = 0; d < Dh; ++d) {
                    float acc = 0.f;
                    for (int64_t i = 0; i < S; ++i) {
                        if (causal && j > i) continue;
                        if (mask && !mask[i * S + j]) continue;
                        float p = Pb[i * S + j];
                        if (p == 0.f) continue;
                        acc = fmaf(p, dOb[i * E + d], acc);
                    }
                    dVb[j * E + d] = acc;
                }
            for (int64_t i = 0; i < S; ++i) {
                float spg = 0.f;
                for (int64_t j = 0; j < S; ++j) {
                    if (causal && j > i) continue;
                    if (mask && !mask[i * S + j]) continue;
                    float p = Pb[i * S + j];
                    if (p == 0.f) continue;
                    float g = 0.f;
                    for (int64_t d = 0; d < Dh; ++d) g = fmaf(dOb[i * E + d], Vb[j * E + d], g);
                    spg += p * g;
                }
                for (int64_t j = 0; j < S; ++j) {
                    if (causal && j > i) continue;
                    if (mask && !mask[i * S + j]) continue;
                    float p = Pb[i * S + j];
                    if (p == 0.f) continue;
                    float g = 0.f;
                    for (int64_t d = 0; d < Dh; ++d) g = fmaf(dOb[i * E + d], Vb[j * E + d], g);
                    float ds = p * (g - spg) * scale;
                    for (int64_t d = 0; d < Dh; ++d) {
                        dQb[i * E + d] += ds * Kb[j * E + d];
                        dKb[j * E + d] += ds * Qb[i * E + d];
                    }
                }
            }
        }
}

/* layernorm.cu:6-76 */
void orc_layernorm_forward(const float *x, const float *g, const float *b, float *y,
                           float *mean, float *rstd, int64_t M, int64_t N, float eps) {
    if (M <= 0 || N <= 0) return;
#pragma omp parallel for
    for (int64_t r = 0; r < M; ++r) {
        const float *xr = x + r * N;
        float s = 0.f;
        for (int64_t i = 0; i < N; ++i) s += xr[i];
        float m = s / (float)N;
        float v = 0.f;
        for (int64_t i = 0; i < N; ++i) { float d = xr[i] - m; v += d * d; }
        v /= (float)N;
        float rs = 1.0f / sqrtf(v + eps);
        if (mean) mean[r] = m;
        if (rstd) rstd[r] = rs;
        for (int64_t i = 0; i < N; ++i) y[r * N + i] = (xr[i] - m) * rs * g[i] + b[i];
    }
}

/* layernorm.cu:79-165 */
void orc_layernorm_backward(const float *x, const float *dy, const float *g,
                            const float *mean, const float *rstd, float *dx,
                            float *dg, float *db, int64_t M, int64_t N) {
    if (M <= 0 || N <= 0) return;
#pragma omp parallel for
    for (int64_t r = 0; r < M; ++r) {
        const float *xr = x + r * N, *dyr = dy + r * N;
        float m = mean[r], rs = rstd[r], s1 = 0.f, s2 = 0.f;
        for (int64_t i = 0; i < N; ++i) {
            float xh = (xr[i] - m) * rs, a = dyr[i] * g[i];
            s1 += a; s2 += a * xh;
        }
        float invN = 1.0f / (float)N;
        for (int64_t i = 0; i < N; ++i) {
            float xh = (xr[i] - m) * rs, a = dyr[i] * g[i];
            dx[r * N + i] = rs * (a - s1 * invN - xh * s2 * invN);
        }
    }
    /* d_gamma / d_beta: reference atomics, summed here row-ascending */
#pragma omp parallel for
    for (int64_t i = 0; i < N; ++i) {
        float sg = 0.f, sb = 0.f;
        for (int64_t r = 0; r < M; ++r) {
            float xh = (x[r * N + i] - mean[r]) * rstd[r];
            sg += dy[r * N + i] * xh; sb += dy[r * N + i];
        }
        dg[i] += sg; db[i] += sb;
    }
}

/* softmax.cu:12-65 */
void orc_softmax(const float *in, float *out, int M, int N) {
#pragma omp parallel for
    for (int r = 0; r < M; ++r) {
        const float *x = in + (int64_t)r * N;
        float *y = out + (int64_t)r * N;
        float mx = -FLT_MAX;
        for (int j = 0; j < N; ++j) mx = fmaxf(mx, x[j]);
        float s = 0.f;
        for (int j = 0; j < N; ++j) { y[j] = expf(x[j] - mx); s += y[j]; }
        for (int j = 0; j < N; ++j) y[j] /= s;
    }
}

/* cross_entropy.cpp:23-79 */
float orc_ce_forward(const float *probs, const int32_t *targets, int rows, int classes, float eps) {
    float total = 0.f;
    for (int i = 0; i < rows; ++i) {
        int t = targets[i];
        if (t >= 0 && t < classes) {
            float p = fmaxf(probs[(int64_t)i * classes + t], eps);
            total += -logf(p);
        }
    }
    return total / (float)rows;
}

/* cross_entropy.cu:5-31 */
void orc_ce_backward(float *dlogits, const float *probs, const int32_t *targets, int rows, int classes) {
#pragma omp parallel for
    for (int i = 0; i < rows; ++i) {
        int t = targets[i];
        for (int c = 0; c < classes; ++c) {
            int64_t idx = (int64_t)i * classes + c;
            float d = probs[idx];
            if (t >= 0 && t < classes && c == t) d = probs[idx] - 1.0f;
            dlogits[idx] = d / (float)rows;
        }
    }
}

/* embedding.cu:6-30 */
void orc_embedding_forward(const int32_t *ids, const float *table, const float *pos,
                           float *out, int B, int S, int D, int V, int max_seq_len) {
    if (B <= 0 || S <= 0 || D <= 0) return;
    for (int b = 0; b < B; ++b)
        for (int s = 0; s < S; ++s) {
            if (s >= max_seq_len) continue;
            int id = ids[b * S + s];
            if (id < 0 || id >= V) continue;
            for (int k = 0; k < D; ++k)
                out[((int64_t)b * S + s) * D + k] = table[(int64_t)id * D + k] + pos[(int64_t)s * D + k];
        }
}

/* embedding.cu:33-53 */
void orc_embedding_backward(const int32_t *ids, const float *dout, float *dtable,
                            int B, int S, int D, int V) {
    if (B <= 0 || S <= 0 || D <= 0) return;
    for (int t = 0; t < B * S; ++t) {
        int id = ids[t];
        if (id < 0 || id >= V) continue;
        for (int k = 0; k < D; ++k) dtable[(int64_t)id * D + k] += dout[(int64_t)t * D + k];
    }
}

void orc_add(const float *a, const float *b, float *out, int64_t n) {        /* add.cu:9-16 */
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}
void orc_add_inplace(float *a, const float *b, int64_t n) {                    /* add.cu:22-31 */
    for (int64_t i = 0; i < n; ++i) a[i] += b[i];
}
void orc_relu_forward(const float *x, float *y, int64_t n) {                   /* relu.cu:6-11 */
    for (int64_t i = 0; i < n; ++i) y[i] = x[i] > 0 ? x[i] : 0.f;
}
void orc_relu_backward(const float *x, const float *gy, float *gx, int64_t n) { /* relu.cu:13-19 */
    for (int64_t i = 0; i < n; ++i) gx[i] = x[i] > 0 ? gy[i] : 0.f;
}
void orc_transpose(const float *in, float *out, int rows, int cols) {          /* transpose.cu:6-15 */
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < cols; ++j) out[(int64_t)j * rows + i] = in[(int64_t)i * cols + j];
}

/* adamw.cu:9-75 */
void orc_adamw(float *p, const float *g, float *m, float *v, int64_t n, float lr, float wd,
               float b1, float b2, float eps, float bc1, float bc2) {
#pragma omp parallel for
    for (int64_t i = 0; i < n; ++i) {
        float pv = p[i], gv = g[i];
        float mv = b1 * m[i] + (1.0f - b1) * gv;
        float vv = b2 * v[i] + (1.0f - b2) * gv * gv;
        m[i] = mv; v[i] = vv;
        float mh = mv / bc1, vh = vv / bc2;
        float step = lr * mh / (sqrtf(vh) + eps);
        float decay = (wd != 0.f) ? lr * wd * pv : 0.f;
        p[i] = pv - (decay + step);
    }
}

/* adam.cu:13-57 */
void orc_adam(float *p, const float *g, float *m, float *v, int64_t n, float lr,
              float b1, float b2, float eps, float bc1, float bc2) {
#pragma omp parallel for
    for (int64_t i = 0; i < n; ++i) {
        float gv = g[i];
        float mv = b1 * m[i] + (1.0f - b1) * gv;
        float vv = b2 * v[i] + (1.0f - b2) * gv * gv;
        m[i] = mv; v[i] = vv;
        p[i] -= lr * (mv / bc1) / (sqrtf(vv / bc2) + eps);
    }
}

/* sgd.cu:14-57 */
void orc_sgd(float *p, const float *g, float *vel, int64_t n, float lr, float momentum, float wd) {
    for (int64_t i = 0; i < n; ++i) {
        float pv = p[i], gv = g[i];
        if (wd != 0.f) gv += wd * pv;
        if (momentum != 0.f && vel) { float vv = momentum * vel[i] + gv; vel[i] = vv; gv = vv; }
        p[i] = pv - lr * gv;
    }
}

/* embedding.cpp:107-126 */
void orc_sinusoid_table(float *out, int max_seq_len, int D) {
    for (int pos = 0; pos < max_seq_len; ++pos)
        for (int i = 0; i < D; ++i) {
            int k = i / 2;
            float ang = (float)pos / powf(10000.0f, (float)(2 * k) / (float)D);
            out[(int64_t)pos * D + i] = (i % 2 == 0) ? sinf(ang) : cosf(ang);
        }
}

/* ======================================================================= */
/* definitions with no reference kernel                                     */
/* ======================================================================= */
void orc_rmsnorm_forward(const float *x, const float *g, float *y, float *rstd,
                         int64_t M, int64_t N, float eps) {
#pragma omp parallel for
    for (int64_t r = 0; r < M; ++r) {
        const float *xr = x + r * N;
        double ss = 0.0;
        for (int64_t i = 0; i < N; ++i) ss += (double)xr[i] * xr[i];
        float rs = (float)(1.0 / sqrt(ss / (double)N + (double)eps));
        if (rstd) rstd[r] = rs;
        for (int64_t i = 0; i < N; ++i) y[r * N + i] = xr[i] * rs * g[i];
    }
}

void orc_rmsnorm_backward(const float *x, const float *dy, const float *g, const float *rstd,
                          float *dx, float *dg, int64_t M, int64_t N) {
#pragma omp parallel for
    for (int64_t r = 0; r < M; ++r) {
        const float *xr = x + r * N, *dyr = dy + r * N;
        float rs = rstd[r];
        double s = 0.0;
        for (int64_t i = 0; i < N; ++i) s += (double)dyr[i] * g[i] * xr[i] * rs;
        float c = (float)(s / (double)N);
        for (int64_t i = 0; i < N; ++i) {
            float xh = xr[i] * rs;
            dx[r * N + i] = rs * (dyr[i] * g[i] - xh * c);
        }
    }
#pragma omp parallel for
    for (int64_t i = 0; i < N; ++i) {
        double sg = 0.0;
        for (int64_t r = 0; r < M; ++r) sg += (double)dy[r * N + i] * x[r * N + i] * rstd[r];
        dg[i] += (float)sg;
    }
}

void orc_rope_table(float *cos_t, float *sin_t, int S, int Dh, double base) {
    int half = Dh / 2;
    for (int p = 0; p < S; ++p)
        for (int i = 0; i < half; ++i) {
            double inv = pow(base, -2.0 * i / (double)Dh);
            double th = (double)p * inv;
            cos_t[(int64_t)p * half + i] = (float)cos(th);
            sin_t[(int64_t)p * half + i] = (float)sin(th);
        }
}

void orc_rope_apply(float *x, int64_t T, int S, int H, int Dh, int row_stride,
                    const float *cos_t, const float *sin_t, int inverse) {
    int half = Dh / 2;
#pragma omp parallel for
    for (int64_t t = 0; t < T; ++t) {
        int p = (int)(t % S);
        for (int h = 0; h < H; ++h) {
            float *xh = x + t * row_stride + (int64_t)h * Dh;
            for (int i = 0; i < half; ++i) {
                float c = cos_t[(int64_t)p * half + i], s = sin_t[(int64_t)p * half + i];
                if (inverse) s = -s;
                float a = xh[2 * i], b = xh[2 * i + 1];
                xh[2 * i] = a * c - b * s;
                xh[2 * i + 1] = a * s + b * c;
            }
        }
    }
}

void orc_attention_forward(const float *q, const float *k, const float *v, int ld,
                           float *o, int ldo, float *lse, int B, int S, int H, int Dh) {
    const float scale = 1.0f / sqrtf((float)Dh);
#pragma omp parallel
    {
        float *p = (float *)malloc((size_t)S * sizeof(float));
#pragma omp for collapse(3) schedule(dynamic, 16)
        for (int b = 0; b < B; ++b)
            for (int h = 0; h < H; ++h)
                for (int i = 0; i < S; ++i) {
                    const float *qi = q + ((int64_t)b * S + i) * ld + (int64_t)h * Dh;
                    float mx = -INFINITY;
                    for (int j = 0; j <= i; ++j) {
                        const float *kj = k + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                        float s = 0.f;
#pragma omp simd reduction(+ : s)
                        for (int d = 0; d < Dh; ++d) s += qi[d] * kj[d];
                        p[j] = s * scale;
                        if (p[j] > mx) mx = p[j];
                    }
                    double l = 0.0;
                    for (int j = 0; j <= i; ++j) { p[j] = expf(p[j] - mx); l += p[j]; }
                    float inv = (float)(1.0 / l);
                    float *oi = o + ((int64_t)b * S + i) * ldo + (int64_t)h * Dh;
                    for (int d = 0; d < Dh; ++d) oi[d] = 0.f;
                    for (int j = 0; j <= i; ++j) {
                        const float *vj = v + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                        float w = p[j] * inv;
#pragma omp simd
                        for (int d = 0; d < Dh; ++d) oi[d] += w * vj[d];
                    }
                    if (lse) lse[((int64_t)b * H + h) * S + i] = mx + (float)log(l);
                }
        free(p);
    }
}

void orc_attention_backward(const float *q, const float *k, const float *v, int ld,
                            const float *o, const float *dO, int ldo, const float *lse,
                            float *dq, float *dk, float *dv, int ldd,
                            int B, int S, int H, int Dh) {
    const float scale = 1.0f / sqrtf((float)Dh);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            float *ds = (float *)malloc((size_t)S * sizeof(float));
            float *Drow = (float *)malloc((size_t)S * sizeof(float));
            for (int t = 0; t < S; ++t) {
                float *a = dq + ((int64_t)b * S + t) * ldd + (int64_t)h * Dh;
                float *c = dk + ((int64_t)b * S + t) * ldd + (int64_t)h * Dh;
                float *e = dv + ((int64_t)b * S + t) * ldd + (int64_t)h * Dh;
                for (int d = 0; d < Dh; ++d) { a[d] = 0.f; c[d] = 0.f; e[d] = 0.f; }
                const float *oi = o + ((int64_t)b * S + t) * ldo + (int64_t)h * Dh;
                const float *gi = dO + ((int64_t)b * S + t) * ldo + (int64_t)h * Dh;
                float s = 0.f;
                for (int d = 0; d < Dh; ++d) s += oi[d] * gi[d];
                Drow[t] = s;
            }
            for (int i = 0; i < S; ++i) {
                const float *qi = q + ((int64_t)b * S + i) * ld + (int64_t)h * Dh;
                const float *gi = dO + ((int64_t)b * S + i) * ldo + (int64_t)h * Dh;
                float L = lse[((int64_t)b * H + h) * S + i];
                float *dqi = dq + ((int64_t)b * S + i) * ldd + (int64_t)h * Dh;
                for (int j = 0; j <= i; ++j) {
                    const float *kj = k + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                    const float *vj = v + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                    float sc = 0.f, dp = 0.f;
                    for (int d = 0; d < Dh; ++d) { sc += qi[d] * kj[d]; dp += gi[d] * vj[d]; }
                    float p = expf(sc * scale - L);
                    float *dvj = dv + ((int64_t)b * S + j) * ldd + (int64_t)h * Dh;
                    for (int d = 0; d < Dh; ++d) dvj[d] += p * gi[d];
                    ds[j] = p * (dp - Drow[i]) * scale;
                }
                for (int j = 0; j <= i; ++j) {
                    const float *kj = k + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                    float *dkj = dk + ((int64_t)b * S + j) * ldd + (int64_t)h * Dh;
                    float w = ds[j];
                    for (int d = 0; d < Dh; ++d) { dqi[d] += w * kj[d]; dkj[d] += w * qi[d]; }
                }
            }
            free(ds); free(Drow);
        }
}

/* Flash-style causal attention forward with the B200 kernels' order: key
 * blocks of 128 when S is a multiple of 128 (tcgen05 kernel), else 64
 * (mma.sync kernel); running max in base 2, probabilities rounded to bf16
 * before the P.V product, row sum of the unrounded probabilities, output / sum. */
static void attention_forward_blockwise(const float *q, const float *k, const float *v, int ld, float *o, int ldo,
                                        float *lse, int B, int S, int H, int Dh) {
    const float scale_log2 = (1.0f / sqrtf((float)Dh)) * 1.4426950408889634f;
#pragma omp parallel
    {
        float *acc = (float *)malloc((size_t)Dh * sizeof(float));
        const int KB = (S % 128 == 0) ? 128 : 64;
        float *sv = (float *)malloc(128 * sizeof(float));
#pragma omp for collapse(3) schedule(dynamic, 16)
        for (int b = 0; b < B; ++b)
            for (int h = 0; h < H; ++h)
                for (int i = 0; i < S; ++i) {
                    const float *qi = q + ((int64_t)b * S + i) * ld + (int64_t)h * Dh;
                    float m = -INFINITY, l = 0.f;
                    for (int d = 0; d < Dh; ++d) acc[d] = 0.f;
                    for (int j0 = 0; j0 <= i; j0 += KB) {
                        const int j1 = (j0 + KB <= i + 1) ? j0 + KB : i + 1;
                        float mx = -INFINITY;
                        for (int j = j0; j < j1; ++j) {
                            const float *kj = k + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                            float sc = 0.f;
                            for (int d = 0; d < Dh; ++d) sc += qi[d] * kj[d];
                            sv[j - j0] = sc * scale_log2;
                            if (sv[j - j0] > mx) mx = sv[j - j0];
                        }
                        const float mnew = m > mx ? m : mx;
                        const float corr = exp2f(m - mnew);
                        float sum = 0.f;
                        for (int d = 0; d < Dh; ++d) acc[d] *= corr;
                        for (int j = j0; j < j1; ++j) {
                            const float p = exp2f(sv[j - j0] - mnew);
                            sum += p;
                            const float pb = bf16r(p);
                            const float *vj = v + ((int64_t)b * S + j) * ld + (int64_t)h * Dh;
                            for (int d = 0; d < Dh; ++d) acc[d] += pb * vj[d];
                        }
                        l = l * corr + sum;
                        m = mnew;
                    }
                    float *oi = o + ((int64_t)b * S + i) * ldo + (int64_t)h * Dh;
                    for (int d = 0; d < Dh; ++d) oi[d] = acc[d] / l;
                    if (lse) lse[((int64_t)b * H + h) * S + i] = (m + log2f(l)) * 0.6931471805599453f;
                }
        free(acc);
        free(sv);
    }
}

float orc_ce_fused(const float *logits, const int32_t *targets, float *dlogits,
                   int rows, int classes, float eps) {
    const float cap = -logf(eps);
    double total = 0.0;
#pragma omp parallel for reduction(+ : total)
    for (int r = 0; r < rows; ++r) {
        const float *x = logits + (int64_t)r * classes;
        float mx = -INFINITY;
        for (int c = 0; c < classes; ++c) mx = fmaxf(mx, x[c]);
        double s = 0.0;
        for (int c = 0; c < classes; ++c) s += exp((double)x[c] - mx);
        float lse = mx + (float)log(s);
        int t = targets[r];
        if (t >= 0 && t < classes) {
            float l = lse - x[t];
            total += (l < cap) ? l : cap;
        }
        if (dlogits) {
            float inv_rows = 1.0f / (float)rows;
            for (int c = 0; c < classes; ++c) {
                float p = expf(x[c] - lse);
                if (c == t) p -= 1.0f;
                dlogits[(int64_t)r * classes + c] = p * inv_rows;
            }
        }
    }
    return (float)(total / rows);
}

/* ======================================================================= */
/* whole step                                                               */
/* ======================================================================= */
enum { K_MAT = 0, K_BIAS = 1, K_GAMMA = 2, K_BETA = 3, K_EMB = 4 };

/* tensor ids inside one layer (reverse forward order) */
enum { L_N2G, L_N2B, L_W2, L_B2, L_W1, L_B1, L_N1G, L_N1B, L_WO, L_BO, L_WQKV, L_BQKV, L_COUNT };

typedef struct {
    int64_t head, nog, nob, emb;
    int64_t lay[64][L_COUNT];
} layout_t;

static int build_layout(const orc_model_cfg *c, layout_t *L, int64_t *offs, int64_t *sizes,
                        int *kinds, int max_n, int64_t *total) {
    int64_t off = 0;
    int n = 0;
    int64_t d = c->dim, F = c->ffn, V = c->vocab;
#define ADD(dst, sz, kind)                                              \
    do {                                                                \
        (dst) = off;                                                    \
        if (n < max_n) { if (offs) offs[n] = off; if (sizes) sizes[n] = (sz); if (kinds) kinds[n] = (kind); } \
        off += (sz); n++;                                               \
    } while (0)
    L->head = L->nob = -1;
    if (!c->tied) ADD(L->head, V * d, K_MAT);
    ADD(L->nog, d, K_GAMMA);
    if (c->norm == 0) ADD(L->nob, d, K_BETA);
    for (int l = c->layers - 1; l >= 0; --l) {
        int64_t *t = L->lay[l];
        for (int q = 0; q < L_COUNT; ++q) t[q] = -1;
        ADD(t[L_N2G], d, K_GAMMA);
        if (c->norm == 0) ADD(t[L_N2B], d, K_BETA);
        ADD(t[L_W2], d * F, K_MAT);
        if (c->bias) ADD(t[L_B2], d, K_BIAS);
        ADD(t[L_W1], F * d, K_MAT);
        if (c->bias) ADD(t[L_B1], F, K_BIAS);
        ADD(t[L_N1G], d, K_GAMMA);
        if (c->norm == 0) ADD(t[L_N1B], d, K_BETA);
        ADD(t[L_WO], d * d, K_MAT);
        if (c->bias) ADD(t[L_BO], d, K_BIAS);
        ADD(t[L_WQKV], 3 * d * d, K_MAT);
        if (c->bias) ADD(t[L_BQKV], 3 * d, K_BIAS);
    }
    ADD(L->emb, V * d, K_EMB);
#undef ADD
    if (total) *total = off;
    return n;
}

int orc_param_layout(const orc_model_cfg *cfg, int64_t *offsets, int64_t *sizes,
                     int *kinds, int max_n, int64_t *total) {
    layout_t L;
    if (cfg->layers > 64) return -1;
    return build_layout(cfg, &L, offsets, sizes, kinds, max_n, total);
}

void orc_init_params(const orc_model_cfg *cfg, float *params, uint64_t seed, float init_std) {
    int64_t offs[1024], sizes[1024];
    int kinds[1024];
    int64_t total;
    int n = orc_param_layout(cfg, offs, sizes, kinds, 1024, &total);
    for (int i = 0; i < n; ++i) {
        float *p = params + offs[i];
        if (kinds[i] == K_MAT || kinds[i] == K_EMB)
            orc_fill_normal(p, sizes[i], seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(i + 1)), 0.f, init_std);
        else if (kinds[i] == K_GAMMA)
            for (int64_t j = 0; j < sizes[i]; ++j) p[j] = 1.f;
        else
            for (int64_t j = 0; j < sizes[i]; ++j) p[j] = 0.f;
    }
}

static float *falloc(int64_t n) { return (float *)calloc((size_t)n, sizeof(float)); }

static void bias_add(float *y, const float *b, int64_t M, int64_t N) {
#pragma omp parallel for
    for (int64_t i = 0; i < M; ++i)
        for (int64_t n = 0; n < N; ++n) y[i * N + n] += b[n];
}
static void colsum_acc(const float *dy, float *db, int64_t M, int64_t N) {
#pragma omp parallel for
    for (int64_t n = 0; n < N; ++n) {
        double s = 0.0;
        for (int64_t i = 0; i < M; ++i) s += dy[i * N + n];
        db[n] += (float)s;
    }
}

static void norm_fwd(const orc_model_cfg *c, const float *x, const float *g, const float *b,
                     float *y, float *mean, float *rstd, int64_t T) {
    if (c->norm == 0) orc_layernorm_forward(x, g, b, y, mean, rstd, T, c->dim, c->eps);
    else orc_rmsnorm_forward(x, g, y, rstd, T, c->dim, c->eps);
}
static void norm_bwd(const orc_model_cfg *c, const float *x, const float *dy, const float *g,
                     const float *mean, const float *rstd, float *dx, float *dg, float *db, int64_t T) {
    if (c->norm == 0) orc_layernorm_backward(x, dy, g, mean, rstd, dx, dg, db, T, c->dim);
    else orc_rmsnorm_backward(x, dy, g, rstd, dx, dg, T, c->dim);
}

typedef struct {
    float *x;      /* layer input [T,d] */
    float *qkv;    /* [T,3d] after bias (and RoPE on q,k) */
    float *attn;   /* [T,d] */
    float *lse;    /* [B,H,S] */
    float *r1, *h1, *mean1, *rstd1;
    float *f;      /* relu output [T,F] */
    float *r2, *mean2, *rstd2;
} layer_acts;

float orc_train_step(const orc_model_cfg *c, float *P, float *G, float *Mo, float *Vo,
                     const int32_t *ids, const int32_t *targets, int B, int S,
                     const orc_adamw_cfg *opt, float *logits_out) {
    layout_t Ly;
    int64_t total;
    build_layout(c, &Ly, NULL, NULL, NULL, 0, &total);
    const int64_t T = (int64_t)B * S, d = c->dim, F = c->ffn, V = c->vocab;
    const int H = c->heads, Dh = (int)(d / H);
    memset(G, 0, (size_t)total * sizeof(float));

    float *pos_tab = NULL, *rc = NULL, *rsn = NULL;
    if (c->pos == 0) { pos_tab = falloc((int64_t)c->max_seq * d); orc_sinusoid_table(pos_tab, c->max_seq, (int)d); }
    else { rc = falloc((int64_t)S * Dh / 2); rsn = falloc((int64_t)S * Dh / 2); orc_rope_table(rc, rsn, S, Dh, c->rope_base); }

    /* weights as the GEMMs see them (bf16 shadow in emulation mode) */
    float *Pw = falloc(total);
    memcpy(Pw, P, (size_t)total * sizeof(float));
    if (g_bf16) {
        int64_t offs_[1024], sizes_[1024];
        int kinds_[1024];
        int nt = orc_param_layout(c, offs_, sizes_, kinds_, 1024, NULL);
        for (int i = 0; i < nt; ++i)
            if (kinds_[i] == K_MAT || kinds_[i] == K_EMB) round_bf16(Pw + offs_[i], sizes_[i]);
    }
    layer_acts *A = (layer_acts *)calloc((size_t)c->layers, sizeof(layer_acts));
    float *x = falloc(T * d);
    /* embedding: x = E[id] (+ PE[s]) */
    for (int64_t t = 0; t < T; ++t) {
        int id = ids[t];
        int s = (int)(t % S);
        if (id < 0 || id >= V) continue;
        for (int64_t k = 0; k < d; ++k)
            x[t * d + k] = P[Ly.emb + (int64_t)id * d + k] + (pos_tab ? pos_tab[(int64_t)s * d + k] : 0.f);
    }
    round_bf16(x, T * d);
    for (int l = 0; l < c->layers; ++l) {
        int64_t *o = Ly.lay[l];
        layer_acts *a = &A[l];
        a->x = x;
        a->qkv = falloc(T * 3 * d);
        gemm_nt(x, d, Pw + o[L_WQKV], d, a->qkv, 3 * d, T, 3 * d, d);
        if (c->bias) bias_add(a->qkv, P + o[L_BQKV], T, 3 * d);
        if (c->pos == 1) {
            orc_rope_apply(a->qkv, T, S, H, Dh, (int)(3 * d), rc, rsn, 0);
            orc_rope_apply(a->qkv + d, T, S, H, Dh, (int)(3 * d), rc, rsn, 0);
        }
        round_bf16(a->qkv, T * 3 * d);
        a->attn = falloc(T * d);
        a->lse = falloc((int64_t)B * H * S);
        if (g_bf16)
            attention_forward_blockwise(a->qkv, a->qkv + d, a->qkv + 2 * d, (int)(3 * d), a->attn, (int)d, a->lse,
                                        B, S, H, Dh);
        else
            orc_attention_forward(a->qkv, a->qkv + d, a->qkv + 2 * d, (int)(3 * d), a->attn, (int)d, a->lse, B, S,
                                  H, Dh);
        round_bf16(a->attn, T * d);
        a->r1 = falloc(T * d);
        gemm_nt(a->attn, d, Pw + o[L_WO], d, a->r1, d, T, d, d);
        if (c->bias) bias_add(a->r1, P + o[L_BO], T, d);
        for (int64_t i = 0; i < T * d; ++i) a->r1[i] += x[i];
        round_bf16(a->r1, T * d);
        a->h1 = falloc(T * d); a->mean1 = falloc(T); a->rstd1 = falloc(T);
        norm_fwd(c, a->r1, P + o[L_N1G], c->norm == 0 ? P + o[L_N1B] : NULL, a->h1, a->mean1, a->rstd1, T);
        round_bf16(a->h1, T * d);
        a->f = falloc(T * F);
        gemm_nt(a->h1, d, Pw + o[L_W1], d, a->f, F, T, F, d);
        if (c->bias) bias_add(a->f, P + o[L_B1], T, F);
        for (int64_t i = 0; i < T * F; ++i) a->f[i] = a->f[i] > 0.f ? a->f[i] : 0.f;
        round_bf16(a->f, T * F);
        a->r2 = falloc(T * d);
        gemm_nt(a->f, F, Pw + o[L_W2], F, a->r2, d, T, d, F);
        if (c->bias) bias_add(a->r2, P + o[L_B2], T, d);
        for (int64_t i = 0; i < T * d; ++i) a->r2[i] += a->h1[i];
        round_bf16(a->r2, T * d);
        a->mean2 = falloc(T); a->rstd2 = falloc(T);
        x = falloc(T * d);
        norm_fwd(c, a->r2, P + o[L_N2G], c->norm == 0 ? P + o[L_N2B] : NULL, x, a->mean2, a->rstd2, T);
        round_bf16(x, T * d);
    }
    float *hf = falloc(T * d), *meanf = falloc(T), *rstdf = falloc(T);
    norm_fwd(c, x, P + Ly.nog, c->norm == 0 ? P + Ly.nob : NULL, hf, meanf, rstdf, T);
    round_bf16(hf, T * d);
    const float *Whead = c->tied ? Pw + Ly.emb : Pw + Ly.head;
    float *logits = falloc(T * V);
    gemm_nt(hf, d, Whead, d, logits, V, T, V, d);
    round_bf16(logits, T * V);
    if (logits_out) memcpy(logits_out, logits, (size_t)(T * V) * sizeof(float));
    float *dlog = logits; /* overwritten in place by the fused CE */
    float *tmp = falloc(T * V);
    float loss = orc_ce_fused(logits, targets, tmp, (int)T, (int)V, 1e-8f);
    memcpy(dlog, tmp, (size_t)(T * V) * sizeof(float));
    free(tmp);
    round_bf16(dlog, T * V);

    /* ---------------- backward ---------------- */
    float *gWhead = c->tied ? G + Ly.emb : G + Ly.head;
    float *dWtmp = falloc(V * d);
    gemm_tn(dlog, V, hf, d, dWtmp, d, T, d, V);
    for (int64_t i = 0; i < V * d; ++i) gWhead[i] += dWtmp[i];
    free(dWtmp);
    float *dhf = falloc(T * d);
    gemm_nn(dlog, V, Whead, d, dhf, d, T, d, V);
    round_bf16(dhf, T * d);
    float *dx = falloc(T * d);
    norm_bwd(c, x, dhf, P + Ly.nog, meanf, rstdf, dx, G + Ly.nog, c->norm == 0 ? G + Ly.nob : NULL, T);
    round_bf16(dx, T * d);
    free(dhf);
    float *dtmp = falloc(T * d), *dF = falloc(T * F), *dqkv = falloc(T * 3 * d), *dattn = falloc(T * d);
    float *dr = falloc(T * d);
    for (int l = c->layers - 1; l >= 0; --l) {
        int64_t *o = Ly.lay[l];
        layer_acts *a = &A[l];
        /* out = norm2(r2) */
        norm_bwd(c, a->r2, dx, P + o[L_N2G], a->mean2, a->rstd2, dr, G + o[L_N2G],
                 c->norm == 0 ? G + o[L_N2B] : NULL, T);
        round_bf16(dr, T * d);
        /* r2 = h1 + f W2^T + b2 */
        gemm_tn(dr, d, a->f, F, G + o[L_W2], F, T, F, d);
        if (c->bias) colsum_acc(dr, G + o[L_B2], T, d);
        gemm_nn(dr, d, Pw + o[L_W2], F, dF, F, T, F, d);
        for (int64_t i = 0; i < T * F; ++i) if (!(a->f[i] > 0.f)) dF[i] = 0.f;
        round_bf16(dF, T * F);
        gemm_tn(dF, F, a->h1, d, G + o[L_W1], d, T, d, F);
        if (c->bias) colsum_acc(dF, G + o[L_B1], T, F);
        gemm_nn(dF, F, Pw + o[L_W1], d, dtmp, d, T, d, F);
        for (int64_t i = 0; i < T * d; ++i) dtmp[i] += dr[i];        /* dh1 */
        round_bf16(dtmp, T * d);
        /* h1 = norm1(r1) */
        norm_bwd(c, a->r1, dtmp, P + o[L_N1G], a->mean1, a->rstd1, dr, G + o[L_N1G],
                 c->norm == 0 ? G + o[L_N1B] : NULL, T);
        round_bf16(dr, T * d);
        /* r1 = x + attn Wo^T + bo */
        gemm_tn(dr, d, a->attn, d, G + o[L_WO], d, T, d, d);
        if (c->bias) colsum_acc(dr, G + o[L_BO], T, d);
        gemm_nn(dr, d, Pw + o[L_WO], d, dattn, d, T, d, d);
        round_bf16(dattn, T * d);
        orc_attention_backward(a->qkv, a->qkv + d, a->qkv + 2 * d, (int)(3 * d), a->attn, dattn, (int)d,
                               a->lse, dqkv, dqkv + d, dqkv + 2 * d, (int)(3 * d), B, S, H, Dh);
        if (c->pos == 1) {
            orc_rope_apply(dqkv, T, S, H, Dh, (int)(3 * d), rc, rsn, 1);
            orc_rope_apply(dqkv + d, T, S, H, Dh, (int)(3 * d), rc, rsn, 1);
        }
        round_bf16(dqkv, T * 3 * d);
        gemm_tn(dqkv, 3 * d, a->x, d, G + o[L_WQKV], d, T, d, 3 * d);
        if (c->bias) colsum_acc(dqkv, G + o[L_BQKV], T, 3 * d);
        gemm_nn(dqkv, 3 * d, Pw + o[L_WQKV], d, dx, d, T, d, 3 * d);
        for (int64_t i = 0; i < T * d; ++i) dx[i] += dr[i];
        round_bf16(dx, T * d);
    }
    /* embedding scatter-add (embedding.cu:33-53) */
    for (int64_t t = 0; t < T; ++t) {
        int id = ids[t];
        if (id < 0 || id >= V) continue;
        for (int64_t k = 0; k < d; ++k) G[Ly.emb + (int64_t)id * d + k] += dx[t * d + k];
    }

    /* ---------------- AdamW ---------------- */
    if (opt) {
        float bc1 = 1.0f - powf(opt->beta1, (float)opt->step);
        float bc2 = 1.0f - powf(opt->beta2, (float)opt->step);
        float *gs = G;
        float *scaled = NULL;
        if (opt->grad_scale != 1.0f) {
            scaled = falloc(total);
            for (int64_t i = 0; i < total; ++i) scaled[i] = G[i] * opt->grad_scale;
            gs = scaled;
        }
        orc_adamw(P, gs, Mo, Vo, total, opt->lr, opt->weight_decay, opt->beta1, opt->beta2, opt->eps, bc1, bc2);
        free(scaled);
    }

    /* cleanup */
    for (int l = 0; l < c->layers; ++l) {
        layer_acts *a = &A[l];
        free(a->x); free(a->qkv); free(a->attn); free(a->lse); free(a->r1); free(a->h1);
        free(a->mean1); free(a->rstd1); free(a->f); free(a->r2); free(a->mean2); free(a->rstd2);
    }
    free(A); free(x); free(hf); free(meanf); free(rstdf); free(logits);
    free(dtmp); free(dF); free(dqkv); free(dattn); free(dr); free(dx);
    free(pos_tab); free(rc); free(rsn); free(Pw);
    return loss;
}
