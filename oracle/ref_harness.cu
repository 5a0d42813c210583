// ref_harness.cu -- C entry points over the reference's own CUDA kernels.
//
// TEST INFRASTRUCTURE ONLY.  Compiled together with the unmodified
// reference sources src/kernel/cuda/*.cu (see Makefile target `ref`) into
// oracle/_ref/libzlref.so, so GPU tests can run the reference kernels on
// the same seeded inputs and pin the CPU oracle against them.  Each
// function calls exactly one reference host launcher, synchronises, and
// returns 0 on success, 1 if the launcher threw, 2 on a CUDA error.
#include <cuda_runtime.h>

#include <cstdint>
#include <exception>

#include "adam.cuh"
#include "adamw.cuh"
#include "add.cuh"
#include "cross_entropy.cuh"
#include "embedding.cuh"
#include "layernorm.cuh"
#include "linear.cuh"
#include "matmul.cuh"
#include "mha.cuh"
#include "relu.cuh"
#include "sgd.cuh"
#include "softmax.cuh"
#include "transpose.cuh"

template <typename F>
static int run(F&& f) {
  try {
    f();
  } catch (const std::exception&) {
    return 1;
  }
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}

extern "C" {
int ref_matmul(const float* A, const float* B, float* C, int M, int N, int K) {
  return run([&] { matmul<float>(A, B, C, M, N, K); });
}
int ref_matmul_tiled(const float* A, const float* B, float* C, int M, int N, int K) {
  return run([&] { matmul_tiled<float>(A, B, C, M, N, K); });
}
int ref_matmul_at_b(const float* A, const float* B, float* C, int M, int N, int K) {
  return run([&] { matmul_transposed_tiled_A_T_B<float>(A, B, C, M, N, K); });
}
int ref_matmul_a_bt(const float* A, const float* B, float* C, int M, int N, int K) {
  return run([&] { matmul_transposed_tiled_A_B_T<float>(A, B, C, M, N, K); });
}
int ref_linear_forward(const float* x, const float* W, const float* b, float* y, int64_t M, int64_t K, int64_t N,
                       int use_bias) {
  return run([&] { linear_forward<float>(x, W, b, y, M, K, N, use_bias != 0); });
}
int ref_linear_backward(const float* dY, const float* X, const float* W, float* dX, float* dW, float* dB, int64_t M,
                        int64_t K, int64_t N, int use_bias) {
  return run([&] { linear_backward<float>(dY, X, W, dX, dW, dB, M, K, N, use_bias != 0); });
}
int ref_mha_forward(const float* Q, const float* K, const float* V, float* out, float* scores, const bool* mask,
                    int64_t B, int64_t S, int64_t H, int64_t Dh, int causal) {
  return run([&] { mha_forward<float>(Q, K, V, out, scores, mask, B, S, H, Dh, causal != 0); });
}
int ref_mha_backward(const float* dO, const float* Q, const float* K, const float* V, const float* P, const bool* mask,
                     float* dQ, float* dK, float* dV, int64_t B, int64_t S, int64_t H, int64_t Dh, int causal) {
  return run([&] { mha_backward<float>(dO, Q, K, V, P, mask, dQ, dK, dV, B, S, H, Dh, causal != 0); });
}
int ref_layernorm_forward(const float* x, const float* g, const float* b, float* y, float* mean, float* rstd,
                          int64_t M, int64_t N, float eps) {
  return run([&] { cuda_layernorm_forward<float>(x, g, b, y, mean, rstd, M, N, eps); });
}
int ref_layernorm_backward(const float* x, const float* dy, const float* g, const float* mean, const float* rstd,
                           float* dx, float* dg, float* db, int64_t M, int64_t N) {
  return run([&] { cuda_layernorm_backward<float>(x, dy, g, mean, rstd, dx, dg, db, M, N); });
}
int ref_softmax(const float* x, float* y, int M, int N) {
  return run([&] { softmax<float>(x, y, M, N); });
}
int ref_ce_backward(float* d, const float* p, const int* t, int rows, int C) {
  return run([&] { cross_entropy_backward_kernel(d, p, t, rows, C); });
}
int ref_embedding_forward(const int* ids, const float* table, const float* pos, float* out, int B, int S, int D, int V,
                          int max_seq_len) {
  return run([&] { cuda_embedding_forward<float, int>(ids, table, pos, out, B, S, D, V, max_seq_len); });
}
int ref_embedding_backward(const int* ids, const float* dout, float* dtable, int B, int S, int D, int V) {
  return run([&] { cuda_embedding_backward<float, int>(ids, dout, dtable, B, S, D, V); });
}
int ref_add(const float* a, const float* b, float* o, int n) { return run([&] { add<float>(a, b, o, n); }); }
int ref_add_inplace(float* a, const float* b, int n) { return run([&] { add_inplace<float>(a, b, n); }); }
int ref_relu_forward(const float* x, float* y, int n) { return run([&] { relu_forward<float>(x, y, n); }); }
int ref_relu_backward(const float* x, const float* gy, float* gx, int n) {
  return run([&] { relu_backward<float>(x, gy, gx, n); });
}
int ref_transpose(const float* x, float* y, int rows, int cols) {
  return run([&] { transpose<float>(x, y, rows, cols); });
}
int ref_adamw(float* p, const float* g, float* m, float* v, int n, float lr, float wd, float b1, float b2, float eps,
              float bc1, float bc2) {
  return run([&] { adamw_step<float>(p, g, m, v, n, lr, wd, b1, b2, eps, bc1, bc2); });
}
int ref_adam(float* p, const float* g, float* m, float* v, int n, float lr, float b1, float b2, float eps, float bc1,
             float bc2) {
  return run([&] { adam_step<float>(p, g, m, v, n, lr, b1, b2, eps, bc1, bc2); });
}
int ref_sgd(float* p, const float* g, float* vel, int n, float lr, float momentum, float wd) {
  return run([&] { sgd_step<float>(p, g, vel, n, lr, momentum, wd); });
}
}
