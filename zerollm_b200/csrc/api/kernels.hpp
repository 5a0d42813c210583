// kernels.hpp -- the reference's Kernel API (src/kernel/cuda/*.cuh) over the
// B200 C ABI.  Same function names, template signatures and default stream
// argument; instantiated for float, and for __nv_bfloat16 where the reference's
// template is generic (linear, mha, layernorm, softmax, add, relu, adamw: the bf16
// GEMMs and attention run on the tcgen05 kernels).  Error behaviour follows the reference
// (src/config.hpp:55-66 and the per-op checks cited below): CUDA failures
// throw std::runtime_error, invalid sizes throw std::invalid_argument, and
// the ops the reference lets return silently on size <= 0 do the same.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "zerollm_b200.h"

namespace zerollm_b200_detail {
inline void raise(zl_status s, const char* what) {
  if (s == ZL_OK) return;
  std::string msg = std::string(what) + ": " + zl_last_error();
  if (s == ZL_EINVAL) throw std::invalid_argument(msg);
  throw std::runtime_error("[CUDA ERROR] " + msg);
}
template <typename T>
inline void only_float() {
  static_assert(std::is_same<T, float>::value, "the reference kernel API is instantiated for float");
}
template <typename T>
inline constexpr bool is_bf16() {
  static_assert(std::is_same<T, float>::value || std::is_same<T, __nv_bfloat16>::value,
                "instantiated for float and __nv_bfloat16");
  return std::is_same<T, __nv_bfloat16>::value;
}
inline const zl_bf16* zb(const void* p) { return static_cast<const zl_bf16*>(p); }
inline zl_bf16* zb(void* p) { return static_cast<zl_bf16*>(p); }
inline const float* zf(const void* p) { return static_cast<const float*>(p); }
inline float* zf(void* p) { return static_cast<float*>(p); }
template <typename T>
inline float to_float(T x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(x);
  else return static_cast<float>(x);
}
}  // namespace zerollm_b200_detail
namespace zd = zerollm_b200_detail;

#define ZLB_CALL(expr, what) zerollm_b200_detail::raise((expr), (what))

// ----------------------------------------------------------------- matmul.cuh:20-99
template <typename T>
void matmul(const T* A, const T* B, T* C, int M, int N, int K, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_matmul_f32(A, B, C, M, N, K, stream), "matmul");
}
template <typename T>
void matmul_tiled(const T* A, const T* B, T* C, int M, int N, int K, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_matmul_f32(A, B, C, M, N, K, stream), "matmul_tiled");
}
template <typename T>
void matmul_transposed_A_T_B(const T* A, const T* B, T* C, int M, int N, int K, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_matmul_at_b_f32(A, B, C, M, N, K, stream), "matmul_transposed_A_T_B");
}
template <typename T>
void matmul_transposed_tiled_A_T_B(const T* A, const T* B, T* C, int M, int N, int K, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_matmul_at_b_f32(A, B, C, M, N, K, stream), "matmul_transposed_tiled_A_T_B");
}
template <typename T>
void matmul_transposed_A_B_T(const T* A, const T* B, T* C, int M, int N, int K, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_matmul_a_bt_f32(A, B, C, M, N, K, stream), "matmul_transposed_A_B_T");
}
template <typename T>
void matmul_transposed_tiled_A_B_T(const T* A, const T* B, T* C, int M, int N, int K, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_matmul_a_bt_f32(A, B, C, M, N, K, stream), "matmul_transposed_tiled_A_B_T");
}

// ----------------------------------------------------------------- linear.cuh:21-59
template <typename T>
void linear_forward(const T* input, const T* weight, const T* bias, T* output, int64_t M, int64_t K, int64_t N,
                    bool use_bias, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>())
    ZLB_CALL(zl_linear_forward_bf16(zd::zb(input), zd::zb(weight), zd::zb(bias), zd::zb(output), M, K, N, use_bias,
                                    stream),
             "linear_forward");
  else
    ZLB_CALL(zl_linear_forward_f32(input, weight, bias, output, M, K, N, use_bias, stream), "linear_forward");
}
template <typename T>
void linear_backward(const T* d_output, const T* input, const T* weight, T* d_input, T* d_weight, T* d_bias,
                     int64_t M, int64_t K, int64_t N, bool use_bias, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>())
    ZLB_CALL(zl_linear_backward_bf16(zd::zb(d_output), zd::zb(input), zd::zb(weight), zd::zb(d_input),
                                     zd::zb(d_weight), zd::zb(d_bias), M, K, N, use_bias, stream),
             "linear_backward");
  else
    ZLB_CALL(zl_linear_backward_f32(d_output, input, weight, d_input, d_weight, d_bias, M, K, N, use_bias, stream),
             "linear_backward");
}

// ----------------------------------------------------------------- mha.cuh:18-48
// The reference backward omits 1/sqrt(head_dim) in dQ/dK (mha.cu:284-295); this drop-in keeps that
// behaviour so results match the reference.  mha_backward_scaled gives the true gradient.
// For __nv_bfloat16 the tcgen05 flash-attention kernels run: causal, no mask, head_dim 64 or 128,
// seq_len a multiple of 128.  attention_scores (B*H*S*S elements, as in the reference) then holds the
// flash-attention state -- row log-sum-exps and a copy of attn_output -- instead of probabilities,
// and mha_backward reads it back (and uses the rest of it as scratch); it is large enough when
// seq_len >= 3 * head_dim + 6.
template <typename T>
void mha_forward(const T* Q, const T* K, const T* V, T* attn_output, T* attention_scores, const bool* mask,
                 int64_t batch_size, int64_t seq_len, int64_t num_heads, int64_t head_dim, bool is_causal,
                 cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) {
    ZLB_CALL(zl_mha_forward_bf16(zd::zb(Q), zd::zb(K), zd::zb(V), zd::zb(attn_output), attention_scores,
                                 (size_t)(batch_size * num_heads * seq_len * seq_len) * sizeof(T),
                                 reinterpret_cast<const uint8_t*>(mask), batch_size, seq_len, num_heads, head_dim,
                                 is_causal, stream),
             "mha_forward");
  } else {
    ZLB_CALL(zl_mha_forward_f32(Q, K, V, attn_output, attention_scores, reinterpret_cast<const uint8_t*>(mask),
                                batch_size, seq_len, num_heads, head_dim, is_causal, stream),
             "mha_forward");
  }
}
template <typename T>
void mha_backward(const T* d_attn_output, const T* Q, const T* K, const T* V, const T* attention_scores,
                  const bool* mask, T* d_Q, T* d_K, T* d_V, int64_t batch_size, int64_t seq_len, int64_t num_heads,
                  int64_t head_dim, bool is_causal, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) {
    ZLB_CALL(zl_mha_backward_bf16(zd::zb(d_attn_output), zd::zb(Q), zd::zb(K), zd::zb(V),
                                  const_cast<T*>(attention_scores),
                                  (size_t)(batch_size * num_heads * seq_len * seq_len) * sizeof(T),
                                  reinterpret_cast<const uint8_t*>(mask), zd::zb(d_Q), zd::zb(d_K), zd::zb(d_V),
                                  batch_size, seq_len, num_heads, head_dim, is_causal, 1, stream),
             "cuda_mha_backward");
  } else {
    ZLB_CALL(zl_mha_backward_f32(d_attn_output, Q, K, V, attention_scores, reinterpret_cast<const uint8_t*>(mask), d_Q,
                                 d_K, d_V, batch_size, seq_len, num_heads, head_dim, is_causal, 1, stream),
             "cuda_mha_backward");
  }
}
template <typename T>
void mha_backward_scaled(const T* d_attn_output, const T* Q, const T* K, const T* V, const T* attention_scores,
                         const bool* mask, T* d_Q, T* d_K, T* d_V, int64_t batch_size, int64_t seq_len,
                         int64_t num_heads, int64_t head_dim, bool is_causal, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) {
    ZLB_CALL(zl_mha_backward_bf16(zd::zb(d_attn_output), zd::zb(Q), zd::zb(K), zd::zb(V),
                                  const_cast<T*>(attention_scores),
                                  (size_t)(batch_size * num_heads * seq_len * seq_len) * sizeof(T),
                                  reinterpret_cast<const uint8_t*>(mask), zd::zb(d_Q), zd::zb(d_K), zd::zb(d_V),
                                  batch_size, seq_len, num_heads, head_dim, is_causal, 0, stream),
             "mha_backward_scaled");
  } else {
    ZLB_CALL(zl_mha_backward_f32(d_attn_output, Q, K, V, attention_scores, reinterpret_cast<const uint8_t*>(mask), d_Q,
                                 d_K, d_V, batch_size, seq_len, num_heads, head_dim, is_causal, 0, stream),
             "mha_backward_scaled");
  }
}

// ----------------------------------------------------------------- layernorm.cuh:22-61
template <typename T>
void cuda_layernorm_forward(const T* input, const T* gamma, const T* beta, T* output, T* mean, T* rstd, int64_t M,
                            int64_t N, T eps, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) {
    ZLB_CALL(zl_layernorm_forward_bf16(zd::zb(input), zd::zb(gamma), zd::zb(beta), zd::zb(output), zd::zb(mean),
                                       zd::zb(rstd), M, N, zd::to_float(eps), stream),
             "layernorm_forward_kernel launch failed");
  } else {
    ZLB_CALL(zl_layernorm_forward_f32(input, gamma, beta, output, mean, rstd, M, N, eps, stream),
             "layernorm_forward_kernel launch failed");
  }
}
template <typename T>
void cuda_layernorm_backward(const T* input, const T* d_output, const T* gamma, const T* mean, const T* rstd,
                             T* d_input, T* d_gamma, T* d_beta, int64_t M, int64_t N, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) {
    ZLB_CALL(zl_layernorm_backward_bf16(zd::zb(input), zd::zb(d_output), zd::zb(gamma), zd::zb(mean), zd::zb(rstd),
                                        zd::zb(d_input), zd::zb(d_gamma), zd::zb(d_beta), M, N, stream),
             "layernorm_backward_kernel launch failed");
  } else {
    ZLB_CALL(zl_layernorm_backward_f32(input, d_output, gamma, mean, rstd, d_input, d_gamma, d_beta, M, N, stream),
             "layernorm_backward_kernel launch failed");
  }
}

// ----------------------------------------------------------------- softmax.cuh, cross_entropy.cuh
template <typename T>
void softmax(const T* input, T* output, int M, int N, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) ZLB_CALL(zl_softmax_bf16(zd::zb(input), zd::zb(output), M, N, stream), "softmax");
  else ZLB_CALL(zl_softmax_f32(input, output, M, N, stream), "softmax");
}
inline void cross_entropy_backward_kernel(float* d_logits, const float* softmax_output, const int* targets,
                                          int batch_size, int num_classes, cudaStream_t stream = 0) {
  ZLB_CALL(zl_cross_entropy_backward_f32(d_logits, softmax_output, targets, batch_size, num_classes, stream),
           "cross_entropy_backward_kernel failed");
}

// ----------------------------------------------------------------- embedding.cuh:23-57
template <typename T, typename IdxType>
void cuda_embedding_forward(const IdxType* input, const T* embedding_table, const T* pos_encoding_table, T* output,
                            int batch_size, int seq_len, int embed_dim, int vocab_size, int max_seq_len,
                            cudaStream_t stream = 0) {
  static_assert(std::is_same<T, float>::value && std::is_same<IdxType, int>::value, "instantiated for <float,int>");
  ZLB_CALL(zl_embedding_forward_f32(input, embedding_table, pos_encoding_table, output, batch_size, seq_len, embed_dim,
                                    vocab_size, max_seq_len, stream),
           "embedding_forward_kernel launch failed");
}
template <typename T, typename IdxType>
void cuda_embedding_backward(const IdxType* input, const T* d_output, T* d_embedding_table, int batch_size,
                             int seq_len, int embed_dim, int vocab_size, cudaStream_t stream = 0) {
  static_assert(std::is_same<T, float>::value && std::is_same<IdxType, int>::value, "instantiated for <float,int>");
  ZLB_CALL(zl_embedding_backward_f32(input, d_output, d_embedding_table, batch_size, seq_len, embed_dim, vocab_size,
                                     stream),
           "embedding_backward_kernel launch failed");
}

// ----------------------------------------------------------------- add.cuh, relu.cuh, transpose.cuh
template <typename T>
void add(const T* a, const T* b, T* output, int size, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) ZLB_CALL(zl_add_bf16(zd::zb(a), zd::zb(b), zd::zb(output), size, stream), "add");
  else ZLB_CALL(zl_add_f32(a, b, output, size, stream), "add");
}
template <typename T>
void add_inplace(T* a, const T* b, int size, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) ZLB_CALL(zl_add_inplace_bf16(zd::zb(a), zd::zb(b), size, stream), "add_inplace");
  else ZLB_CALL(zl_add_inplace_f32(a, b, size, stream), "add_inplace");
}
template <typename T>
void relu_forward(const T* input, T* output, int size, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>())
    ZLB_CALL(zl_relu_forward_bf16(zd::zb(input), zd::zb(output), size, stream),
             "CUDA kernel launch error in relu_forward()");
  else ZLB_CALL(zl_relu_forward_f32(input, output, size, stream), "CUDA kernel launch error in relu_forward()");
}
template <typename T>
void relu_backward(const T* input, const T* grad_output, T* grad_input, int size, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>())
    ZLB_CALL(zl_relu_backward_bf16(zd::zb(input), zd::zb(grad_output), zd::zb(grad_input), size, stream),
             "CUDA kernel launch error in relu_backward()");
  else
    ZLB_CALL(zl_relu_backward_f32(input, grad_output, grad_input, size, stream),
             "CUDA kernel launch error in relu_backward()");
}
template <typename T>
void transpose(const T* input, T* output, int rows, int cols, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_transpose_f32(input, output, rows, cols, stream), "CUDA kernel launch error in transpose()");
}

// ----------------------------------------------------------------- adamw.cuh, adam.cuh, sgd.cuh
template <typename T>
void adamw_step(T* params, const T* grads, T* m, T* v, int size, float learning_rate, float weight_decay, float beta1,
                float beta2, float eps, float bias_correction1, float bias_correction2, cudaStream_t stream = 0) {
  if constexpr (zd::is_bf16<T>()) {
    ZLB_CALL(zl_adamw_step_bf16(zd::zb(params), zd::zb(grads), zd::zb(m), zd::zb(v), size, learning_rate,
                                weight_decay, beta1, beta2, eps, bias_correction1, bias_correction2, stream),
             "adamw_step");
  } else {
    ZLB_CALL(zl_adamw_step_f32(params, grads, m, v, size, learning_rate, weight_decay, beta1, beta2, eps,
                               bias_correction1, bias_correction2, stream),
             "adamw_step");
  }
}
template <typename T>
void adam_step(T* params, const T* grads, T* m, T* v, int size, float learning_rate, float beta1, float beta2,
               float eps, float bias_correction1, float bias_correction2, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_adam_step_f32(params, grads, m, v, size, learning_rate, beta1, beta2, eps, bias_correction1,
                            bias_correction2, stream),
           "adam_step");
}
template <typename T>
void sgd_step(T* params, const T* grads, T* velocity, int size, float learning_rate, float momentum,
              float weight_decay, cudaStream_t stream = 0) {
  zerollm_b200_detail::only_float<T>();
  ZLB_CALL(zl_sgd_step_f32(params, grads, velocity, size, learning_rate, momentum, weight_decay, stream), "sgd_step");
}
