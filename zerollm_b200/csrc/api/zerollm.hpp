// zerollm.hpp -- the reference's Layer -> Model / Loss / Optimizer /
// Distributed C++ API over the B200 C ABI (header-only).
//
// Class and method names follow buladuo/ZeroLLM:
//   src/layer/module.hpp:22-146        Parameter, Module
//   src/optimizer/optimizer.hpp:28-117 Optimizer, OptimizerType, OptimizerConfig; sgd/adam/adamw.hpp
//   src/loss/loss.hpp, cross_entropy.hpp  Loss, CrossEntropyLoss
//   src/layer/{linear,layernorm,relu,embedding,mha,feedward,transformer_block,transformer_decoder}.hpp
//   src/model/zerollm_config.hpp, zerollm.hpp  ZeroLLMConfig (+ factories), ZeroLLM
//   src/distributed/{dist_types,abstract_backend,gpu_backend,dist_factory}.hpp
//
// The standalone layers are fp32 and run the fp32 kernel API (tf32 tensor
// cores for the GEMMs); they own their parameters like the reference's
// layers but never synchronise the device per call and never alias a saved
// input with an in-place output.  ZeroLLM is the fused bf16 training step
// over one arena (zl_model_*): its forward/backward/step keep the reference
// signatures and it adds train_step().
#pragma once
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <fstream>
#include <map>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "kernels.hpp"
#include "zerollm_b200.h"

namespace zerollm_b200_detail {
inline float* dmalloc(size_t n) {
  void* p = nullptr;
  if (n && cudaMalloc(&p, n * sizeof(float)) != cudaSuccess) throw std::runtime_error("[CUDA ERROR] cudaMalloc failed");
  return static_cast<float*>(p);
}
inline void dfree(void* p) {
  if (p) cudaFree(p);
}
inline void upload(float* d, const std::vector<float>& h) {
  if (cudaMemcpy(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
    throw std::runtime_error("[CUDA ERROR] H2D copy failed");
}
// Xavier-uniform init of a [out, in] weight (linear.cpp:68-88), from a seeded engine.
inline std::vector<float> xavier(int out, int in, std::mt19937& gen) {
  const float a = std::sqrt(6.0f / (float)(in + out));
  std::uniform_real_distribution<float> u(-a, a);
  std::vector<float> w((size_t)out * in);
  for (auto& x : w) x = u(gen);
  return w;
}
inline std::mt19937& rng() {
  static std::mt19937 g(0);
  return g;
}
}  // namespace zerollm_b200_detail

// =================================================================== module.hpp
struct Parameter {
  std::string name;
  float* data;
  float* grad;
  size_t size;
  bool requires_grad;
  Parameter(std::string n, float* d, float* g, size_t s, bool req)
      : name(std::move(n)), data(d), grad(g), size(s), requires_grad(req) {}
};

class Module {
 protected:
  std::string name_;
  std::map<std::string, Module*> sub_modules_;
  std::vector<Parameter> params_;

 public:
  explicit Module(std::string name = "") : name_(std::move(name)) {}
  virtual ~Module() = default;
  virtual std::string type_name() const { return "Module"; }
  void register_parameter(std::string name, float* data, float* grad, size_t size, bool requires_grad = true) {
    params_.emplace_back(std::move(name), data, grad, size, requires_grad);
  }
  void register_module(std::string name, Module* m) {
    if (m) sub_modules_[std::move(name)] = m;
  }
  void get_parameters(std::vector<Parameter>& out, const std::string& prefix = "") {
    for (auto& p : params_) {
      Parameter q = p;
      q.name = (prefix.empty() ? "" : prefix + ".") + p.name;
      out.push_back(q);
    }
    for (auto& kv : sub_modules_) kv.second->get_parameters(out, (prefix.empty() ? "" : prefix + ".") + kv.first);
  }
  void print_structure(const std::string& indent = "") const {
    std::printf("%s%s (%s)\n", indent.c_str(), name_.empty() ? "Root" : name_.c_str(), type_name().c_str());
    for (auto& p : params_) std::printf("%s  %s [Size: %zu]\n", indent.c_str(), p.name.c_str(), p.size);
    for (auto& kv : sub_modules_) {
      std::printf("%s  %s\n", indent.c_str(), kv.first.c_str());
      kv.second->print_structure(indent + "    ");
    }
  }
};

// =================================================================== optimizer.hpp
class Optimizer {
 public:
  virtual ~Optimizer() = default;
  virtual void step(float* param, const float* grad, int num_elements, float learning_rate) = 0;
  virtual void zero_grad() {}
};

enum class OptimizerType { SGD, Adam, AdamW };

struct OptimizerConfig {
  OptimizerType type = OptimizerType::SGD;
  float momentum = 0.0f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.0f;
  static OptimizerConfig createSGD(float momentum = 0.0f) {
    OptimizerConfig c;
    c.type = OptimizerType::SGD;
    c.momentum = momentum;
    return c;
  }
  static OptimizerConfig createAdam(float beta1 = 0.9f, float beta2 = 0.999f, float eps = 1e-8f) {
    OptimizerConfig c;
    c.type = OptimizerType::Adam;
    c.beta1 = beta1;
    c.beta2 = beta2;
    c.eps = eps;
    return c;
  }
  static OptimizerConfig createAdamW(float weight_decay, float beta1 = 0.9f, float beta2 = 0.999f,
                                     float eps = 1e-8f) {
    OptimizerConfig c;
    c.type = OptimizerType::AdamW;
    c.weight_decay = weight_decay;
    c.beta1 = beta1;
    c.beta2 = beta2;
    c.eps = eps;
    return c;
  }
};

// sgd.cpp:21-44 (weight decay is passed as 0 there as well)
class SGD : public Optimizer {
  float momentum_;
  float* velocity_ = nullptr;
  int n_ = 0;

 public:
  explicit SGD(float momentum = 0.0f) : momentum_(momentum) {}
  ~SGD() override { zerollm_b200_detail::dfree(velocity_); }
  void step(float* p, const float* g, int n, float lr) override {
    if (n <= 0) throw std::invalid_argument("Number of elements must be positive");
    if (momentum_ != 0.0f && n != n_) {
      zerollm_b200_detail::dfree(velocity_);
      velocity_ = zerollm_b200_detail::dmalloc(n);
      cudaMemset(velocity_, 0, n * sizeof(float));
      n_ = n;
    }
    sgd_step<float>(p, g, momentum_ != 0.0f ? velocity_ : nullptr, n, lr, momentum_, 0.0f);
  }
};

// adam.cpp:26-63 / adamw.cpp:12-53: moments allocated at the first step, host powf bias corrections
class Adam : public Optimizer {
 protected:
  float beta1_, beta2_, eps_;
  float *m_ = nullptr, *v_ = nullptr;
  int n_ = 0, t_ = 0;
  void ensure(int n) {
    if (n != n_) {
      zerollm_b200_detail::dfree(m_);
      zerollm_b200_detail::dfree(v_);
      m_ = zerollm_b200_detail::dmalloc(n);
      v_ = zerollm_b200_detail::dmalloc(n);
      cudaMemset(m_, 0, n * sizeof(float));
      cudaMemset(v_, 0, n * sizeof(float));
      n_ = n;
    }
  }

 public:
  Adam(float beta1 = 0.9f, float beta2 = 0.999f, float eps = 1e-8f) : beta1_(beta1), beta2_(beta2), eps_(eps) {}
  ~Adam() override {
    zerollm_b200_detail::dfree(m_);
    zerollm_b200_detail::dfree(v_);
  }
  void step(float* p, const float* g, int n, float lr) override {
    if (n <= 0) throw std::invalid_argument("Number of elements must be positive");
    ensure(n);
    ++t_;
    adam_step<float>(p, g, m_, v_, n, lr, beta1_, beta2_, eps_, 1.0f - powf(beta1_, (float)t_),
                     1.0f - powf(beta2_, (float)t_));
  }
};
class AdamW : public Adam {
  float weight_decay_;

 public:
  AdamW(float weight_decay = 0.01f, float beta1 = 0.9f, float beta2 = 0.999f, float eps = 1e-8f)
      : Adam(beta1, beta2, eps), weight_decay_(weight_decay) {}
  void step(float* p, const float* g, int n, float lr) override {
    if (n <= 0) throw std::invalid_argument("Number of elements must be positive");
    ensure(n);
    ++t_;
    adamw_step<float>(p, g, m_, v_, n, lr, weight_decay_, beta1_, beta2_, eps_, 1.0f - powf(beta1_, (float)t_),
                      1.0f - powf(beta2_, (float)t_));
  }
};
inline std::unique_ptr<Optimizer> make_optimizer(const OptimizerConfig& c) {
  switch (c.type) {
    case OptimizerType::SGD: return std::make_unique<SGD>(c.momentum);
    case OptimizerType::Adam: return std::make_unique<Adam>(c.beta1, c.beta2, c.eps);
    default: return std::make_unique<AdamW>(c.weight_decay, c.beta1, c.beta2, c.eps);
  }
}

// =================================================================== loss.hpp, cross_entropy.hpp
class Loss {
 public:
  virtual ~Loss() = default;
  virtual float forward(const float* logits, const int* targets, int batch_size, int num_classes) = 0;
  virtual void backward(float* d_logits, const float* logits, const int* targets, int batch_size,
                        int num_classes) = 0;
};

// cross_entropy.cpp:23-94 without the host round trip: softmax and the clamped NLL
// mean are computed on the device; only the 4-byte loss is read back.
class CrossEntropyLoss : public Loss {
  float* softmax_output_ = nullptr;
  float* loss_dev_ = nullptr;
  int rows_ = 0, classes_ = 0;
  float eps_;

 public:
  explicit CrossEntropyLoss(float eps = 1e-8f) : eps_(eps) {}
  ~CrossEntropyLoss() override {
    zerollm_b200_detail::dfree(softmax_output_);
    zerollm_b200_detail::dfree(loss_dev_);
  }
  float forward(const float* logits, const int* targets, int batch_size, int num_classes) override {
    if (batch_size <= 0 || num_classes <= 0)
      throw std::invalid_argument("Batch size and number of classes must be positive");
    if (batch_size != rows_ || num_classes != classes_) {
      zerollm_b200_detail::dfree(softmax_output_);
      softmax_output_ = zerollm_b200_detail::dmalloc((size_t)batch_size * num_classes);
      rows_ = batch_size;
      classes_ = num_classes;
    }
    if (!loss_dev_) loss_dev_ = zerollm_b200_detail::dmalloc(1);
    softmax<float>(logits, softmax_output_, batch_size, num_classes);
    ZLB_CALL(zl_cross_entropy_forward_f32(softmax_output_, targets, batch_size, num_classes, eps_, loss_dev_, nullptr),
             "CrossEntropyLoss::forward");
    float h = 0.f;
    cudaMemcpy(&h, loss_dev_, sizeof(float), cudaMemcpyDeviceToHost);
    return h;
  }
  void backward(float* d_logits, const float*, const int* targets, int batch_size, int num_classes) override {
    if (!softmax_output_) throw std::runtime_error("Must call forward() before backward()");
    cross_entropy_backward_kernel(d_logits, softmax_output_, targets, batch_size, num_classes);
  }
};

// =================================================================== layers (fp32)
class Linear : public Module {
  int in_, out_;
  bool use_bias_, with_grad_;
  float *w_, *b_ = nullptr, *dw_ = nullptr, *db_ = nullptr;
  const float* input_ = nullptr;
  int last_batch_ = 0;
  std::unique_ptr<Optimizer> opt_w_, opt_b_;

 public:
  Linear(int in_features, int out_features, bool use_bias = true, bool with_grad = false)
      : Module("Linear"), in_(in_features), out_(out_features), use_bias_(use_bias), with_grad_(with_grad) {
    w_ = zerollm_b200_detail::dmalloc((size_t)in_ * out_);
    zerollm_b200_detail::upload(w_, zerollm_b200_detail::xavier(out_, in_, zerollm_b200_detail::rng()));
    if (use_bias_) {
      b_ = zerollm_b200_detail::dmalloc(out_);
      cudaMemset(b_, 0, out_ * sizeof(float));
    }
    if (with_grad_) {
      dw_ = zerollm_b200_detail::dmalloc((size_t)in_ * out_);
      if (use_bias_) db_ = zerollm_b200_detail::dmalloc(out_);
      zero_grad();
    }
    register_parameter("weight", w_, dw_, (size_t)in_ * out_, with_grad_);
    if (use_bias_) register_parameter("bias", b_, db_, out_, with_grad_);
  }
  ~Linear() override {
    for (float* p : {w_, b_, dw_, db_}) zerollm_b200_detail::dfree(p);
  }
  std::string type_name() const override { return "Linear"; }
  void zero_grad() {
    if (dw_) cudaMemsetAsync(dw_, 0, (size_t)in_ * out_ * sizeof(float));
    if (db_) cudaMemsetAsync(db_, 0, out_ * sizeof(float));
  }
  void forward(float* output, const float* input, int batch_size) {
    if (with_grad_) {
      input_ = input;
      last_batch_ = batch_size;
    }
    linear_forward<float>(input, w_, b_, output, batch_size, in_, out_, use_bias_);
  }
  void backward(float* d_input, const float* d_output) {
    if (!with_grad_) throw std::runtime_error("Cannot call backward() when with_grad=false");
    if (!input_) throw std::runtime_error("Must call forward() before backward()");
    linear_backward<float>(d_output, input_, w_, d_input, dw_, db_, last_batch_, in_, out_, use_bias_);
  }
  void set_optimizer(OptimizerConfig c) {
    opt_w_ = make_optimizer(c);
    if (use_bias_) opt_b_ = make_optimizer(c);
  }
  void step(float lr) {
    if (opt_w_) opt_w_->step(w_, dw_, in_ * out_, lr);
    if (opt_b_) opt_b_->step(b_, db_, out_, lr);
  }
  float* weight() { return w_; }
  float* bias() { return b_; }
  float* d_weight() { return dw_; }
  float* d_bias() { return db_; }
};

class LayerNorm : public Module {
  int n_;
  bool with_grad_;
  float eps_;
  float *g_, *b_, *dg_ = nullptr, *db_ = nullptr;
  float *mean_ = nullptr, *rstd_ = nullptr, *saved_ = nullptr;
  const float* input_ = nullptr;
  int rows_ = 0, cap_ = 0;
  std::unique_ptr<Optimizer> opt_g_, opt_b_;

 public:
  LayerNorm(int feature_size, bool with_grad = false, float eps = 1e-5f)
      : Module("LayerNorm"), n_(feature_size), with_grad_(with_grad), eps_(eps) {
    g_ = zerollm_b200_detail::dmalloc(n_);
    b_ = zerollm_b200_detail::dmalloc(n_);
    zerollm_b200_detail::upload(g_, std::vector<float>(n_, 1.0f));
    cudaMemset(b_, 0, n_ * sizeof(float));
    if (with_grad_) {
      dg_ = zerollm_b200_detail::dmalloc(n_);
      db_ = zerollm_b200_detail::dmalloc(n_);
      zero_grad();
    }
    register_parameter("gamma", g_, dg_, n_, with_grad_);
    register_parameter("beta", b_, db_, n_, with_grad_);
  }
  ~LayerNorm() override {
    for (float* p : {g_, b_, dg_, db_, mean_, rstd_, saved_}) zerollm_b200_detail::dfree(p);
  }
  std::string type_name() const override { return "LayerNorm"; }
  void zero_grad() {
    if (dg_) cudaMemsetAsync(dg_, 0, n_ * sizeof(float));
    if (db_) cudaMemsetAsync(db_, 0, n_ * sizeof(float));
  }
  // In-place calls (output == input) keep a private copy of the input for backward.
  void forward(float* output, const float* input, int batch_size) {
    float *mean = nullptr, *rstd = nullptr;
    if (with_grad_) {
      if (batch_size > cap_) {
        for (float* p : {mean_, rstd_, saved_}) zerollm_b200_detail::dfree(p);
        mean_ = zerollm_b200_detail::dmalloc(batch_size);
        rstd_ = zerollm_b200_detail::dmalloc(batch_size);
        saved_ = zerollm_b200_detail::dmalloc((size_t)batch_size * n_);
        cap_ = batch_size;
      }
      input_ = input;
      if (output == input) {
        cudaMemcpyAsync(saved_, input, (size_t)batch_size * n_ * sizeof(float), cudaMemcpyDeviceToDevice);
        input_ = saved_;
      }
      rows_ = batch_size;
      mean = mean_;
      rstd = rstd_;
    }
    cuda_layernorm_forward<float>(input, g_, b_, output, mean, rstd, batch_size, n_, eps_);
  }
  void backward(float* d_input, const float* d_output) {
    if (!with_grad_) throw std::runtime_error("Cannot call backward() when with_grad=false");
    if (!input_) throw std::runtime_error("Must call forward() before backward()");
    cuda_layernorm_backward<float>(input_, d_output, g_, mean_, rstd_, d_input, dg_, db_, rows_, n_);
  }
  void set_optimizer(OptimizerConfig c) {
    opt_g_ = make_optimizer(c);
    opt_b_ = make_optimizer(c);
  }
  void step(float lr) {
    if (opt_g_) opt_g_->step(g_, dg_, n_, lr);
    if (opt_b_) opt_b_->step(b_, db_, n_, lr);
  }
};

class ReLU : public Module {
  const float* input_ = nullptr;
  int size_ = 0;

 public:
  ReLU() : Module("ReLU") {}
  std::string type_name() const override { return "ReLU"; }
  void forward(float* output, const float* input, int batch_size, int features) {
    input_ = input;
    size_ = batch_size * features;
    relu_forward<float>(input, output, size_);
  }
  void backward(float* d_input, const float* d_output) { relu_backward<float>(input_, d_output, d_input, size_); }
};

// embedding.cpp: token table + fixed sinusoid position table (embedding.cpp:107-126)
class Embedding : public Module {
  int V_, D_, max_seq_;
  bool with_grad_;
  float *table_, *pos_, *dtable_ = nullptr;
  std::unique_ptr<Optimizer> opt_;

 public:
  Embedding(int vocab_size, int embed_dim, int max_seq_len, bool with_grad = false)
      : Module("Embedding"), V_(vocab_size), D_(embed_dim), max_seq_(max_seq_len), with_grad_(with_grad) {
    table_ = zerollm_b200_detail::dmalloc((size_t)V_ * D_);
    std::uniform_real_distribution<float> u(-0.01f, 0.01f);  // embedding.cpp:90-98 range
    std::vector<float> h((size_t)V_ * D_);
    for (auto& x : h) x = u(zerollm_b200_detail::rng());
    zerollm_b200_detail::upload(table_, h);
    std::vector<float> p((size_t)max_seq_ * D_);
    for (int s = 0; s < max_seq_; ++s)
      for (int i = 0; i < D_; ++i) {
        const float ang = (float)s / powf(10000.0f, (float)(2 * (i / 2)) / (float)D_);
        p[(size_t)s * D_ + i] = (i % 2 == 0) ? sinf(ang) : cosf(ang);
      }
    pos_ = zerollm_b200_detail::dmalloc(p.size());
    zerollm_b200_detail::upload(pos_, p);
    if (with_grad_) {
      dtable_ = zerollm_b200_detail::dmalloc((size_t)V_ * D_);
      zero_grad();
    }
    register_parameter("embedding_table", table_, dtable_, (size_t)V_ * D_, with_grad_);
    register_parameter("pos_encoding_table", pos_, nullptr, (size_t)max_seq_ * D_, false);
  }
  ~Embedding() override {
    for (float* p : {table_, pos_, dtable_}) zerollm_b200_detail::dfree(p);
  }
  std::string type_name() const override { return "Embedding"; }
  void zero_grad() {
    if (dtable_) cudaMemsetAsync(dtable_, 0, (size_t)V_ * D_ * sizeof(float));
  }
  void forward(float* output, const int* input, int batch_size, int seq_len) {
    cuda_embedding_forward<float, int>(input, table_, pos_, output, batch_size, seq_len, D_, V_, max_seq_);
  }
  void backward(const int* input, const float* d_output, int batch_size, int seq_len, bool accumulate = false) {
    if (!with_grad_) return;
    if (!accumulate) zero_grad();
    cuda_embedding_backward<float, int>(input, d_output, dtable_, batch_size, seq_len, D_, V_);
  }
  void set_optimizer(OptimizerConfig c) { opt_ = make_optimizer(c); }
  void step(float lr) {
    if (opt_) opt_->step(table_, dtable_, V_ * D_, lr);
  }
  const float* embedding_table_device() const { return table_; }
  float* d_embedding_table() { return dtable_; }
};

// mha.cpp: q/k/v/out projections + causal attention with stored probabilities (reference semantics,
// including the unscaled dQ/dK of mha.cu:284-295 unless scaled_backward is set)
class MultiHeadAttention : public Module {
  int E_, H_;
  bool causal_, with_grad_;
  bool scaled_backward_ = false;
  Linear *q_, *k_, *v_, *o_;
  float *Q_ = nullptr, *K_ = nullptr, *V_ = nullptr, *A_ = nullptr, *P_ = nullptr;
  float *dA_ = nullptr, *dQ_ = nullptr, *dK_ = nullptr, *dV_ = nullptr, *tmp_ = nullptr;
  int B_ = 0, S_ = 0;

  void release() {
    for (float* p : {Q_, K_, V_, A_, P_, dA_, dQ_, dK_, dV_, tmp_}) zerollm_b200_detail::dfree(p);
    Q_ = K_ = V_ = A_ = P_ = dA_ = dQ_ = dK_ = dV_ = tmp_ = nullptr;
  }

 public:
  MultiHeadAttention(int embed_dim, int num_heads, bool is_causal = true, bool with_grad = false)
      : Module("MultiHeadAttention"), E_(embed_dim), H_(num_heads), causal_(is_causal), with_grad_(with_grad) {
    q_ = new Linear(E_, E_, true, with_grad);
    k_ = new Linear(E_, E_, true, with_grad);
    v_ = new Linear(E_, E_, true, with_grad);
    o_ = new Linear(E_, E_, true, with_grad);
    register_module("q_proj", q_);
    register_module("k_proj", k_);
    register_module("v_proj", v_);
    register_module("out_proj", o_);  // registered (the reference omits it, mha.cpp:44-46)
  }
  ~MultiHeadAttention() override {
    release();
    delete q_; delete k_; delete v_; delete o_;
  }
  std::string type_name() const override { return "MultiHeadAttention"; }
  void set_scaled_backward(bool on) { scaled_backward_ = on; }
  void zero_grad() { q_->zero_grad(); k_->zero_grad(); v_->zero_grad(); o_->zero_grad(); }
  void forward(float* output, const float* input, int batch_size, int seq_len) {
    if (batch_size != B_ || seq_len != S_) {
      release();
      const size_t n = (size_t)batch_size * seq_len * E_;
      Q_ = zerollm_b200_detail::dmalloc(n); K_ = zerollm_b200_detail::dmalloc(n);
      V_ = zerollm_b200_detail::dmalloc(n); A_ = zerollm_b200_detail::dmalloc(n);
      P_ = zerollm_b200_detail::dmalloc((size_t)batch_size * H_ * seq_len * seq_len);
      B_ = batch_size;
      S_ = seq_len;
    }
    const int T = batch_size * seq_len;
    q_->forward(Q_, input, T);
    k_->forward(K_, input, T);
    v_->forward(V_, input, T);
    mha_forward<float>(Q_, K_, V_, A_, P_, nullptr, B_, S_, H_, E_ / H_, causal_);
    o_->forward(output, A_, T);
  }
  void backward(float* d_input, const float* d_output) {
    if (!B_) throw std::runtime_error("Must call forward() before backward()");
    const size_t n = (size_t)B_ * S_ * E_;
    if (!dA_) {
      dA_ = zerollm_b200_detail::dmalloc(n); dQ_ = zerollm_b200_detail::dmalloc(n);
      dK_ = zerollm_b200_detail::dmalloc(n); dV_ = zerollm_b200_detail::dmalloc(n);
      tmp_ = zerollm_b200_detail::dmalloc(n);
    }
    o_->backward(dA_, d_output);
    if (scaled_backward_)
      mha_backward_scaled<float>(dA_, Q_, K_, V_, P_, nullptr, dQ_, dK_, dV_, B_, S_, H_, E_ / H_, causal_);
    else
      mha_backward<float>(dA_, Q_, K_, V_, P_, nullptr, dQ_, dK_, dV_, B_, S_, H_, E_ / H_, causal_);
    q_->backward(d_input, dQ_);
    k_->backward(tmp_, dK_);
    add_inplace<float>(d_input, tmp_, (int)n);
    v_->backward(tmp_, dV_);
    add_inplace<float>(d_input, tmp_, (int)n);
  }
  void set_optimizer(OptimizerConfig c) { q_->set_optimizer(c); k_->set_optimizer(c); v_->set_optimizer(c); o_->set_optimizer(c); }
  void step(float lr) { q_->step(lr); k_->step(lr); v_->step(lr); o_->step(lr); }
};

class FeedForward : public Module {
  int E_, F_;
  Linear *ff1_, *ff2_;
  ReLU relu_;
  float *h1_ = nullptr, *h2_ = nullptr, *d2_ = nullptr, *d1_ = nullptr;
  int T_ = 0;

 public:
  FeedForward(int embed_dim, int ff_hidden_dim, bool with_grad = false)
      : Module("FeedForward"), E_(embed_dim), F_(ff_hidden_dim) {
    ff1_ = new Linear(E_, F_, true, with_grad);
    ff2_ = new Linear(F_, E_, true, with_grad);
    register_module("ff1", ff1_);
    register_module("ff2", ff2_);
  }
  ~FeedForward() override {
    for (float* p : {h1_, h2_, d2_, d1_}) zerollm_b200_detail::dfree(p);
    delete ff1_; delete ff2_;
  }
  std::string type_name() const override { return "FeedForward"; }
  void zero_grad() { ff1_->zero_grad(); ff2_->zero_grad(); }
  void forward(float* output, const float* input, int batch_size, int seq_len) {
    const int T = batch_size * seq_len;
    if (T != T_) {
      for (float* p : {h1_, h2_, d2_, d1_}) zerollm_b200_detail::dfree(p);
      h1_ = zerollm_b200_detail::dmalloc((size_t)T * F_); h2_ = zerollm_b200_detail::dmalloc((size_t)T * F_);
      d2_ = zerollm_b200_detail::dmalloc((size_t)T * F_); d1_ = zerollm_b200_detail::dmalloc((size_t)T * F_);
      T_ = T;
    }
    ff1_->forward(h1_, input, T);
    relu_.forward(h2_, h1_, T, F_);
    ff2_->forward(output, h2_, T);
  }
  void backward(float* d_input, const float* d_output) {
    ff2_->backward(d2_, d_output);
    relu_.backward(d1_, d2_);
    ff1_->backward(d_input, d1_);
  }
  void set_optimizer(OptimizerConfig c) { ff1_->set_optimizer(c); ff2_->set_optimizer(c); }
  void step(float lr) { ff1_->step(lr); ff2_->step(lr); }
};

// transformer_block.cpp:68-211 (post-norm), with private buffers so saved inputs never alias
class TransformerDecoderBlock : public Module {
  int E_;
  MultiHeadAttention* attn_;
  LayerNorm *ln1_, *ln2_;
  FeedForward* ff_;
  float *a_ = nullptr, *r1_ = nullptr, *h1_ = nullptr, *f_ = nullptr, *r2_ = nullptr;
  float *d1_ = nullptr, *d2_ = nullptr, *d3_ = nullptr;
  int B_ = 0, S_ = 0;

 public:
  TransformerDecoderBlock(int embed_dim, int num_heads, int ff_hidden_dim, bool with_grad = false)
      : Module("TransformerDecoderBlock"), E_(embed_dim) {
    attn_ = new MultiHeadAttention(E_, num_heads, true, with_grad);
    ln1_ = new LayerNorm(E_, with_grad, 1e-5f);
    ff_ = new FeedForward(E_, ff_hidden_dim, with_grad);
    ln2_ = new LayerNorm(E_, with_grad, 1e-5f);
    register_module("self_attn", attn_);
    register_module("ln1", ln1_);
    register_module("ff", ff_);
    register_module("ln2", ln2_);
  }
  ~TransformerDecoderBlock() override {
    for (float* p : {a_, r1_, h1_, f_, r2_, d1_, d2_, d3_}) zerollm_b200_detail::dfree(p);
    delete attn_; delete ln1_; delete ff_; delete ln2_;
  }
  std::string type_name() const override { return "TransformerDecoderBlock"; }
  void zero_grad() { attn_->zero_grad(); ln1_->zero_grad(); ff_->zero_grad(); ln2_->zero_grad(); }
  void forward(float* output, const float* input, int batch_size, int seq_len) {
    const size_t n = (size_t)batch_size * seq_len * E_;
    if (batch_size != B_ || seq_len != S_) {
      for (float* p : {a_, r1_, h1_, f_, r2_, d1_, d2_, d3_}) zerollm_b200_detail::dfree(p);
      a_ = zerollm_b200_detail::dmalloc(n); r1_ = zerollm_b200_detail::dmalloc(n); h1_ = zerollm_b200_detail::dmalloc(n);
      f_ = zerollm_b200_detail::dmalloc(n); r2_ = zerollm_b200_detail::dmalloc(n); d1_ = zerollm_b200_detail::dmalloc(n);
      d2_ = zerollm_b200_detail::dmalloc(n); d3_ = zerollm_b200_detail::dmalloc(n);
      B_ = batch_size;
      S_ = seq_len;
    }
    attn_->forward(a_, input, batch_size, seq_len);
    add<float>(input, a_, r1_, (int)n);
    ln1_->forward(h1_, r1_, batch_size * seq_len);
    ff_->forward(f_, h1_, batch_size, seq_len);
    add<float>(h1_, f_, r2_, (int)n);
    ln2_->forward(output, r2_, batch_size * seq_len);
  }
  void backward(float* d_input, const float* d_output) {
    const int n = B_ * S_ * E_;
    ln2_->backward(d1_, d_output);           // d r2
    ff_->backward(d2_, d1_);                 // d h1 from the FFN branch
    add_inplace<float>(d2_, d1_, n);         // + residual branch
    ln1_->backward(d3_, d2_);                // d r1
    attn_->backward(d_input, d3_);           // d x from attention
    add_inplace<float>(d_input, d3_, n);     // + residual branch
  }
  void set_optimizer(OptimizerConfig c) { attn_->set_optimizer(c); ln1_->set_optimizer(c); ff_->set_optimizer(c); ln2_->set_optimizer(c); }
  void step(float lr) { attn_->step(lr); ln1_->step(lr); ff_->step(lr); ln2_->step(lr); }
};

// transformer_decoder.cpp:57-141 with one output buffer per layer (no shared in-place buffer)
class TransformerDecoder : public Module {
  int E_;
  std::vector<TransformerDecoderBlock*> layers_;
  std::vector<float*> outs_;
  float *g0_ = nullptr, *g1_ = nullptr;
  int B_ = 0, S_ = 0;

 public:
  TransformerDecoder(int num_layers, int embed_dim, int num_heads, int ff_hidden_dim, bool with_grad = false)
      : Module("TransformerDecoder"), E_(embed_dim) {
    for (int i = 0; i < num_layers; ++i) {
      layers_.push_back(new TransformerDecoderBlock(E_, num_heads, ff_hidden_dim, with_grad));
      register_module("layer_" + std::to_string(i), layers_.back());
    }
  }
  ~TransformerDecoder() override {
    for (float* p : outs_) zerollm_b200_detail::dfree(p);
    zerollm_b200_detail::dfree(g0_);
    zerollm_b200_detail::dfree(g1_);
    for (auto* l : layers_) delete l;
  }
  std::string type_name() const override { return "TransformerDecoder"; }
  int num_layers() const { return (int)layers_.size(); }
  void zero_grad() { for (auto* l : layers_) l->zero_grad(); }
  void forward(float* output, const float* input, int batch_size, int seq_len) {
    const size_t n = (size_t)batch_size * seq_len * E_;
    if (batch_size != B_ || seq_len != S_) {
      for (float* p : outs_) zerollm_b200_detail::dfree(p);
      outs_.clear();
      for (size_t i = 0; i + 1 < layers_.size(); ++i) outs_.push_back(zerollm_b200_detail::dmalloc(n));
      zerollm_b200_detail::dfree(g0_);
      zerollm_b200_detail::dfree(g1_);
      g0_ = zerollm_b200_detail::dmalloc(n);
      g1_ = zerollm_b200_detail::dmalloc(n);
      B_ = batch_size;
      S_ = seq_len;
    }
    const float* cur = input;
    for (size_t i = 0; i < layers_.size(); ++i) {
      float* o = (i + 1 == layers_.size()) ? output : outs_[i];
      layers_[i]->forward(o, cur, batch_size, seq_len);
      cur = o;
    }
  }
  void backward(float* d_input, const float* d_output) {
    const float* cur = d_output;
    for (int i = (int)layers_.size() - 1; i >= 0; --i) {
      float* dst = (i == 0) ? d_input : ((i % 2) ? g0_ : g1_);
      layers_[i]->backward(dst, cur);
      cur = dst;
    }
  }
  void set_optimizer(OptimizerConfig c) { for (auto* l : layers_) l->set_optimizer(c); }
  void step(float lr) { for (auto* l : layers_) l->step(lr); }
};

// =================================================================== zerollm_config.hpp, zerollm.hpp
struct ZeroLLMConfig {
  int vocab_size, embed_dim, num_layers, num_heads, ff_hidden_dim, max_seq_len;
  bool with_grad;
  // topology of the B200 arena model (reference defaults: LayerNorm, sinusoid, tied head, biases)
  int norm = 0, pos = 0, tied = 1, bias = 1;
  ZeroLLMConfig(int v, int e, int l, int h, int f, int max_seq = 2048, bool wg = false)
      : vocab_size(v), embed_dim(e), num_layers(l), num_heads(h), ff_hidden_dim(f), max_seq_len(max_seq),
        with_grad(wg) {}
};
inline ZeroLLMConfig create_zerollm_26m_config() { return ZeroLLMConfig(6400, 512, 6, 8, 2048, 2048, true); }
inline ZeroLLMConfig create_zerollm_58m_config() { return ZeroLLMConfig(6400, 512, 12, 8, 2048, 2048, true); }
inline ZeroLLMConfig create_zerollm_110m_config() { return ZeroLLMConfig(6400, 768, 12, 12, 3072, 2048, true); }
inline ZeroLLMConfig create_zerollm_340m_config() { return ZeroLLMConfig(6400, 1024, 24, 16, 4096, 2048, true); }

// The whole model on one arena (bf16 activations, fp32 master weights) behind zl_model_*.
class ZeroLLM : public Module {
  ZeroLLMConfig cfg_;
  zl_model* m_ = nullptr;
  float lr_last_ = 0.f;

 public:
  explicit ZeroLLM(const ZeroLLMConfig& c, int64_t max_tokens = 16 * 2048, uint64_t seed = 0, float init_std = 0.02f)
      : Module("ZeroLLM"), cfg_(c) {
    zl_model_config mc{c.vocab_size, c.embed_dim, c.num_layers, c.num_heads, c.ff_hidden_dim, c.max_seq_len,
                       c.norm, c.pos, c.tied, c.bias, 1e-5f, 10000.0f};
    ZLB_CALL(zl_model_create(&mc, max_tokens, seed, init_std, &m_), "ZeroLLM");
    float *p, *g;
    ZLB_CALL(zl_model_buffers(m_, &p, &g, nullptr, nullptr), "ZeroLLM");
    int64_t n = 0;
    zl_model_num_params(m_, &n);
    register_parameter("arena", p, g, (size_t)n, c.with_grad);
  }
  ~ZeroLLM() override { zl_model_destroy(m_); }
  std::string type_name() const override { return "ZeroLLM"; }
  zl_model* handle() { return m_; }
  double calculate_num_params() const {
    int64_t n = 0;
    zl_model_num_params(m_, &n);
    return (double)n / 1e6;
  }
  void forward(float* logits, const int* input_ids, int batch_size, int seq_len, cudaStream_t s = 0) {
    ZLB_CALL(zl_model_forward(m_, input_ids, batch_size, seq_len, logits, s), "ZeroLLM::forward");
  }
  void backward(const int* input_ids, const float* d_logits, int batch_size, int seq_len, cudaStream_t s = 0) {
    if (!cfg_.with_grad) throw std::runtime_error("Cannot call backward() when with_grad=false");
    ZLB_CALL(zl_model_backward(m_, input_ids, d_logits, batch_size, seq_len, s), "ZeroLLM::backward");
  }
  void zero_grad(cudaStream_t s = 0) { ZLB_CALL(zl_model_zero_grad(m_, s), "ZeroLLM::zero_grad"); }
  void set_optimizer(OptimizerConfig c) {
    zl_adamw_config o{c.beta1, c.beta2, c.eps, c.type == OptimizerType::AdamW ? c.weight_decay : 0.0f};
    ZLB_CALL(zl_model_set_optimizer(m_, &o), "ZeroLLM::set_optimizer");
  }
  void step(float learning_rate, cudaStream_t s = 0) { ZLB_CALL(zl_model_step(m_, learning_rate, s), "ZeroLLM::step"); }
  // zerollm.cpp:334-425: the reference's checkpoint directory (config.bin and one raw fp32 file per
  // tensor); a configuration mismatch throws std::runtime_error as there.  with_optimizer adds the
  // AdamW moments and step count, which the reference does not save.
  void save(const std::string& path, bool with_optimizer = false) {
    ZLB_CALL(zl_model_save(m_, path.c_str(), with_optimizer ? 1 : 0), "ZeroLLM::save");
  }
  void load(const std::string& path, bool with_optimizer = false) {
    ZLB_CALL(zl_model_load(m_, path.c_str(), with_optimizer ? 1 : 0), "ZeroLLM::load");
  }
  // Fused step; the mean loss is written to loss_dev (device float).
  void train_step(const int* ids, const int* targets, int batch_size, int seq_len, float lr, float* loss_dev,
                  cudaStream_t s = 0) {
    ZLB_CALL(zl_model_train_step(m_, ids, targets, batch_size, seq_len, lr, 1, loss_dev, s), "ZeroLLM::train_step");
  }
};

// =================================================================== distributed
namespace zerollm {
namespace dist {
enum class ReduceOp { SUM, PROD, MIN, MAX, AVG };
enum class DataType { FLOAT32, FLOAT16, BFLOAT16, INT32, INT64 };
enum class BackendType { NCCL, RCCL, MPI_CPU };

class AbstractBackend {
 public:
  virtual ~AbstractBackend() = default;
  virtual void init(int rank, int world_size) = 0;
  virtual void all_reduce(void* buffer, size_t count, DataType dtype, ReduceOp op, void* stream = nullptr) = 0;
  virtual void broadcast(void* buffer, size_t count, DataType dtype, int root_rank, void* stream = nullptr) = 0;
  virtual void all_gather(const void* sendbuf, void* recvbuf, size_t count, DataType dtype, void* stream = nullptr) = 0;
  virtual void barrier() = 0;
  virtual std::string name() const = 0;
};

// gpu_backend.cpp:66-130 without MPI: init() rendezvous through the file named by
// $ZEROLLM_NCCL_ID_FILE (rank 0 writes the NCCL id, the others wait, bounded by
// $ZEROLLM_NCCL_TIMEOUT seconds, default 120).  Device = rank % device count.
class GPUBackend : public AbstractBackend {
  zl_comm* comm_ = nullptr;
  int rank_ = 0, world_ = 1;
  double timeout_ = 120.0;

 public:
  ~GPUBackend() override { zl_comm_destroy(comm_); }
  void init(int rank, int world_size) override {
    int ndev = 1;
    cudaGetDeviceCount(&ndev);
    cudaSetDevice(rank % (ndev > 0 ? ndev : 1));
    const char* path = std::getenv("ZEROLLM_NCCL_ID_FILE");
    if (const char* t = std::getenv("ZEROLLM_NCCL_TIMEOUT")) timeout_ = std::atof(t);
    if (!path) throw std::runtime_error("GPUBackend::init: set ZEROLLM_NCCL_ID_FILE to a path shared by all ranks");
    ZLB_CALL(zl_comm_create_from_file(path, rank, world_size, timeout_, &comm_), "GPUBackend::init");
    rank_ = rank;
    world_ = world_size;
  }
  void all_reduce(void* buffer, size_t count, DataType dtype, ReduceOp op, void* stream = nullptr) override {
    ZLB_CALL(zl_comm_all_reduce(comm_, buffer, count, (int)dtype, (int)op, stream), "all_reduce");
  }
  void broadcast(void* buffer, size_t count, DataType dtype, int root_rank, void* stream = nullptr) override {
    ZLB_CALL(zl_comm_broadcast(comm_, buffer, count, (int)dtype, root_rank, stream), "broadcast");
  }
  void all_gather(const void* sendbuf, void* recvbuf, size_t count, DataType dtype, void* stream = nullptr) override {
    ZLB_CALL(zl_comm_all_gather(comm_, sendbuf, recvbuf, count, (int)dtype, stream), "all_gather");
  }
  // Collective barrier: a 1-element all-reduce, waited on with the deadline (MPI_Barrier in the reference).
  void barrier() override {
    static float* one = nullptr;
    if (!one) one = zerollm_b200_detail::dmalloc(1);
    all_reduce(one, 1, DataType::FLOAT32, ReduceOp::SUM, nullptr);
    ZLB_CALL(zl_comm_check(comm_, nullptr, timeout_), "barrier");
  }
  std::string name() const override { return "NCCL"; }
  int rank() const { return rank_; }
  int world_size() const { return world_; }
};

class BackendFactory {
 public:
  static std::unique_ptr<AbstractBackend> create_backend() { return std::make_unique<GPUBackend>(); }
};
}  // namespace dist
}  // namespace zerollm
