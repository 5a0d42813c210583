// api_test.cpp -- exercises the C++ drop-in API (zerollm_b200/csrc/api/*.hpp)
// the way the reference's tests/kernel_*.cpp use theirs: known-answer cases
// through the reference function names, then the Layer/Loss/Optimizer/Model
// classes.  Exits non-zero on the first failure (the reference's tests print
// PASS/FAIL and always exit 0).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "kernels.hpp"
#include "zerollm.hpp"

static int g_fail = 0;
#define EXPECT(cond, ...)                       \
  do {                                          \
    if (!(cond)) {                              \
      std::fprintf(stderr, "FAIL %s:%d ", __FILE__, __LINE__); \
      std::fprintf(stderr, __VA_ARGS__);        \
      std::fprintf(stderr, "\n");               \
      ++g_fail;                                 \
    }                                           \
  } while (0)

template <typename T>
static T* dev(const std::vector<T>& h) {
  T* d = nullptr;
  cudaMalloc(&d, h.size() * sizeof(T));
  cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
  return d;
}
template <typename T>
static std::vector<T> host(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaDeviceSynchronize();
  cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
  return h;
}

static void test_matmul_kat() {  // kernel_matmul.cpp:55-83
  std::vector<float> A = {1, 2, 3, 4, 5, 6}, B = {1, 2, 3, 4, 5, 6, 7, 8};
  float *dA = dev(A), *dB = dev(B), *dC = dev(std::vector<float>(12, 0.f));
  matmul_tiled<float>(dA, dB, dC, 3, 4, 2);
  auto C = host(dC, 12);
  const float want[] = {11, 14, 17, 20, 23, 30, 37, 44, 35, 46, 57, 68};
  for (int i = 0; i < 12; ++i) EXPECT(std::fabs(C[i] - want[i]) < 1e-3f, "matmul[%d]=%f", i, C[i]);
  cudaFree(dA); cudaFree(dB); cudaFree(dC);
}

static void test_relu_add_transpose() {  // kernel_relu.cpp:80-81, kernel_add.cpp:29-31, kernel_transpose.cpp:22-43
  std::vector<float> x = {-3, -1, 0, 1, 2, -0.5f, 4, -2, 0, 5};
  float *dx = dev(x), *dy = dev(std::vector<float>(10));
  relu_forward<float>(dx, dy, 10);
  auto y = host(dy, 10);
  const float want[] = {0, 0, 0, 1, 2, 0, 4, 0, 0, 5};
  for (int i = 0; i < 10; ++i) EXPECT(y[i] == want[i], "relu[%d]", i);
  std::vector<float> a(10), b(10);
  for (int i = 0; i < 10; ++i) { a[i] = (float)(i + 1); b[i] = (float)(10 - i); }
  float *da = dev(a), *db = dev(b), *dout = dev(std::vector<float>(10));
  add<float>(da, db, dout, 10);
  for (float v : host(dout, 10)) EXPECT(v == 11.f, "add");
  std::vector<float> t(12);
  for (int i = 0; i < 12; ++i) t[i] = (float)(i + 1);
  float *dt = dev(t), *dtt = dev(std::vector<float>(12));
  transpose<float>(dt, dtt, 3, 4);
  auto tt = host(dtt, 12);
  const float tw[] = {1, 5, 9, 2, 6, 10, 3, 7, 11, 4, 8, 12};
  for (int i = 0; i < 12; ++i) EXPECT(tt[i] == tw[i], "transpose[%d]", i);
  bool threw = false;
  try { add<float>(da, db, dout, 0); } catch (const std::invalid_argument&) { threw = true; }
  EXPECT(threw, "add(size=0) must throw std::invalid_argument (add.cu:36-38)");
  relu_forward<float>(dx, dy, 0);  // silent return (relu.cu:23)
  for (float* p : {dx, dy, da, db, dout, dt, dtt}) cudaFree(p);
}

static void test_embedding_kat() {  // kernel_embedding.cpp:216-275 (invalid ids leave rows untouched)
  std::vector<int> ids = {-1, 2, 10};
  std::vector<float> table(10), pos(6);
  for (int i = 0; i < 10; ++i) table[i] = (float)i;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 2; ++j) pos[i * 2 + j] = (float)i + (float)j * 0.1f;
  int* di = dev(ids);
  float *dt = dev(table), *dp = dev(pos), *dout = dev(std::vector<float>(6, 0.f));
  cuda_embedding_forward<float, int>(di, dt, dp, dout, 1, 3, 2, 5, 3);
  auto o = host(dout, 6);
  EXPECT(o[0] == 0.f && o[1] == 0.f && o[4] == 0.f && o[5] == 0.f, "invalid ids must leave rows untouched");
  EXPECT(o[2] == table[4] + pos[2] && o[3] == table[5] + pos[3], "valid row");
  cudaFree(di); cudaFree(dt); cudaFree(dp); cudaFree(dout);
}

static void test_mha_causal_kat() {  // kernel_mha.cpp:140-213
  std::vector<float> Q = {1, 0, 0, 1, 1, 1}, V = {1, 2, 3, 4, 5, 6};
  float *dq = dev(Q), *dk = dev(Q), *dv = dev(V), *dout = dev(std::vector<float>(6)), *ds = dev(std::vector<float>(9));
  mha_forward<float>(dq, dk, dv, dout, ds, nullptr, 1, 3, 1, 2, true);
  auto P = host(ds, 9);
  EXPECT(std::fabs(P[1]) < 1e-4f && std::fabs(P[2]) < 1e-4f && std::fabs(P[5]) < 1e-4f, "causal mask");
  for (float* p : {dq, dk, dv, dout, ds}) cudaFree(p);
}

static void test_layers_and_loss() {
  // Linear + CrossEntropyLoss + AdamW through the layer API: loss must drop on a fixed batch.
  const int B = 64, IN = 32, C = 16;
  Linear lin(IN, C, true, true);
  lin.set_optimizer(OptimizerConfig::createAdamW(0.0f));
  std::vector<float> x(B * IN);
  std::vector<int> t(B);
  std::mt19937 g(1);
  std::normal_distribution<float> n(0, 1);
  for (auto& v : x) v = n(g);
  for (int i = 0; i < B; ++i) t[i] = i % C;
  float* dx = dev(x);
  int* dt = dev(t);
  float *logits = dev(std::vector<float>(B * C)), *dl = dev(std::vector<float>(B * C));
  CrossEntropyLoss ce;
  float first = 0.f, last = 0.f;
  for (int it = 0; it < 50; ++it) {
    lin.zero_grad();
    lin.forward(logits, dx, B);
    const float l = ce.forward(logits, dt, B, C);
    if (it == 0) first = l;
    last = l;
    ce.backward(dl, logits, dt, B, C);
    lin.backward(nullptr, dl);
    lin.step(1e-2f);
  }
  EXPECT(std::fabs(first - std::log((float)C)) < 1.5f, "initial CE %f", first);
  EXPECT(last < first - 0.5f, "loss must decrease: %f -> %f", first, last);
  std::vector<Parameter> ps;
  lin.get_parameters(ps);
  EXPECT(ps.size() == 2 && ps[0].name == "weight" && ps[1].name == "bias", "parameter registration");
  cudaFree(dx); cudaFree(dt); cudaFree(logits); cudaFree(dl);

  // TransformerDecoder (fp32 layers, reference topology) forward/backward runs and is finite
  const int S = 16, E = 64, H = 2, F = 128, Bt = 2;
  TransformerDecoder dec(2, E, H, F, true);
  std::vector<float> h(Bt * S * E);
  for (auto& v : h) v = n(g);
  float *dh = dev(h), *dy = dev(std::vector<float>(Bt * S * E)), *dg = dev(std::vector<float>(Bt * S * E, 1e-3f));
  float* dxin = dev(std::vector<float>(Bt * S * E));
  dec.forward(dy, dh, Bt, S);
  dec.backward(dxin, dg);
  auto gx = host(dxin, Bt * S * E);
  bool finite = true;
  double norm = 0;
  for (float v : gx) { finite = finite && std::isfinite(v); norm += v * v; }
  EXPECT(finite && norm > 0, "decoder backward finite and non-zero");
  std::vector<Parameter> dp;
  dec.get_parameters(dp);
  EXPECT(dp.size() == 2u * (4 * 2 + 2 + 2 * 2 + 2), "decoder parameter count %zu", dp.size());  // incl. out_proj
  cudaFree(dh); cudaFree(dy); cudaFree(dg); cudaFree(dxin);
}

static void test_model_api() {
  // ZeroLLM on the arena: reference-style forward -> loss -> backward -> step reduces the loss.
  ZeroLLMConfig c(512, 128, 2, 2, 256, 128, true);
  c.norm = 1; c.pos = 1; c.tied = 0;
  const int B = 2, S = 128, T = B * S;
  ZeroLLM model(c, T, 0, 0.02f);
  model.set_optimizer(OptimizerConfig::createAdamW(0.1f, 0.9f, 0.95f));
  std::vector<int> ids(T), tg(T);
  for (int i = 0; i < T; ++i) { ids[i] = (i * 37) % 512; tg[i] = (i * 37 + 11) % 512; }
  int *di = dev(ids), *dtg = dev(tg);
  float *logits = dev(std::vector<float>((size_t)T * 512)), *dl = dev(std::vector<float>((size_t)T * 512));
  CrossEntropyLoss ce;
  float l0 = 0.f, l1 = 0.f;
  for (int it = 0; it < 20; ++it) {
    model.zero_grad();
    model.forward(logits, di, B, S);
    const float l = ce.forward(logits, dtg, T, 512);
    if (it == 0) l0 = l;
    l1 = l;
    ce.backward(dl, logits, dtg, T, 512);
    model.backward(di, dl, B, S);
    model.step(3e-3f);
  }
  EXPECT(std::isfinite(l0) && l1 < l0 - 0.5f, "model loss %f -> %f", l0, l1);
  bool threw = false;
  try { model.backward(di, dl, B, S / 2); } catch (const std::exception&) { threw = true; }
  EXPECT(threw, "backward with a different shape than forward must throw (zerollm.cpp:205-208)");
  cudaFree(di); cudaFree(dtg); cudaFree(logits); cudaFree(dl);
}

int main() {
  test_matmul_kat();
  test_relu_add_transpose();
  test_embedding_kat();
  test_mha_causal_kat();
  test_layers_and_loss();
  test_model_api();
  if (g_fail) {
    std::fprintf(stderr, "%d check(s) failed\n", g_fail);
    return 1;
  }
  std::printf("api_test: all checks passed\n");
  return 0;
}
