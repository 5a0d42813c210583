// api_test.cpp -- exercises the C++ drop-in API (zerollm_b200/csrc/api/*.hpp)
// the way the reference's tests/kernel_*.cpp use theirs: known-answer cases
// through the reference function names, then the Layer/Loss/Optimizer/Model
// classes.  Exits non-zero on the first failure (the reference's tests print
// PASS/FAIL and always exit 0).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
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

// ---------------------------------------------------------------- __nv_bfloat16 instances
// Each bf16 instance against the float instance of the same template on the same inputs (values
// representable in bf16), normwise max|bf16 - f32| / max|f32| < 2e-2.
static std::vector<float> seeded(size_t n, unsigned seed, float scale) {
  std::vector<float> v(n);
  uint64_t s = 0x9E3779B97F4A7C15ull * (seed + 1);
  for (size_t i = 0; i < n; ++i) {
    s ^= s << 13; s ^= s >> 7; s ^= s << 17;
    const float u = (float)((s >> 11) * (1.0 / 9007199254740992.0)) * 2.f - 1.f;
    v[i] = __bfloat162float(__float2bfloat16(u * scale));
  }
  return v;
}
static std::vector<__nv_bfloat16> to_bf(const std::vector<float>& v) {
  std::vector<__nv_bfloat16> o(v.size());
  for (size_t i = 0; i < v.size(); ++i) o[i] = __float2bfloat16(v[i]);
  return o;
}
static float rel_err(const std::vector<__nv_bfloat16>& got, const std::vector<float>& want) {
  float num = 0.f, den = 1e-30f;
  for (size_t i = 0; i < want.size(); ++i) {
    num = std::fmax(num, std::fabs(__bfloat162float(got[i]) - want[i]));
    den = std::fmax(den, std::fabs(want[i]));
  }
  return num / den;
}
template <typename F>
static void both(const std::vector<float>& h, F&& f) {  // run f(float*, bf16*) on device copies
  float* a = dev(h);
  __nv_bfloat16* b = dev(to_bf(h));
  f(a, b);
  cudaFree(a);
  cudaFree(b);
}

static void test_bf16_instances() {
  const float tol = 2e-2f;
  {  // linear_forward / linear_backward (tcgen05 GEMM vs the f32 kernels)
    const int M = 256, K = 192, N = 320;
    auto x = seeded((size_t)M * K, 1, 1.f), w = seeded((size_t)N * K, 2, 0.1f), bias = seeded(N, 3, 0.5f);
    auto dy = seeded((size_t)M * N, 4, 1.f);
    float *xf = dev(x), *wf = dev(w), *bf = dev(bias), *dyf = dev(dy), *yf = dev(std::vector<float>((size_t)M * N));
    __nv_bfloat16 *xb = dev(to_bf(x)), *wb = dev(to_bf(w)), *bb = dev(to_bf(bias)), *dyb = dev(to_bf(dy));
    __nv_bfloat16* yb = dev(std::vector<__nv_bfloat16>((size_t)M * N));
    linear_forward<float>(xf, wf, bf, yf, M, K, N, true);
    linear_forward<__nv_bfloat16>(xb, wb, bb, yb, M, K, N, true);
    const float e = rel_err(host(yb, (size_t)M * N), host(yf, (size_t)M * N));
    EXPECT(e < tol, "linear_forward<bf16> rel %g", e);
    std::vector<float> db0 = seeded(N, 5, 1.f);
    float *dxf = dev(std::vector<float>((size_t)M * K)), *dwf = dev(std::vector<float>((size_t)N * K)), *dbf = dev(db0);
    __nv_bfloat16 *dxb = dev(std::vector<__nv_bfloat16>((size_t)M * K)),
                  *dwb = dev(std::vector<__nv_bfloat16>((size_t)N * K)), *dbb = dev(to_bf(db0));
    linear_backward<float>(dyf, xf, wf, dxf, dwf, dbf, M, K, N, true);
    linear_backward<__nv_bfloat16>(dyb, xb, wb, dxb, dwb, dbb, M, K, N, true);
    float e1 = rel_err(host(dxb, (size_t)M * K), host(dxf, (size_t)M * K));
    float e2 = rel_err(host(dwb, (size_t)N * K), host(dwf, (size_t)N * K));
    float e3 = rel_err(host(dbb, N), host(dbf, N));
    EXPECT(e1 < tol && e2 < tol && e3 < tol, "linear_backward<bf16> rel dX %g dW %g dB %g", e1, e2, e3);
    for (void* p : {(void*)xf, (void*)wf, (void*)bf, (void*)dyf, (void*)yf, (void*)xb, (void*)wb, (void*)bb,
                    (void*)dyb, (void*)yb, (void*)dxf, (void*)dwf, (void*)dbf, (void*)dxb, (void*)dwb, (void*)dbb})
      cudaFree(p);
  }
  {  // mha_forward / mha_backward (tcgen05 flash attention vs the f32 kernels), causal
    const int B = 1, S = 256, H = 2, Dh = 64, E = H * Dh;
    const size_t n = (size_t)B * S * E, np = (size_t)B * H * S * S;
    auto q = seeded(n, 6, 1.f), k = seeded(n, 7, 1.f), v = seeded(n, 8, 1.f), go = seeded(n, 9, 1.f);
    float *qf = dev(q), *kf = dev(k), *vf = dev(v), *gf = dev(go), *of = dev(std::vector<float>(n)),
          *pf = dev(std::vector<float>(np));
    __nv_bfloat16 *qb = dev(to_bf(q)), *kb = dev(to_bf(k)), *vb = dev(to_bf(v)), *gb = dev(to_bf(go)),
                  *ob = dev(std::vector<__nv_bfloat16>(n)), *pb = dev(std::vector<__nv_bfloat16>(np));
    mha_forward<float>(qf, kf, vf, of, pf, nullptr, B, S, H, Dh, true);
    mha_forward<__nv_bfloat16>(qb, kb, vb, ob, pb, nullptr, B, S, H, Dh, true);
    const float e = rel_err(host(ob, n), host(of, n));
    EXPECT(e < tol, "mha_forward<bf16> rel %g", e);
    float *dqf = dev(std::vector<float>(n)), *dkf = dev(std::vector<float>(n)), *dvf = dev(std::vector<float>(n));
    __nv_bfloat16 *dqb = dev(std::vector<__nv_bfloat16>(n)), *dkb = dev(std::vector<__nv_bfloat16>(n)),
                  *dvb = dev(std::vector<__nv_bfloat16>(n));
    for (int scaled = 0; scaled < 2; ++scaled) {
      if (scaled) {
        mha_backward_scaled<float>(gf, qf, kf, vf, pf, nullptr, dqf, dkf, dvf, B, S, H, Dh, true);
        mha_backward_scaled<__nv_bfloat16>(gb, qb, kb, vb, pb, nullptr, dqb, dkb, dvb, B, S, H, Dh, true);
      } else {  // the reference's own semantics (no 1/sqrt(head_dim) in dQ, dK)
        mha_backward<float>(gf, qf, kf, vf, pf, nullptr, dqf, dkf, dvf, B, S, H, Dh, true);
        mha_backward<__nv_bfloat16>(gb, qb, kb, vb, pb, nullptr, dqb, dkb, dvb, B, S, H, Dh, true);
      }
      const float a = rel_err(host(dqb, n), host(dqf, n)), b2 = rel_err(host(dkb, n), host(dkf, n)),
                  c = rel_err(host(dvb, n), host(dvf, n));
      EXPECT(a < tol && b2 < tol && c < tol, "mha_backward<bf16> (scaled %d) rel dQ %g dK %g dV %g", scaled, a, b2, c);
    }
    bool threw = false;
    try { mha_forward<__nv_bfloat16>(qb, kb, vb, ob, pb, nullptr, B, S, H, Dh, false); } catch (const std::runtime_error&) { threw = true; }
    EXPECT(threw, "mha_forward<bf16> without the causal mask must throw (flash path is causal only)");
    for (void* p : {(void*)qf, (void*)kf, (void*)vf, (void*)gf, (void*)of, (void*)pf, (void*)qb, (void*)kb, (void*)vb,
                    (void*)gb, (void*)ob, (void*)pb, (void*)dqf, (void*)dkf, (void*)dvf, (void*)dqb, (void*)dkb,
                    (void*)dvb})
      cudaFree(p);
  }
  {  // layernorm, softmax, add, relu, adamw
    const int M = 64, N = 256;
    const size_t n = (size_t)M * N;
    auto x = seeded(n, 10, 2.f), g = seeded(N, 11, 0.5f), bta = seeded(N, 12, 0.5f), dy = seeded(n, 13, 1.f);
    for (auto& t : g) t = __bfloat162float(__float2bfloat16(1.f + t));
    float *xf = dev(x), *gf = dev(g), *bf = dev(bta), *dyf = dev(dy), *yf = dev(std::vector<float>(n)),
          *mf = dev(std::vector<float>(M)), *rf = dev(std::vector<float>(M)), *dxf = dev(std::vector<float>(n)),
          *dgf = dev(std::vector<float>(N)), *dbf = dev(std::vector<float>(N));
    __nv_bfloat16 *xb = dev(to_bf(x)), *gb = dev(to_bf(g)), *bb = dev(to_bf(bta)), *dyb = dev(to_bf(dy)),
                  *yb = dev(std::vector<__nv_bfloat16>(n)), *mb = dev(std::vector<__nv_bfloat16>(M)),
                  *rb = dev(std::vector<__nv_bfloat16>(M)), *dxb = dev(std::vector<__nv_bfloat16>(n)),
                  *dgb = dev(std::vector<__nv_bfloat16>(N)), *dbb = dev(std::vector<__nv_bfloat16>(N));
    cuda_layernorm_forward<float>(xf, gf, bf, yf, mf, rf, M, N, 1e-5f);
    cuda_layernorm_forward<__nv_bfloat16>(xb, gb, bb, yb, mb, rb, M, N, __float2bfloat16(1e-5f));
    float e = rel_err(host(yb, n), host(yf, n));
    EXPECT(e < tol, "cuda_layernorm_forward<bf16> rel %g", e);
    cuda_layernorm_backward<float>(xf, dyf, gf, mf, rf, dxf, dgf, dbf, M, N);
    cuda_layernorm_backward<__nv_bfloat16>(xb, dyb, gb, mb, rb, dxb, dgb, dbb, M, N);
    const float e1 = rel_err(host(dxb, n), host(dxf, n)), e2 = rel_err(host(dgb, N), host(dgf, N)),
                e3 = rel_err(host(dbb, N), host(dbf, N));
    EXPECT(e1 < tol && e2 < tol && e3 < tol, "cuda_layernorm_backward<bf16> rel %g %g %g", e1, e2, e3);
    softmax<float>(xf, yf, M, N);
    softmax<__nv_bfloat16>(xb, yb, M, N);
    e = rel_err(host(yb, n), host(yf, n));
    EXPECT(e < tol, "softmax<bf16> rel %g", e);
    add<float>(xf, dyf, yf, (int)n);
    add<__nv_bfloat16>(xb, dyb, yb, (int)n);
    e = rel_err(host(yb, n), host(yf, n));
    EXPECT(e < tol, "add<bf16> rel %g", e);
    relu_backward<float>(xf, dyf, yf, (int)n);
    relu_backward<__nv_bfloat16>(xb, dyb, yb, (int)n);
    e = rel_err(host(yb, n), host(yf, n));
    EXPECT(e < tol, "relu_backward<bf16> rel %g", e);
    auto m0 = seeded(n, 14, 1e-3f), v0 = seeded(n, 15, 1e-4f);
    for (auto& t : v0) t = std::fabs(t);
    float *mvf = dev(m0), *vvf = dev(v0);
    __nv_bfloat16 *mvb = dev(to_bf(m0)), *vvb = dev(to_bf(v0));
    adamw_step<float>(xf, dyf, mvf, vvf, (int)n, 1e-2f, 0.1f, 0.9f, 0.95f, 1e-8f, 0.1f, 0.05f);
    adamw_step<__nv_bfloat16>(xb, dyb, mvb, vvb, (int)n, 1e-2f, 0.1f, 0.9f, 0.95f, 1e-8f, 0.1f, 0.05f);
    e = rel_err(host(xb, n), host(xf, n));
    EXPECT(e < tol, "adamw_step<bf16> rel %g", e);
    for (void* p : {(void*)xf, (void*)gf, (void*)bf, (void*)dyf, (void*)yf, (void*)mf, (void*)rf, (void*)dxf,
                    (void*)dgf, (void*)dbf, (void*)xb, (void*)gb, (void*)bb, (void*)dyb, (void*)yb, (void*)mb,
                    (void*)rb, (void*)dxb, (void*)dgb, (void*)dbb, (void*)mvf, (void*)vvf, (void*)mvb, (void*)vvb})
      cudaFree(p);
  }
}

int main() {
  test_matmul_kat();
  test_relu_add_transpose();
  test_embedding_kat();
  test_mha_causal_kat();
  test_layers_and_loss();
  test_model_api();
  test_bf16_instances();
  if (g_fail) {
    std::fprintf(stderr, "%d check(s) failed\n", g_fail);
    return 1;
  }
  std::printf("api_test: all checks passed\n");
  return 0;
}
