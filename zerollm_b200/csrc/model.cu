// model.cu -- the ZeroLLM training step on one arena (host orchestration).
//
// Mirrors the reference dataflow of src/model/zerollm.cpp:101-323 and
// src/layer/transformer_block.cpp:68-211 (post-norm decoder blocks:
// x -> MHA -> add -> norm1 -> FFN(ReLU) -> add -> norm2), with the topology
// switches norm={LayerNorm,RMSNorm}, pos={sinusoid,RoPE}, head={tied,untied}.
// Differences from the reference, by design:
//  * every activation lives in a preallocated arena (no cudaMalloc in the
//    step, no device syncs), activations are bf16, master weights fp32;
//  * the forward saves what backward needs under distinct names (the
//    reference's in-place LayerNorm and shared decoder buffers alias saved
//    inputs, transformer_block.cpp:97, transformer_decoder.cpp:79);
//  * Q/K/V projections are one GEMM, bias/ReLU/residual/RoPE are GEMM
//    epilogues, softmax + cross-entropy + its gradient is one kernel, and
//    AdamW is one launch over the flat parameter arena.
//  * data parallelism: gradients are produced in arena order (the arena is
//    laid out in reverse forward order), so buckets become ready during
//    backward and are all-reduced on a side stream (NCCL) while backward
//    continues; the 1/world average is folded into AdamW.
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <string>
#include <thread>
#include <vector>

#include <nccl.h>

#include "common.cuh"

namespace zl {
// kernels.cu: norm backward that also accumulates column sums of its output (a bias gradient)
zl_status norm_backward_bf16(int kind, const zl_bf16* x, const zl_bf16* dy, const float* gamma, const float* mean,
                             const float* rstd, zl_bf16* dx, float* dgamma, float* dbeta, float* dcol,
                             float* workspace, int64_t M, int N, cudaStream_t s, bool fused);
// kernels.cu: column sums added straight into db (one launch)
zl_status colsum_bf16_add(const zl_bf16* dy, float* db, int64_t M, int N, cudaStream_t s);
// gemm.cu: a bf16 GEMM whose epilogue also adds the column sums of its output into colsum (may be
// null), writes its ReLU mask as bits (bits_out) or masks with bits written earlier (bits_in)
zl_status gemm_bf16_colsum(const zl_bf16* A, const zl_bf16* B, void* D, int M, int N, int K, int layout, int flags,
                           const zl_epilogue* epi, float* ws, float* colsum, cudaStream_t st, uint32_t* bits_out,
                           const uint32_t* bits_in, int* sched);
// attention.cu: the attention backward with events recorded around its main kernel
zl_status attention_backward_bf16(const zl_bf16* qkv, const zl_bf16* o, const zl_bf16* d_o, const float* lse,
                                  zl_bf16* d_qkv, float* workspace, int batch, int seq_len, int num_heads,
                                  int head_dim, const float* rope_cos, const float* rope_sin, zl_stream stream,
                                  cudaEvent_t ev0, cudaEvent_t ev1);
}  // namespace zl


// ============================================================== host RNG (same stream as the oracle)
namespace {
uint64_t splitmix64(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Normals by Box-Muller, one pair per two draws.  splitmix64 advances its state by a fixed step
// per draw, so the pair range [p0, p1) starts from seed + 2 * p0 * step and large tensors are filled
// by several host threads with exactly the serial sequence.
void fill_normal_range(float* out, int64_t n, uint64_t seed, float mean, float stdv, int64_t p0, int64_t p1) {
  uint64_t s = seed + 2ull * (uint64_t)p0 * 0x9E3779B97F4A7C15ull;
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t p = p0; p < p1; ++p) {
    const int64_t i = 2 * p;
    const double u1 = ((double)(splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);
    const double r = sqrt(-2.0 * log(u1));
    out[i] = (float)(mean + stdv * r * cos(two_pi * u2));
    if (i + 1 < n) out[i + 1] = (float)(mean + stdv * r * sin(two_pi * u2));
  }
}
void fill_normal(float* out, int64_t n, uint64_t seed, float mean, float stdv) {
  const int64_t pairs = (n + 1) / 2;
  const int64_t nt = std::min<int64_t>(std::max(1u, std::thread::hardware_concurrency()), 32);
  if (pairs < (1 << 18) || nt == 1) {
    fill_normal_range(out, n, seed, mean, stdv, 0, pairs);
    return;
  }
  std::vector<std::thread> th;
  for (int64_t t = 0; t < nt; ++t)
    th.emplace_back(fill_normal_range, out, n, seed, mean, stdv, pairs * t / nt, pairs * (t + 1) / nt);
  for (auto& x : th) x.join();
}

enum Kind { K_MAT = 0, K_BIAS = 1, K_GAMMA = 2, K_BETA = 3, K_EMB = 4 };
enum { L_N2G, L_N2B, L_W2, L_B2, L_W1, L_B1, L_N1G, L_N1B, L_WO, L_BO, L_WQKV, L_BQKV, L_COUNT };

struct Layout {
  std::vector<int64_t> off, size;
  std::vector<int> kind;
  int64_t head = -1, nog = -1, nob = -1, emb = -1;
  std::vector<std::array<int64_t, L_COUNT>> lay;
  int64_t total = 0;
};

// Canonical layout: reverse forward order (the order backward completes gradients).
Layout build_layout(const zl_model_config& c) {
  Layout L;
  const int64_t d = c.embed_dim, F = c.ff_hidden_dim, V = c.vocab_size;
  auto add = [&](int64_t sz, int kind) {
    L.off.push_back(L.total);
    L.size.push_back(sz);
    L.kind.push_back(kind);
    L.total += sz;
    return L.off.back();
  };
  if (!c.tied) L.head = add(V * d, K_MAT);
  L.nog = add(d, K_GAMMA);
  if (c.norm == 0) L.nob = add(d, K_BETA);
  L.lay.assign(c.num_layers, {});
  for (int l = c.num_layers - 1; l >= 0; --l) {
    auto& t = L.lay[l];
    t.fill(-1);
    t[L_N2G] = add(d, K_GAMMA);
    if (c.norm == 0) t[L_N2B] = add(d, K_BETA);
    t[L_W2] = add(d * F, K_MAT);
    if (c.bias) t[L_B2] = add(d, K_BIAS);
    t[L_W1] = add(F * d, K_MAT);
    if (c.bias) t[L_B1] = add(F, K_BIAS);
    t[L_N1G] = add(d, K_GAMMA);
    if (c.norm == 0) t[L_N1B] = add(d, K_BETA);
    t[L_WO] = add(d * d, K_MAT);
    if (c.bias) t[L_BO] = add(d, K_BIAS);
    t[L_WQKV] = add(3 * d * d, K_MAT);
    if (c.bias) t[L_BQKV] = add(3 * d, K_BIAS);
  }
  L.emb = add(V * d, K_EMB);
  return L;
}

zl_status validate(const zl_model_config& c) {
  if (c.vocab_size <= 0 || c.embed_dim <= 0 || c.num_layers <= 0 || c.num_heads <= 0 || c.ff_hidden_dim <= 0 ||
      c.max_seq_len <= 0)
    return zl::set_error(ZL_EINVAL, "model config: sizes must be positive");
  if (c.embed_dim % c.num_heads) return zl::set_error(ZL_EINVAL, "model config: embed_dim %% num_heads != 0");
  if (c.num_heads <= 0 || c.embed_dim % c.num_heads ||
      (c.embed_dim / c.num_heads != 64 && c.embed_dim / c.num_heads != 128))
    return zl::set_error(ZL_EUNSUPPORTED, "model: head_dim must be 64 or 128");
  if (c.embed_dim % 64 || c.ff_hidden_dim % 64 || c.vocab_size % 64)
    return zl::set_error(ZL_EUNSUPPORTED, "model: embed_dim, ff_hidden_dim and vocab_size must be multiples of 64");
  if (c.num_layers > 256) return zl::set_error(ZL_EUNSUPPORTED, "model: at most 256 layers");
  if (c.norm != 0 && c.norm != 1) return zl::set_error(ZL_EINVAL, "model: norm must be 0 or 1");
  if (c.pos != 0 && c.pos != 1) return zl::set_error(ZL_EINVAL, "model: pos must be 0 or 1");
  return ZL_OK;
}
}  // namespace

using bf16 = __nv_bfloat16;

struct DistState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  cudaStream_t comm_stream = nullptr;
  std::vector<int64_t> b_start, b_len;
  std::vector<cudaEvent_t> ready_ev;  // recorded on the compute stream when a bucket's grads are final
  cudaEvent_t done_ev = nullptr;      // recorded on comm stream after the last bucket
  int next_bucket = 0;
  bool joined = false;  // the last step ran as a graph that already waits for its all-reduces
};

struct zl_model {
  zl_model_config cfg;
  Layout L;
  int64_t max_tokens = 0;
  int dev = 0;
  // arenas
  float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr;
  bf16* pbf = nullptr;
  float *pos_table = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
  float *rope_cos_pm = nullptr, *rope_sin_pm = nullptr;  // the same tables pair-major ([Dh/2, S]) for the QKV epilogue
  // activations
  std::vector<bf16*> x, qkv, attn, r1, h1, f, r2;
  // per layer, f > 0 as bits ([T][F/32] words), written by the FF1 product and read by the ReLU
  // backward in place of f itself (empty when F is not a multiple of 128: the backward then reads f)
  std::vector<uint32_t*> fbits;
  std::vector<float*> lse, mean1, rstd1, mean2, rstd2;
  bf16* hf = nullptr;
  float *meanf = nullptr, *rstdf = nullptr;
  bf16* logits = nullptr;
  float* loss_rows = nullptr;
  // backward temporaries
  bf16 *dx = nullptr, *dr = nullptr, *dtmp = nullptr, *dF = nullptr, *dqkv = nullptr, *dattn = nullptr;
  // workspaces
  float* ws = nullptr;
  int64_t ws_floats = 0;
  std::vector<void*> allocs;
  // optimizer
  zl_adamw_config opt{0.9f, 0.95f, 1e-8f, 0.1f};
  int t = 0;
  // state
  int last_B = 0, last_S = 0;
  int launches = 0;
  DistState dist;
  int64_t ready_prefix = 0;  // grads in [0, ready_prefix) are final for this step
  // CUDA graph of zero_grad -> forward -> CE -> backward for one (ids, targets, loss, B, S) binding
  int use_graph = 1;
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  const void *g_ids = nullptr, *g_tgt = nullptr, *g_loss = nullptr;
  int g_B = 0, g_S = 0, g_seen = 0, g_launches = 0;
  // In-step kernel timing: per layer, events just before and after the attention forward kernel
  // and the attention backward's main kernel (graph event nodes in the captured step).
  std::vector<cudaEvent_t> kt_ev;  // [layer][fwd start, fwd end, bwd start, bwd end], then step start,
                                   // end of the last backward kernel, step end (side stream rejoined)
  bool kt_valid = false;           // a step has recorded them
};

namespace {

template <typename T>
zl_status dalloc(zl_model* M, T** p, int64_t n) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, (size_t)std::max<int64_t>(n, 1) * sizeof(T));
  if (e != cudaSuccess) return zl::set_error(ZL_ENOMEM, "model arena: cudaMalloc(%lld bytes): %s",
                                             (long long)(n * sizeof(T)), cudaGetErrorString(e));
  M->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return ZL_OK;
}

#define TRY(x)                         \
  do {                                 \
    zl_status _s = (x);                \
    if (_s != ZL_OK) return _s;        \
  } while (0)

// Workspace needed by the step's GEMMs and reductions at T tokens.
int64_t step_workspace(const zl_model_config& c, int64_t T, int B_max) {
  const int d = c.embed_dim, F = c.ff_hidden_dim, V = c.vocab_size;
  const int Ti = (int)T;
  int64_t w = 0;
  auto g = [&](int M, int N, int K, int layout) { w = std::max(w, zl_gemm_workspace_floats(M, N, K, layout, 0)); };
  const int KK = ZL_A_KMAJOR | ZL_B_KMAJOR;
  g(Ti, 3 * d, d, KK); g(Ti, d, d, KK); g(Ti, F, d, KK); g(Ti, d, F, KK); g(Ti, V, d, KK);
  g(V, d, Ti, 0); g(Ti, d, V, ZL_A_KMAJOR);
  g(d, F, Ti, 0); g(Ti, F, d, ZL_A_KMAJOR); g(F, d, Ti, 0); g(Ti, d, F, ZL_A_KMAJOR);
  g(d, d, Ti, 0); g(Ti, d, d, ZL_A_KMAJOR); g(3 * d, d, Ti, 0); g(Ti, d, 3 * d, ZL_A_KMAJOR);
  w = std::max(w, zl_attention_workspace_floats(B_max, (int)(T / B_max), c.num_heads, d / c.num_heads));
  w = std::max(w, (int64_t)3 * d * zl_norm_bwd_blocks(T));  // dgamma | dbeta | bias column sums
  w = std::max(w, zl_colsum_workspace_floats(T, std::max(3 * d, F)));
  return w;
}

zl_status gemm(zl_model* M, const bf16* A, const bf16* B, void* D, int m, int n, int k, int layout, int flags,
               const zl_epilogue* e, cudaStream_t st) {
  M->launches += 1;
  return zl_gemm_bf16(reinterpret_cast<const zl_bf16*>(A), reinterpret_cast<const zl_bf16*>(B), D, m, n, k, layout,
                      flags, e, M->ws, st);
}

// the same, also adding the column sums of the bf16 output D into colsum (a bias gradient) and writing
// (bits_out) or reading (bits_in) the ReLU mask as bits
zl_status gemm_ext(zl_model* M, const bf16* A, const bf16* B, void* D, int m, int n, int k, int layout, int flags,
                   const zl_epilogue* e, float* colsum, uint32_t* bits_out, const uint32_t* bits_in, cudaStream_t st) {
  M->launches += 1;
  return zl::gemm_bf16_colsum(reinterpret_cast<const zl_bf16*>(A), reinterpret_cast<const zl_bf16*>(B), D, m, n, k,
                              layout, flags, e, M->ws, colsum, st, bits_out, bits_in, nullptr);
}

const bf16* W(zl_model* M, int64_t off) { return M->pbf + off; }
const float* P(zl_model* M, int64_t off) { return off >= 0 ? M->params + off : nullptr; }
float* G(zl_model* M, int64_t off) { return off >= 0 ? M->grads + off : nullptr; }

// ----------------------------------------------------------------------------- DP bucket hook
// Called after the gradients in [0, prefix) became final on `st`.
zl_status grads_ready(zl_model* M, int64_t prefix, cudaStream_t st) {
  M->ready_prefix = prefix;
  DistState& D = M->dist;
  if (!D.comm) return ZL_OK;
  while (D.next_bucket < (int)D.b_start.size() && D.b_start[D.next_bucket] + D.b_len[D.next_bucket] <= prefix) {
    const int b = D.next_bucket++;
    cudaEventRecord(D.ready_ev[b], st);
    cudaStreamWaitEvent(D.comm_stream, D.ready_ev[b], 0);
    ncclResult_t r = ncclAllReduce(M->grads + D.b_start[b], M->grads + D.b_start[b], (size_t)D.b_len[b], ncclFloat,
                                   ncclSum, D.comm, D.comm_stream);
    if (r != ncclSuccess) return zl::set_error(ZL_ENCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
  }
  return ZL_OK;
}

int64_t end_of(zl_model* M, int64_t off) {
  for (size_t i = 0; i < M->L.off.size(); ++i)
    if (M->L.off[i] == off) return M->L.off[i] + M->L.size[i];
  return -1;
}
// Last present tensor of a group (skipping absent optional tensors).
int64_t end_of_any(zl_model* M, std::initializer_list<int64_t> offs) {
  int64_t e = -1;
  for (int64_t o : offs)
    if (o >= 0) e = std::max(e, end_of(M, o));
  return e;
}

// ----------------------------------------------------------------------------- forward
// Runs the forward to the bf16 logits (kept in M->logits).  If logits_f32 is non-null the head GEMM
// writes fp32 logits there instead.
zl_status forward(zl_model* M, const int32_t* ids, int B, int S, float* logits_f32, cudaStream_t st) {
  const zl_model_config& c = M->cfg;
  const int64_t T = (int64_t)B * S;
  const int d = c.embed_dim, F = c.ff_hidden_dim, V = c.vocab_size, H = c.num_heads;
  const int KK = ZL_A_KMAJOR | ZL_B_KMAJOR;
  TRY(zl_embedding_forward_bf16(ids, P(M, M->L.emb), c.pos == 0 ? M->pos_table : nullptr,
                                reinterpret_cast<zl_bf16*>(M->x[0]), T, S, d, V, st));
  M->launches++;
  for (int l = 0; l < c.num_layers; ++l) {
    const auto& t = M->L.lay[l];
    zl_epilogue e{};
    e.bias = P(M, t[L_BQKV]);
    int fl = c.bias ? ZL_EPI_BIAS : 0;
    if (c.pos == 1) {
      fl |= ZL_EPI_ROPE;
      // pair-major tables ([Dh/2, max_seq_len]) serve when the step's sequence fills the table rows
      const bool pm = S == c.max_seq_len;
      e.rope_cos = pm ? M->rope_cos_pm : M->rope_cos;
      e.rope_sin = pm ? M->rope_sin_pm : M->rope_sin;
      e.rope_pair_major = pm ? 1 : 0;
      e.rope_cols = 2 * d;
      e.rope_seq = S;
      e.head_dim = d / H;
    }
    TRY(gemm(M, M->x[l], W(M, t[L_WQKV]), M->qkv[l], (int)T, 3 * d, d, KK, fl, &e, st));
    if (!M->kt_ev.empty()) zl::record_timing_event(M->kt_ev[4 * l], st);
    TRY(zl_attention_forward_bf16(reinterpret_cast<zl_bf16*>(M->qkv[l]), reinterpret_cast<zl_bf16*>(M->attn[l]),
                                  M->lse[l], B, S, H, d / H, st));
    if (!M->kt_ev.empty()) zl::record_timing_event(M->kt_ev[4 * l + 1], st);
    M->launches++;
    e = zl_epilogue{};
    e.bias = P(M, t[L_BO]);
    e.residual = reinterpret_cast<zl_bf16*>(M->x[l]);
    TRY(gemm(M, M->attn[l], W(M, t[L_WO]), M->r1[l], (int)T, d, d, KK, (c.bias ? ZL_EPI_BIAS : 0) | ZL_EPI_RESIDUAL,
             &e, st));
    TRY(zl_norm_forward_bf16(c.norm, reinterpret_cast<zl_bf16*>(M->r1[l]), P(M, t[L_N1G]), P(M, t[L_N1B]),
                             reinterpret_cast<zl_bf16*>(M->h1[l]), M->mean1[l], M->rstd1[l], T, d, c.eps, st));
    M->launches++;
    e = zl_epilogue{};
    e.bias = P(M, t[L_B1]);
    // f = relu(h1 W1^T + b1), and f > 0 as bits for the ReLU backward
    TRY(gemm_ext(M, M->h1[l], W(M, t[L_W1]), M->f[l], (int)T, F, d, KK, (c.bias ? ZL_EPI_BIAS : 0) | ZL_EPI_RELU, &e,
                 nullptr, M->fbits.empty() ? nullptr : M->fbits[l], nullptr, st));
    e = zl_epilogue{};
    e.bias = P(M, t[L_B2]);
    e.residual = reinterpret_cast<zl_bf16*>(M->h1[l]);
    TRY(gemm(M, M->f[l], W(M, t[L_W2]), M->r2[l], (int)T, d, F, KK, (c.bias ? ZL_EPI_BIAS : 0) | ZL_EPI_RESIDUAL, &e,
             st));
    TRY(zl_norm_forward_bf16(c.norm, reinterpret_cast<zl_bf16*>(M->r2[l]), P(M, t[L_N2G]), P(M, t[L_N2B]),
                             reinterpret_cast<zl_bf16*>(M->x[l + 1]), M->mean2[l], M->rstd2[l], T, d, c.eps, st));
    M->launches++;
  }
  TRY(zl_norm_forward_bf16(c.norm, reinterpret_cast<zl_bf16*>(M->x[c.num_layers]), P(M, M->L.nog), P(M, M->L.nob),
                           reinterpret_cast<zl_bf16*>(M->hf), M->meanf, M->rstdf, T, d, c.eps, st));
  M->launches++;
  const int64_t head_off = c.tied ? M->L.emb : M->L.head;
  if (logits_f32) {
    TRY(gemm(M, M->hf, W(M, head_off), logits_f32, (int)T, V, d, KK, ZL_EPI_OUT_F32, nullptr, st));
  } else {
    TRY(gemm(M, M->hf, W(M, head_off), M->logits, (int)T, V, d, KK, 0, nullptr, st));
  }
  M->last_B = B;
  M->last_S = S;
  return ZL_OK;
}

// ----------------------------------------------------------------------------- backward
// Expects d_logits (bf16) in M->logits.  Gradients: weight GEMMs overwrite, everything else accumulates
// (the grad arena must be zeroed before the step, zl_model_zero_grad).
zl_status backward(zl_model* M, const int32_t* ids, int B, int S, cudaStream_t st) {
  const zl_model_config& c = M->cfg;
  const int64_t T = (int64_t)B * S;
  const int d = c.embed_dim, F = c.ff_hidden_dim, V = c.vocab_size, H = c.num_heads;
  const int Ti = (int)T;
  const int64_t head_off = c.tied ? M->L.emb : M->L.head;
  // head: dW (accumulate: tied heads share the embedding gradient) and dhf
  TRY(gemm(M, M->logits, M->hf, G(M, head_off), V, d, Ti, 0, ZL_EPI_OUT_F32 | ZL_EPI_ACCUM, nullptr, st));
  if (!c.tied) TRY(grads_ready(M, end_of(M, M->L.head), st));
  TRY(gemm(M, M->logits, W(M, head_off), M->dtmp, Ti, d, V, ZL_A_KMAJOR, 0, nullptr, st));
  TRY(zl::norm_backward_bf16(c.norm, reinterpret_cast<zl_bf16*>(M->x[c.num_layers]),
                             reinterpret_cast<zl_bf16*>(M->dtmp), P(M, M->L.nog), M->meanf, M->rstdf,
                             reinterpret_cast<zl_bf16*>(M->dx), G(M, M->L.nog), c.norm == 0 ? G(M, M->L.nob) : nullptr,
                             nullptr, M->ws, T, d, st, true));
  M->launches += 1;
  TRY(grads_ready(M, end_of_any(M, {M->L.nog, M->L.nob}), st));
  for (int l = c.num_layers - 1; l >= 0; --l) {
    const auto& t = M->L.lay[l];
    // out = norm2(r2)
    // also the FF2 bias gradient: column sums of this norm's output dr
    TRY(zl::norm_backward_bf16(c.norm, reinterpret_cast<zl_bf16*>(M->r2[l]), reinterpret_cast<zl_bf16*>(M->dx),
                               P(M, t[L_N2G]), M->mean2[l], M->rstd2[l], reinterpret_cast<zl_bf16*>(M->dr),
                               G(M, t[L_N2G]), G(M, t[L_N2B]), c.bias ? G(M, t[L_B2]) : nullptr, M->ws, T, d, st,
                               true));
    M->launches += 1;
    TRY(grads_ready(M, end_of_any(M, {t[L_N2G], t[L_N2B]}), st));
    // r2 = h1 + f W2^T + b2
    TRY(gemm(M, M->dr, M->f[l], G(M, t[L_W2]), d, F, Ti, 0, ZL_EPI_OUT_F32 | ZL_EPI_ACCUM, nullptr, st));
    TRY(grads_ready(M, end_of_any(M, {t[L_W2], t[L_B2]}), st));
    zl_epilogue e{};
    if (M->fbits.empty()) e.aux = reinterpret_cast<zl_bf16*>(M->f[l]);
    // dF = (dr W2) masked by f > 0 (the forward's mask bits), and with it the FF1 bias gradient: its
    // column sums, added by the GEMM's epilogue
    TRY(gemm_ext(M, M->dr, W(M, t[L_W2]), M->dF, Ti, F, d, ZL_A_KMAJOR, ZL_EPI_RELU_MASK, &e,
                 c.bias ? G(M, t[L_B1]) : nullptr, nullptr, M->fbits.empty() ? nullptr : M->fbits[l], st));
    TRY(gemm(M, M->dF, M->h1[l], G(M, t[L_W1]), F, d, Ti, 0, ZL_EPI_OUT_F32 | ZL_EPI_ACCUM, nullptr, st));
    TRY(grads_ready(M, end_of_any(M, {t[L_W1], t[L_B1]}), st));
    e = zl_epilogue{};
    e.residual = reinterpret_cast<zl_bf16*>(M->dr);
    TRY(gemm(M, M->dF, W(M, t[L_W1]), M->dtmp, Ti, d, F, ZL_A_KMAJOR, ZL_EPI_RESIDUAL, &e, st));
    // h1 = norm1(r1)
    // also the output-projection bias gradient: column sums of this norm's output dr
    TRY(zl::norm_backward_bf16(c.norm, reinterpret_cast<zl_bf16*>(M->r1[l]), reinterpret_cast<zl_bf16*>(M->dtmp),
                               P(M, t[L_N1G]), M->mean1[l], M->rstd1[l], reinterpret_cast<zl_bf16*>(M->dr),
                               G(M, t[L_N1G]), G(M, t[L_N1B]), c.bias ? G(M, t[L_BO]) : nullptr, M->ws, T, d, st,
                               true));
    M->launches += 1;
    TRY(grads_ready(M, end_of_any(M, {t[L_N1G], t[L_N1B]}), st));
    // r1 = x + attn Wo^T + bo
    TRY(gemm(M, M->dr, M->attn[l], G(M, t[L_WO]), d, d, Ti, 0, ZL_EPI_OUT_F32 | ZL_EPI_ACCUM, nullptr, st));
    TRY(grads_ready(M, end_of_any(M, {t[L_WO], t[L_BO]}), st));
    TRY(gemm(M, M->dr, W(M, t[L_WO]), M->dattn, Ti, d, d, ZL_A_KMAJOR, 0, nullptr, st));
    TRY(zl::attention_backward_bf16(reinterpret_cast<zl_bf16*>(M->qkv[l]), reinterpret_cast<zl_bf16*>(M->attn[l]),
                                    reinterpret_cast<zl_bf16*>(M->dattn), M->lse[l],
                                    reinterpret_cast<zl_bf16*>(M->dqkv), M->ws, B, S, H, d / H,
                                    c.pos == 1 ? M->rope_cos : nullptr, c.pos == 1 ? M->rope_sin : nullptr, st,
                                    M->kt_ev.empty() ? nullptr : M->kt_ev[4 * l + 2],
                                    M->kt_ev.empty() ? nullptr : M->kt_ev[4 * l + 3]));
    M->launches += 3;
    TRY(gemm(M, M->dqkv, M->x[l], G(M, t[L_WQKV]), 3 * d, d, Ti, 0, ZL_EPI_OUT_F32 | ZL_EPI_ACCUM, nullptr, st));
    if (c.bias) { TRY(zl::colsum_bf16_add(reinterpret_cast<zl_bf16*>(M->dqkv), G(M, t[L_BQKV]), T, 3 * d, st)); M->launches += 1; }
    TRY(grads_ready(M, end_of_any(M, {t[L_WQKV], t[L_BQKV]}), st));
    e = zl_epilogue{};
    e.residual = reinterpret_cast<zl_bf16*>(M->dr);
    TRY(gemm(M, M->dqkv, W(M, t[L_WQKV]), M->dx, Ti, d, 3 * d, ZL_A_KMAJOR, ZL_EPI_RESIDUAL, &e, st));
  }
  TRY(zl_embedding_backward_bf16(ids, reinterpret_cast<zl_bf16*>(M->dx), G(M, M->L.emb), T, d, V, st));
  M->launches++;
  TRY(grads_ready(M, M->L.total, st));
  return ZL_OK;
}

zl_status adamw(zl_model* M, float lr, cudaStream_t st) {
  M->t += 1;
  // adamw.cpp:39-43: bias corrections on the host in fp32 powf
  const float bc1 = 1.0f - powf(M->opt.beta1, (float)M->t);
  const float bc2 = 1.0f - powf(M->opt.beta2, (float)M->t);
  const float gs = 1.0f / (float)M->dist.world;
  if (M->dist.comm && !M->dist.joined) {
    cudaEventRecord(M->dist.done_ev, M->dist.comm_stream);
    cudaStreamWaitEvent(st, M->dist.done_ev, 0);
  }
  M->launches++;
  return zl_adamw_flat(M->params, M->grads, M->m, M->v, reinterpret_cast<zl_bf16*>(M->pbf), M->L.total, lr,
                       M->opt.weight_decay, M->opt.beta1, M->opt.beta2, M->opt.eps, bc1, bc2, gs, st);
}

zl_status check_shape(zl_model* M, int B, int S) {
  if (B <= 0 || S <= 0) return zl::set_error(ZL_EINVAL, "batch and seq_len must be positive");
  if (S > M->cfg.max_seq_len) return zl::set_error(ZL_EINVAL, "Sequence length exceeds max_seq_len");  // zerollm.cpp:105-108
  if ((int64_t)B * S > M->max_tokens) return zl::set_error(ZL_EINVAL, "batch*seq_len exceeds the arena (%lld)", (long long)M->max_tokens);
  return ZL_OK;
}

}  // namespace

// ============================================================== C ABI
extern "C" zl_status zl_model_param_layout(const zl_model_config* cfg, int64_t* offsets, int64_t* sizes, int* kinds,
                                           int max_n, int* count, int64_t* total) {
  if (!cfg) return zl::set_error(ZL_EINVAL, "null config");
  TRY(validate(*cfg));
  Layout L = build_layout(*cfg);
  const int n = (int)L.off.size();
  for (int i = 0; i < n && i < max_n; ++i) {
    if (offsets) offsets[i] = L.off[i];
    if (sizes) sizes[i] = L.size[i];
    if (kinds) kinds[i] = L.kind[i];
  }
  if (count) *count = n;
  if (total) *total = L.total;
  return ZL_OK;
}

extern "C" zl_status zl_model_create(const zl_model_config* cfg, int64_t max_tokens, uint64_t seed, float init_std,
                                     zl_model** out) {
  if (!cfg || !out) return zl::set_error(ZL_EINVAL, "null argument");
  TRY(validate(*cfg));
  if (max_tokens <= 0) return zl::set_error(ZL_EINVAL, "max_tokens must be positive");
  zl_model* M = new zl_model();
  M->cfg = *cfg;
  M->L = build_layout(*cfg);
  M->max_tokens = max_tokens;
  cudaGetDevice(&M->dev);
  const zl_model_config& c = *cfg;
  const int64_t T = max_tokens, d = c.embed_dim, F = c.ff_hidden_dim, V = c.vocab_size;
  const int64_t NP = M->L.total;
  auto fail = [&](zl_status s) {
    zl_model_destroy(M);
    return s;
  };
  zl_status s;
#define A(p, n) if ((s = dalloc(M, &(p), (n))) != ZL_OK) return fail(s)
  A(M->params, NP); A(M->grads, NP); A(M->m, NP); A(M->v, NP); A(M->pbf, NP);
  const int L = c.num_layers;
  M->x.resize(L + 1); M->qkv.resize(L); M->attn.resize(L); M->r1.resize(L); M->h1.resize(L); M->f.resize(L);
  M->r2.resize(L); M->lse.resize(L); M->mean1.resize(L); M->rstd1.resize(L); M->mean2.resize(L); M->rstd2.resize(L);
  for (int l = 0; l <= L; ++l) A(M->x[l], T * d);
  for (int l = 0; l < L; ++l) {
    A(M->qkv[l], T * 3 * d); A(M->attn[l], T * d); A(M->r1[l], T * d); A(M->h1[l], T * d); A(M->f[l], T * F);
    A(M->r2[l], T * d); A(M->lse[l], T * c.num_heads); A(M->mean1[l], T); A(M->rstd1[l], T); A(M->mean2[l], T);
    A(M->rstd2[l], T);
  }
  if (F % 128 == 0) {  // the FF1 epilogue writes a row's mask words 16 bytes at a time
    M->fbits.resize(L);
    for (int l = 0; l < L; ++l) A(M->fbits[l], T * (F / 32));
  }
  A(M->hf, T * d); A(M->meanf, T); A(M->rstdf, T); A(M->logits, T * V); A(M->loss_rows, T);
  A(M->dx, T * d); A(M->dr, T * d); A(M->dtmp, T * d); A(M->dF, T * F); A(M->dqkv, T * 3 * d); A(M->dattn, T * d);
  // batch can be as small as 1 -> attention workspace sized for B=1 (T tokens) is the max of B*S*E + B*H*S
  M->ws_floats = step_workspace(c, T, 1);
  A(M->ws, M->ws_floats);
  // constant tables
  const int Dh = (int)(d / c.num_heads);
  if (c.pos == 0) {
    std::vector<float> pt((size_t)c.max_seq_len * d);
    for (int p = 0; p < c.max_seq_len; ++p)  // embedding.cpp:107-126
      for (int i = 0; i < d; ++i) {
        const int k = i / 2;
        const float ang = (float)p / powf(10000.0f, (float)(2 * k) / (float)d);
        pt[(size_t)p * d + i] = (i % 2 == 0) ? sinf(ang) : cosf(ang);
      }
    A(M->pos_table, (int64_t)pt.size());
    cudaMemcpy(M->pos_table, pt.data(), pt.size() * sizeof(float), cudaMemcpyHostToDevice);
  } else {
    const int half = Dh / 2;
    std::vector<float> cs((size_t)c.max_seq_len * half), sn(cs.size());
    for (int p = 0; p < c.max_seq_len; ++p)
      for (int i = 0; i < half; ++i) {
        const double th = (double)p * pow((double)c.rope_base, -2.0 * i / (double)Dh);
        cs[(size_t)p * half + i] = (float)cos(th);
        sn[(size_t)p * half + i] = (float)sin(th);
      }
    A(M->rope_cos, (int64_t)cs.size());
    A(M->rope_sin, (int64_t)sn.size());
    cudaMemcpy(M->rope_cos, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemcpy(M->rope_sin, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice);
    std::vector<float> cst(cs.size()), snt(cs.size());
    for (int p = 0; p < c.max_seq_len; ++p)
      for (int i = 0; i < half; ++i) {
        cst[(size_t)i * c.max_seq_len + p] = cs[(size_t)p * half + i];
        snt[(size_t)i * c.max_seq_len + p] = sn[(size_t)p * half + i];
      }
    A(M->rope_cos_pm, (int64_t)cst.size());
    A(M->rope_sin_pm, (int64_t)snt.size());
    cudaMemcpy(M->rope_cos_pm, cst.data(), cst.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemcpy(M->rope_sin_pm, snt.data(), snt.size() * sizeof(float), cudaMemcpyHostToDevice);
  }
#undef A
  // weights
  std::vector<float> hp((size_t)NP);
  for (size_t i = 0; i < M->L.off.size(); ++i) {
    float* p = hp.data() + M->L.off[i];
    const int k = M->L.kind[i];
    if (k == K_MAT || k == K_EMB)
      fill_normal(p, M->L.size[i], seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(i + 1)), 0.f, init_std);
    else
      for (int64_t j = 0; j < M->L.size[i]; ++j) p[j] = (k == K_GAMMA) ? 1.f : 0.f;
  }
  cudaMemcpy(M->params, hp.data(), (size_t)NP * sizeof(float), cudaMemcpyHostToDevice);
  cudaMemset(M->m, 0, (size_t)NP * sizeof(float));
  cudaMemset(M->v, 0, (size_t)NP * sizeof(float));
  cudaMemset(M->grads, 0, (size_t)NP * sizeof(float));
  s = zl_f32_to_bf16(M->params, reinterpret_cast<zl_bf16*>(M->pbf), NP, nullptr);
  if (s != ZL_OK) return fail(s);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(zl::set_error(ZL_ECUDA, "model init: %s", cudaGetErrorString(e)));
  *out = M;
  return ZL_OK;
}

extern "C" zl_status zl_model_destroy(zl_model* M) {
  if (!M) return ZL_OK;
  if (M->graph_exec) cudaGraphExecDestroy(M->graph_exec);
  if (M->cap_stream) cudaStreamDestroy(M->cap_stream);
  for (cudaEvent_t ev : M->kt_ev) cudaEventDestroy(ev);
  if (M->dist.comm) {
    cudaStreamSynchronize(M->dist.comm_stream);
    ncclCommDestroy(M->dist.comm);
    for (auto ev : M->dist.ready_ev) cudaEventDestroy(ev);
    if (M->dist.done_ev) cudaEventDestroy(M->dist.done_ev);
    cudaStreamDestroy(M->dist.comm_stream);
  }
  for (void* p : M->allocs) cudaFree(p);
  delete M;
  return ZL_OK;
}

extern "C" zl_status zl_model_num_params(zl_model* M, int64_t* n) {
  if (!M || !n) return zl::set_error(ZL_EINVAL, "null argument");
  *n = M->L.total;
  return ZL_OK;
}
extern "C" zl_status zl_model_buffers(zl_model* M, float** params, float** grads, float** adam_m, float** adam_v) {
  if (!M) return zl::set_error(ZL_EINVAL, "null model");
  if (params) *params = M->params;
  if (grads) *grads = M->grads;
  if (adam_m) *adam_m = M->m;
  if (adam_v) *adam_v = M->v;
  return ZL_OK;
}
extern "C" zl_status zl_model_params_updated(zl_model* M, zl_stream s) {
  if (!M) return zl::set_error(ZL_EINVAL, "null model");
  return zl_f32_to_bf16(M->params, reinterpret_cast<zl_bf16*>(M->pbf), M->L.total, s);
}
extern "C" zl_status zl_model_set_optimizer(zl_model* M, const zl_adamw_config* o) {
  if (!M || !o) return zl::set_error(ZL_EINVAL, "null argument");
  M->opt = *o;
  return ZL_OK;
}
extern "C" zl_status zl_model_zero_grad(zl_model* M, zl_stream s) {
  if (!M) return zl::set_error(ZL_EINVAL, "null model");
  cudaError_t e = cudaMemsetAsync(M->grads, 0, (size_t)M->L.total * sizeof(float), (cudaStream_t)s);
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "zero_grad: %s", cudaGetErrorString(e));
  return ZL_OK;
}

namespace {
// zero_grad -> forward -> fused CE -> backward on `st` (gradient buckets are all-reduced on the
// side stream as they become final when a communicator is attached).
zl_status step_body(zl_model* M, const int32_t* ids, const int32_t* targets, int B, int S, float* loss_out,
                    cudaStream_t st) {
  M->launches = 0;
  M->dist.next_bucket = 0;
  const size_t kt_step = 4 * (size_t)M->cfg.num_layers;  // step-phase events follow the per-layer ones
  if (!M->kt_ev.empty()) zl::record_timing_event(M->kt_ev[kt_step], st);
  TRY(zl_model_zero_grad(M, st));
  M->launches++;
  TRY(forward(M, ids, B, S, nullptr, st));
  const int64_t T = (int64_t)B * S;
  TRY(zl_cross_entropy_fused_bf16(reinterpret_cast<zl_bf16*>(M->logits), targets, (int)T, M->cfg.vocab_size, 1e-8f,
                                  1.0f / (float)T, M->loss_rows, loss_out, st));
  M->launches += loss_out ? 2 : 1;
  TRY(backward(M, ids, B, S, st));
  if (!M->kt_ev.empty()) zl::record_timing_event(M->kt_ev[kt_step + 1], st);
  return ZL_OK;
}

// Replays (or captures, the second time a binding is seen) the step body as one CUDA graph.
zl_status step_graph(zl_model* M, const int32_t* ids, const int32_t* targets, int B, int S, float* loss_out,
                     cudaStream_t st) {
  const bool same = M->graph_exec && M->g_ids == ids && M->g_tgt == targets && M->g_loss == loss_out &&
                    M->g_B == B && M->g_S == S;
  M->dist.joined = false;
  if (same) {
    cudaError_t e = cudaGraphLaunch(M->graph_exec, st);
    if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "cudaGraphLaunch: %s", cudaGetErrorString(e));
    M->launches = M->g_launches;
    M->dist.joined = true;
    return ZL_OK;
  }
  const bool seen = M->g_ids == ids && M->g_tgt == targets && M->g_loss == loss_out && M->g_B == B && M->g_S == S;
  M->g_ids = ids; M->g_tgt = targets; M->g_loss = loss_out; M->g_B = B; M->g_S = S;
  if (!seen) return step_body(M, ids, targets, B, S, loss_out, st);  // first sighting: run eagerly (warm-up)
  if (M->graph_exec) { cudaGraphExecDestroy(M->graph_exec); M->graph_exec = nullptr; }
  if (!M->cap_stream) cudaStreamCreateWithFlags(&M->cap_stream, cudaStreamNonBlocking);
  cudaEvent_t ev;
  cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  cudaEventRecord(ev, st);
  cudaStreamWaitEvent(M->cap_stream, ev, 0);  // order capture-time work after the caller's stream
  cudaStreamSynchronize(M->cap_stream);
  cudaEventDestroy(ev);
  cudaError_t e = cudaStreamBeginCapture(M->cap_stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "cudaStreamBeginCapture: %s", cudaGetErrorString(e));
  zl_status body = step_body(M, ids, targets, B, S, loss_out, M->cap_stream);
  if (body == ZL_OK && M->dist.comm) {
    // the gradient all-reduces on the side stream rejoin the captured stream, so one graph launch
    // covers the whole exchange
    cudaEventRecord(M->dist.done_ev, M->dist.comm_stream);
    cudaStreamWaitEvent(M->cap_stream, M->dist.done_ev, 0);
  }
  cudaGraph_t graph = nullptr;
  e = cudaStreamEndCapture(M->cap_stream, &graph);
  if (body != ZL_OK) {
    if (graph) cudaGraphDestroy(graph);
    return body;
  }
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&M->graph_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    M->graph_exec = nullptr;
    return zl::set_error(ZL_ECUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
  }
  M->g_launches = M->launches;
  e = cudaGraphLaunch(M->graph_exec, st);
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "cudaGraphLaunch: %s", cudaGetErrorString(e));
  M->dist.joined = true;
  return ZL_OK;
}
}  // namespace

extern "C" zl_status zl_model_set_graph(zl_model* M, int enabled) {
  if (!M) return zl::set_error(ZL_EINVAL, "null model");
  M->use_graph = enabled;
  if (!enabled && M->graph_exec) {
    cudaGraphExecDestroy(M->graph_exec);
    M->graph_exec = nullptr;
  }
  return ZL_OK;
}

extern "C" zl_status zl_model_set_kernel_timing(zl_model* M, int enabled) {
  if (!M) return zl::set_error(ZL_EINVAL, "null model");
  if ((enabled != 0) == !M->kt_ev.empty()) return ZL_OK;
  cudaDeviceSynchronize();  // no recorded event may be pending when it is destroyed
  for (cudaEvent_t ev : M->kt_ev) cudaEventDestroy(ev);
  M->kt_ev.clear();
  M->kt_valid = false;
  if (enabled) {
    M->kt_ev.resize(4 * (size_t)M->cfg.num_layers + 3);
    for (auto& ev : M->kt_ev) {
      cudaError_t e = cudaEventCreate(&ev);
      if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "kernel timing: cudaEventCreate: %s", cudaGetErrorString(e));
    }
  }
  if (M->graph_exec) {  // the captured step must gain (or lose) its event nodes
    cudaGraphExecDestroy(M->graph_exec);
    M->graph_exec = nullptr;
  }
  return ZL_OK;
}

extern "C" zl_status zl_model_kernel_times(zl_model* M, float* attn_fwd_ms, float* attn_bwd_ms) {
  if (!M || !attn_fwd_ms || !attn_bwd_ms) return zl::set_error(ZL_EINVAL, "null argument");
  if (M->kt_ev.empty()) return zl::set_error(ZL_ESTATE, "kernel timing is off");
  if (!M->kt_valid) return zl::set_error(ZL_ESTATE, "kernel timing: no step has run since timing was enabled");
  const int L = M->cfg.num_layers;
  cudaError_t e = cudaEventSynchronize(M->kt_ev[4 * (L - 1) + 1]);  // forward of the last layer
  if (e == cudaSuccess) e = cudaEventSynchronize(M->kt_ev[3]);      // backward of layer 0 (last)
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "kernel timing: %s", cudaGetErrorString(e));
  double f = 0, b = 0;
  for (int l = 0; l < L; ++l) {
    float x = 0, y = 0;
    e = cudaEventElapsedTime(&x, M->kt_ev[4 * l], M->kt_ev[4 * l + 1]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&y, M->kt_ev[4 * l + 2], M->kt_ev[4 * l + 3]);
    if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "kernel timing: %s", cudaGetErrorString(e));
    f += x;
    b += y;
  }
  *attn_fwd_ms = (float)(f / L);
  *attn_bwd_ms = (float)(b / L);
  return ZL_OK;
}

extern "C" zl_status zl_model_step_times(zl_model* M, float* step_ms, float* exposed_exchange_ms) {
  if (!M || !step_ms || !exposed_exchange_ms) return zl::set_error(ZL_EINVAL, "null argument");
  if (M->kt_ev.empty()) return zl::set_error(ZL_ESTATE, "kernel timing is off");
  if (!M->kt_valid) return zl::set_error(ZL_ESTATE, "kernel timing: no step has run since timing was enabled");
  const size_t k = 4 * (size_t)M->cfg.num_layers;
  cudaError_t e = cudaEventSynchronize(M->kt_ev[k + 2]);
  float a = 0, b = 0;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&a, M->kt_ev[k], M->kt_ev[k + 2]);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&b, M->kt_ev[k + 1], M->kt_ev[k + 2]);
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "step timing: %s", cudaGetErrorString(e));
  *step_ms = a;
  *exposed_exchange_ms = b;
  return ZL_OK;
}

extern "C" zl_status zl_model_train_step(zl_model* M, const int32_t* ids, const int32_t* targets, int B, int S, float lr,
                                         int update, float* loss_out, zl_stream stream) {
  if (!M || !ids || !targets) return zl::set_error(ZL_EINVAL, "null argument");
  TRY(check_shape(M, B, S));
  cudaStream_t st = (cudaStream_t)stream;
  M->dist.joined = false;
  if (M->use_graph) TRY(step_graph(M, ids, targets, B, S, loss_out, st));
  else TRY(step_body(M, ids, targets, B, S, loss_out, st));
  if (!M->kt_ev.empty()) {
    // step end: once the gradient exchange on the side stream has rejoined this stream
    if (M->dist.comm && !M->dist.joined) {
      cudaEventRecord(M->dist.done_ev, M->dist.comm_stream);
      cudaStreamWaitEvent(st, M->dist.done_ev, 0);
      M->dist.joined = true;
    }
    zl::record_timing_event(M->kt_ev[4 * (size_t)M->cfg.num_layers + 2], st);
    M->kt_valid = true;
  }
  if (update) TRY(adamw(M, lr, st));
  else if (M->dist.comm && !M->dist.joined) {
    cudaEventRecord(M->dist.done_ev, M->dist.comm_stream);
    cudaStreamWaitEvent(st, M->dist.done_ev, 0);
  }
  return zl::check_launch("train_step");
}

extern "C" zl_status zl_model_forward(zl_model* M, const int32_t* ids, int B, int S, float* logits, zl_stream stream) {
  if (!M || !ids || !logits) return zl::set_error(ZL_EINVAL, "null argument");
  TRY(check_shape(M, B, S));
  return forward(M, ids, B, S, logits, (cudaStream_t)stream);
}

namespace zl {
__global__ void f32_to_bf16_scaled_kernel(const float* __restrict__ x, bf16* __restrict__ y, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}
}  // namespace zl

extern "C" zl_status zl_model_backward(zl_model* M, const int32_t* ids, const float* d_logits, int B, int S,
                                       zl_stream stream) {
  if (!M || !ids || !d_logits) return zl::set_error(ZL_EINVAL, "null argument");
  if (B != M->last_B || S != M->last_S)  // zerollm.cpp:205-208
    return zl::set_error(ZL_ESTATE, "Must call forward() with same batch_size and seq_len before backward()");
  cudaStream_t st = (cudaStream_t)stream;
  TRY(zl_f32_to_bf16(d_logits, reinterpret_cast<zl_bf16*>(M->logits), (int64_t)B * S * M->cfg.vocab_size, stream));
  M->dist.next_bucket = (int)M->dist.b_start.size();  // no collective on this path
  M->dist.joined = false;
  return backward(M, ids, B, S, st);
}

extern "C" zl_status zl_model_step(zl_model* M, float lr, zl_stream stream) {
  if (!M) return zl::set_error(ZL_EINVAL, "null model");
  return adamw(M, lr, (cudaStream_t)stream);
}

extern "C" zl_status zl_model_last_launches(zl_model* M, int* count) {
  if (!M || !count) return zl::set_error(ZL_EINVAL, "null argument");
  *count = M->launches;
  return ZL_OK;
}

// ------------------------------------------------------------------ data parallel
extern "C" zl_status zl_bucket_plan(const int64_t* tensor_offsets, const int64_t* tensor_sizes, int n_tensors,
                                    int64_t bucket_floats, int64_t* starts, int64_t* lens, int max_buckets,
                                    int* n_buckets) {
  if (!tensor_offsets || !tensor_sizes || n_tensors <= 0 || bucket_floats <= 0 || !n_buckets)
    return zl::set_error(ZL_EINVAL, "bucket_plan: invalid arguments");
  for (int i = 1; i < n_tensors; ++i)
    if (tensor_offsets[i] != tensor_offsets[i - 1] + tensor_sizes[i - 1])
      return zl::set_error(ZL_EINVAL, "bucket_plan: tensors must be contiguous and ordered");
  // Buckets are formed from the end of the arena, where backward finishes: the last bucket may hold
  // bucket_floats / 8, the one before it twice that, and so on up to bucket_floats, each closed at a
  // tensor boundary (a tensor larger than its bucket's share gets a bucket of its own; one larger
  // than bucket_floats is split into bucket_floats pieces).  What is still to be all-reduced when
  // backward ends is then the last tensors alone, not a whole bucket_floats of them.
  std::vector<std::pair<int64_t, int64_t>> rev;  // buckets, last first: (start, length)
  auto cap = [&](size_t j) {
    int64_t c = std::max<int64_t>(bucket_floats >> 3, 1);
    for (size_t k = 0; k < j && c < bucket_floats; ++k) c *= 2;
    return std::min(c, bucket_floats);
  };
  int64_t cur_end = tensor_offsets[n_tensors - 1] + tensor_sizes[n_tensors - 1], cur_len = 0;
  auto close = [&]() {
    if (cur_len > 0) rev.emplace_back(cur_end - cur_len, cur_len);
    cur_end -= cur_len;
    cur_len = 0;
  };
  for (int i = n_tensors - 1; i >= 0; --i) {
    int64_t sz = tensor_sizes[i];
    if (cur_len > 0 && cur_len + sz > cap(rev.size())) close();
    while (sz > bucket_floats) {  // pieces of bucket_floats from the tensor's end
      close();
      rev.emplace_back(cur_end - bucket_floats, bucket_floats);
      cur_end -= bucket_floats;
      sz -= bucket_floats;
    }
    cur_len += sz;
  }
  close();
  const int nb = (int)rev.size();
  for (int b = 0; b < nb && b < max_buckets; ++b) {
    if (starts) starts[b] = rev[nb - 1 - b].first;
    if (lens) lens[b] = rev[nb - 1 - b].second;
  }
  *n_buckets = nb;
  if (nb > max_buckets) return zl::set_error(ZL_EINVAL, "bucket_plan: more than %d buckets", max_buckets);
  return ZL_OK;
}

extern "C" zl_status zl_nccl_unique_id(void* id_out, size_t id_bytes) {
  if (!id_out || id_bytes < sizeof(ncclUniqueId)) return zl::set_error(ZL_EINVAL, "nccl id buffer too small");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return zl::set_error(ZL_ENCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  memcpy(id_out, &id, sizeof(id));
  return ZL_OK;
}

extern "C" zl_status zl_model_attach_nccl(zl_model* M, const void* id, int rank, int world, int64_t bucket_bytes) {
  if (!M || !id || world <= 0 || rank < 0 || rank >= world || bucket_bytes < 4)
    return zl::set_error(ZL_EINVAL, "attach_nccl: invalid arguments");
  if (M->dist.comm) return zl::set_error(ZL_ESTATE, "attach_nccl: already attached");
  DistState& D = M->dist;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = ncclCommInitRank(&D.comm, world, uid, rank);
  if (r != ncclSuccess) return zl::set_error(ZL_ENCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
  D.rank = rank;
  D.world = world;
  cudaStreamCreateWithFlags(&D.comm_stream, cudaStreamNonBlocking);
  std::vector<int64_t> st(4096), ln(4096);
  int nb = 0;
  TRY(zl_bucket_plan(M->L.off.data(), M->L.size.data(), (int)M->L.off.size(), bucket_bytes / 4, st.data(), ln.data(),
                     4096, &nb));
  D.b_start.assign(st.begin(), st.begin() + nb);
  D.b_len.assign(ln.begin(), ln.begin() + nb);
  D.ready_ev.resize(nb);
  for (auto& ev : D.ready_ev) cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  cudaEventCreateWithFlags(&D.done_ev, cudaEventDisableTiming);
  // identical initial weights on every rank: broadcast rank 0's arena (train_zerollm_dp.cpp:335-341)
  r = ncclBroadcast(M->params, M->params, (size_t)M->L.total, ncclFloat, 0, D.comm, D.comm_stream);
  if (r != ncclSuccess) return zl::set_error(ZL_ENCCL, "ncclBroadcast: %s", ncclGetErrorString(r));
  cudaStreamSynchronize(D.comm_stream);
  return zl_model_params_updated(M, nullptr);
}

namespace zl {
__global__ void checksum_kernel(const uint32_t* __restrict__ p, int64_t n, unsigned long long* out) {
  uint64_t h = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    h += (uint64_t)p[i] * (0x9E3779B97F4A7C15ull ^ (uint64_t)i);
  atomicAdd(out, (unsigned long long)h);
}
}  // namespace zl

extern "C" zl_status zl_model_param_checksum(zl_model* M, uint64_t* out, zl_stream s) {
  if (!M || !out) return zl::set_error(ZL_EINVAL, "null argument");
  unsigned long long* d = nullptr;
  // the checksum word lives in the spare tail of the workspace
  d = reinterpret_cast<unsigned long long*>(M->ws);
  cudaMemsetAsync(d, 0, sizeof(unsigned long long), (cudaStream_t)s);
  zl::checksum_kernel<<<592, 256, 0, (cudaStream_t)s>>>(reinterpret_cast<const uint32_t*>(M->params), M->L.total, d);
  unsigned long long h = 0;
  cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, (cudaStream_t)s);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)s);
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "checksum: %s", cudaGetErrorString(e));
  *out = h;
  return ZL_OK;
}

// ===================================================================== checkpoints
// The reference's directory layout (serializer.hpp:24-56; zerollm.cpp:334-425; the layers' save /
// load: embedding.cpp:255-285, transformer_decoder.cpp:148-160, transformer_block.cpp:218-232,
// mha.cpp:261-275, feedward.cpp:148-160, linear.cpp:215-250, layernorm.cpp:172-190): one raw fp32
// file per tensor under <dir>/<module path>/weights/, and <dir>/config.bin, the raw ZeroLLMConfig
// struct (zerollm_config.hpp:10-17).  The fused q|k|v matrix of this library is split into the
// reference's q_proj / k_proj / v_proj files.
namespace {
struct CkptEntry {
  std::string rel;
  int64_t off, count;
};

std::vector<CkptEntry> checkpoint_entries(const zl_model_config& c, const Layout& L) {
  std::vector<CkptEntry> e;
  const int64_t d = c.embed_dim, F = c.ff_hidden_dim, V = c.vocab_size;
  e.push_back({"embedding/weights/table.bin", L.emb, V * d});
  for (int l = 0; l < c.num_layers; ++l) {
    const auto& t = L.lay[l];
    const std::string b = "decoder/layer_" + std::to_string(l) + "/";
    const char* proj[3] = {"q_proj", "k_proj", "v_proj"};
    for (int j = 0; j < 3; ++j) {
      e.push_back({b + "self_attn/" + proj[j] + "/weights/weight.bin", t[L_WQKV] + j * d * d, d * d});
      if (c.bias) e.push_back({b + "self_attn/" + proj[j] + "/weights/bias.bin", t[L_BQKV] + j * d, d});
    }
    e.push_back({b + "self_attn/out_proj/weights/weight.bin", t[L_WO], d * d});
    if (c.bias) e.push_back({b + "self_attn/out_proj/weights/bias.bin", t[L_BO], d});
    e.push_back({b + "ln1/weights/gamma.bin", t[L_N1G], d});
    if (c.norm == 0) e.push_back({b + "ln1/weights/beta.bin", t[L_N1B], d});
    e.push_back({b + "ff/ff1/weights/weight.bin", t[L_W1], F * d});
    if (c.bias) e.push_back({b + "ff/ff1/weights/bias.bin", t[L_B1], F});
    e.push_back({b + "ff/ff2/weights/weight.bin", t[L_W2], d * F});
    if (c.bias) e.push_back({b + "ff/ff2/weights/bias.bin", t[L_B2], d});
    e.push_back({b + "ln2/weights/gamma.bin", t[L_N2G], d});
    if (c.norm == 0) e.push_back({b + "ln2/weights/beta.bin", t[L_N2B], d});
  }
  e.push_back({"output_ln/weights/gamma.bin", L.nog, d});
  if (c.norm == 0) e.push_back({"output_ln/weights/beta.bin", L.nob, d});
  if (!c.tied) e.push_back({"head/weights/weight.bin", L.head, V * d});  // no reference counterpart
  return e;
}

// config.bin: six int32 and a bool, padded to 28 bytes as the reference's compiler lays it out
struct RefConfigFile {
  int32_t vocab_size, embed_dim, num_layers, num_heads, ff_hidden_dim, max_seq_len;
  uint8_t with_grad, pad[3];
};
static_assert(sizeof(RefConfigFile) == 28, "config.bin layout");

bool write_file(const std::string& path, const void* data, size_t bytes) {
  FILE* f = fopen(path.c_str(), "wb");
  if (!f) return false;
  const bool ok = bytes == 0 || fwrite(data, 1, bytes, f) == bytes;
  return fclose(f) == 0 && ok;
}

// Reads exactly `bytes` bytes; false when the file is missing or has another size.
bool read_file(const std::string& path, void* data, size_t bytes) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  bool ok = fseek(f, 0, SEEK_END) == 0 && (size_t)ftell(f) == bytes && fseek(f, 0, SEEK_SET) == 0;
  ok = ok && (bytes == 0 || fread(data, 1, bytes, f) == bytes);
  fclose(f);
  return ok;
}

std::string topology_line(const zl_model_config& c) {
  char buf[160];
  snprintf(buf, sizeof buf, "norm=%d pos=%d tied=%d bias=%d eps=%.9g rope_base=%.9g\n", c.norm, c.pos, c.tied, c.bias,
           (double)c.eps, (double)c.rope_base);
  return buf;
}
}  // namespace

extern "C" zl_status zl_checkpoint_manifest(const zl_model_config* cfg, char* buf, int64_t cap, int64_t* len) {
  if (!cfg || !len) return zl::set_error(ZL_EINVAL, "checkpoint manifest: null argument");
  TRY(validate(*cfg));
  const Layout L = build_layout(*cfg);
  std::string s;
  for (const auto& e : checkpoint_entries(*cfg, L))
    s += e.rel + " " + std::to_string(e.off) + " " + std::to_string(e.count) + "\n";
  *len = (int64_t)s.size();
  if (buf && cap > 0) {
    const size_t n = std::min<size_t>((size_t)cap - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return ZL_OK;
}

extern "C" zl_status zl_model_save(zl_model* M, const char* dir, int with_optimizer) {
  if (!M || !dir) return zl::set_error(ZL_EINVAL, "save: null argument");
  namespace fs = std::filesystem;
  const std::string root(dir);
  const zl_model_config& c = M->cfg;
  std::vector<float> host((size_t)M->L.total);
  cudaError_t ce = cudaMemcpy(host.data(), M->params, host.size() * sizeof(float), cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return zl::set_error(ZL_ECUDA, "save: %s", cudaGetErrorString(ce));
  std::error_code ec;
  fs::create_directories(root, ec);
  if (ec) return zl::set_error(ZL_EIO, "save: cannot create %s: %s", root.c_str(), ec.message().c_str());
  const RefConfigFile rc{c.vocab_size, c.embed_dim, c.num_layers, c.num_heads, c.ff_hidden_dim, c.max_seq_len, 1, {0, 0, 0}};
  if (!write_file(root + "/config.bin", &rc, sizeof rc))
    return zl::set_error(ZL_EIO, "Failed to open file for writing: %s/config.bin", root.c_str());
  const std::string topo = topology_line(c);
  if (!write_file(root + "/zerollm_b200.txt", topo.data(), topo.size()))
    return zl::set_error(ZL_EIO, "Failed to open file for writing: %s/zerollm_b200.txt", root.c_str());
  for (const auto& e : checkpoint_entries(c, M->L)) {
    const std::string path = root + "/" + e.rel;
    fs::create_directories(fs::path(path).parent_path(), ec);
    if (ec || !write_file(path, host.data() + e.off, (size_t)e.count * sizeof(float)))
      return zl::set_error(ZL_EIO, "Failed to open file for writing: %s", path.c_str());
  }
  if (with_optimizer) {
    fs::create_directories(root + "/optimizer", ec);
    if (ec) return zl::set_error(ZL_EIO, "save: cannot create %s/optimizer", root.c_str());
    const char* names[2] = {"adamw_m.bin", "adamw_v.bin"};
    float* src[2] = {M->m, M->v};
    for (int i = 0; i < 2; ++i) {
      ce = cudaMemcpy(host.data(), src[i], host.size() * sizeof(float), cudaMemcpyDeviceToHost);
      if (ce != cudaSuccess) return zl::set_error(ZL_ECUDA, "save: %s", cudaGetErrorString(ce));
      if (!write_file(root + "/optimizer/" + names[i], host.data(), host.size() * sizeof(float)))
        return zl::set_error(ZL_EIO, "Failed to open file for writing: %s/optimizer/%s", root.c_str(), names[i]);
    }
    const int32_t t = M->t;
    if (!write_file(root + "/optimizer/state.bin", &t, sizeof t))
      return zl::set_error(ZL_EIO, "Failed to open file for writing: %s/optimizer/state.bin", root.c_str());
  }
  return ZL_OK;
}

extern "C" zl_status zl_model_load(zl_model* M, const char* dir, int with_optimizer) {
  if (!M || !dir) return zl::set_error(ZL_EINVAL, "load: null argument");
  const std::string root(dir);
  const zl_model_config& c = M->cfg;
  // config check as in zerollm.cpp:378-396: a missing config.bin is not an error
  RefConfigFile rc{};
  if (read_file(root + "/config.bin", &rc, sizeof rc)) {
    if (rc.embed_dim != c.embed_dim || rc.num_layers != c.num_layers || rc.vocab_size != c.vocab_size)
      return zl::set_error(ZL_EINVAL, "Model configuration mismatch detected during load (file: embed_dim=%d "
                                       "num_layers=%d vocab_size=%d)", rc.embed_dim, rc.num_layers, rc.vocab_size);
  }
  // this library's topology record, when present, must match too
  std::string topo(160, '\0');
  FILE* tf = fopen((root + "/zerollm_b200.txt").c_str(), "rb");
  if (tf) {
    const size_t n = fread(&topo[0], 1, topo.size() - 1, tf);
    fclose(tf);
    topo.resize(n);
    int nm = -1, ps = -1, td = -1, bs = -1;
    if (sscanf(topo.c_str(), "norm=%d pos=%d tied=%d bias=%d", &nm, &ps, &td, &bs) == 4 &&
        (nm != c.norm || ps != c.pos || td != c.tied || bs != c.bias))
      return zl::set_error(ZL_EINVAL, "load: checkpoint topology (norm=%d pos=%d tied=%d bias=%d) differs from the model",
                           nm, ps, td, bs);
  }
  std::vector<float> host((size_t)M->L.total);
  cudaError_t ce = cudaMemcpy(host.data(), M->params, host.size() * sizeof(float), cudaMemcpyDeviceToHost);
  if (ce != cudaSuccess) return zl::set_error(ZL_ECUDA, "load: %s", cudaGetErrorString(ce));
  for (const auto& e : checkpoint_entries(c, M->L)) {
    const std::string path = root + "/" + e.rel;
    if (!read_file(path, host.data() + e.off, (size_t)e.count * sizeof(float)))
      return zl::set_error(ZL_EIO, "Failed to read %lld floats from %s", (long long)e.count, path.c_str());
  }
  std::vector<float> mh, vh;
  int32_t t = 0;
  if (with_optimizer) {
    mh.resize(host.size());
    vh.resize(host.size());
    if (!read_file(root + "/optimizer/adamw_m.bin", mh.data(), mh.size() * sizeof(float)) ||
        !read_file(root + "/optimizer/adamw_v.bin", vh.data(), vh.size() * sizeof(float)) ||
        !read_file(root + "/optimizer/state.bin", &t, sizeof t))
      return zl::set_error(ZL_EIO, "load: optimizer state missing or of the wrong size under %s/optimizer", root.c_str());
  }
  // every file read: only now does the model change
  ce = cudaMemcpy(M->params, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (ce == cudaSuccess && with_optimizer) {
    ce = cudaMemcpy(M->m, mh.data(), mh.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(M->v, vh.data(), vh.size() * sizeof(float), cudaMemcpyHostToDevice);
    M->t = t;
  }
  if (ce != cudaSuccess) return zl::set_error(ZL_ECUDA, "load: %s", cudaGetErrorString(ce));
  return zl_model_params_updated(M, nullptr);
}
