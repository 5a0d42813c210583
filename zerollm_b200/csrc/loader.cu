// loader.cu -- token data pipeline: the reference's LLMDataLoader (src/runtime/dataloader.cpp:35-149)
// over stories held as one int32 token array with offsets, plus an asynchronous device feed (a host
// thread assembles batches into pinned buffers ahead of use; their host-to-device copies are enqueued
// on the caller's stream).
#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

#include "common.cuh"

struct zl_loader {
  std::vector<int32_t> tokens;
  std::vector<int64_t> offsets;                    // n_stories + 1
  std::vector<std::pair<int64_t, int64_t>> samples;  // (story, start position)
  int batch = 0, seq = 0;
  int32_t eos = 0, pad = 0;
  bool shuffle = false;
  std::mt19937_64 gen;
  int64_t cur = 0;  // next sample
  // asynchronous feed
  struct Slot {
    int32_t* host = nullptr;  // pinned [2][batch * seq]: ids, targets
    cudaEvent_t copied = nullptr;
    int count = 0;
    int state = 0;  // 0 free, 1 ready, 2 copy in flight
  };
  std::vector<Slot> slots;
  std::thread worker;
  std::mutex mu;
  std::condition_variable cv;
  bool stop = false, running = false;
  int dev = 0;
  int64_t next_fill = 0, next_use = 0;  // slot sequence numbers
};

namespace {
// dataloader.cpp:109-119: story tokens, then eos at the story's length, then pad
inline int32_t token_at(const zl_loader* L, int64_t story, int64_t pos) {
  const int64_t b = L->offsets[story], len = L->offsets[story + 1] - b;
  if (pos < len) return L->tokens[b + pos];
  return pos == len ? L->eos : L->pad;
}

// dataloader.cpp:125-149: up to `batch` samples from the current position
int fill_batch(zl_loader* L, int32_t* ids, int32_t* tg) {
  int count = 0;
  while (count < L->batch && L->cur < (int64_t)L->samples.size()) {
    const auto s = L->samples[L->cur++];
    int32_t* in = ids + (size_t)count * L->seq;
    int32_t* out = tg + (size_t)count * L->seq;
    for (int i = 0; i < L->seq; ++i) {
      in[i] = token_at(L, s.first, s.second + i);
      out[i] = token_at(L, s.first, s.second + i + 1);
    }
    ++count;
  }
  return count;
}

void stop_worker(zl_loader* L) {
  {
    std::lock_guard<std::mutex> g(L->mu);
    L->stop = true;
  }
  L->cv.notify_all();
  if (L->worker.joinable()) L->worker.join();
  L->stop = false;
  L->running = false;
  // copies still in flight must finish before their pinned buffers are refilled or freed
  for (auto& s : L->slots) {
    if (s.state == 2) cudaEventSynchronize(s.copied);
    s.state = 0;
    s.count = 0;
  }
  L->next_fill = L->next_use = 0;
}
}  // namespace

extern "C" zl_status zl_loader_create(const int32_t* tokens, const int64_t* offsets, int64_t n_stories, int batch,
                                      int seq_len, int32_t eos_id, int32_t pad_id, int shuffle, uint64_t seed,
                                      zl_loader** out) {
  if (!out || n_stories < 0 || batch <= 0 || seq_len <= 0 || (n_stories > 0 && (!tokens || !offsets)))
    return zl::set_error(ZL_EINVAL, "loader: bad arguments");
  for (int64_t i = 0; i < n_stories; ++i)
    if (offsets[i + 1] < offsets[i] || offsets[i] < 0) return zl::set_error(ZL_EINVAL, "loader: offsets must ascend");
  zl_loader* L = new zl_loader;
  const int64_t base = n_stories > 0 ? offsets[0] : 0, n_tok = n_stories > 0 ? offsets[n_stories] - base : 0;
  L->tokens.assign(tokens + base, tokens + base + n_tok);
  L->offsets.resize((size_t)n_stories + 1);
  for (int64_t i = 0; i <= n_stories; ++i) L->offsets[i] = n_stories > 0 ? offsets[i] - base : 0;
  L->batch = batch;
  L->seq = seq_len;
  L->eos = eos_id;
  L->pad = pad_id;
  L->shuffle = shuffle != 0;
  L->gen.seed(seed);
  // dataloader.cpp:57-66: a sample starts every seq_len positions of story + eos; empty stories add none
  for (int64_t i = 0; i < n_stories; ++i) {
    const int64_t len = L->offsets[i + 1] - L->offsets[i];
    if (len == 0) continue;
    for (int64_t p = 0; p < len + 1; p += seq_len) L->samples.emplace_back(i, p);
  }
  if (L->shuffle) std::shuffle(L->samples.begin(), L->samples.end(), L->gen);
  cudaGetDevice(&L->dev);
  *out = L;
  return ZL_OK;
}

extern "C" zl_status zl_loader_destroy(zl_loader* L) {
  if (!L) return ZL_OK;
  stop_worker(L);
  for (auto& s : L->slots) {
    if (s.host) cudaFreeHost(s.host);
    if (s.copied) cudaEventDestroy(s.copied);
  }
  delete L;
  return ZL_OK;
}

// dataloader.cpp:17-21: rewind and reshuffle
extern "C" zl_status zl_loader_reset(zl_loader* L) {
  if (!L) return zl::set_error(ZL_EINVAL, "loader: null");
  stop_worker(L);
  L->cur = 0;
  if (L->shuffle) std::shuffle(L->samples.begin(), L->samples.end(), L->gen);
  return ZL_OK;
}

extern "C" zl_status zl_loader_info(zl_loader* L, int64_t* samples, int64_t* batches) {
  if (!L) return zl::set_error(ZL_EINVAL, "loader: null");
  const int64_t n = (int64_t)L->samples.size();
  if (samples) *samples = n;
  if (batches) *batches = (n + L->batch - 1) / L->batch;  // dataloader.cpp:27-29
  return ZL_OK;
}

extern "C" zl_status zl_loader_next(zl_loader* L, int32_t* ids, int32_t* targets, int* count) {
  if (!L || !ids || !targets || !count) return zl::set_error(ZL_EINVAL, "loader: null argument");
  if (L->running) return zl::set_error(ZL_ESTATE, "loader: the device feed is running (zl_loader_reset stops it)");
  *count = fill_batch(L, ids, targets);
  return ZL_OK;
}

extern "C" zl_status zl_loader_start(zl_loader* L, int depth) {
  if (!L || depth <= 0 || depth > 64) return zl::set_error(ZL_EINVAL, "loader: depth must be in [1, 64]");
  stop_worker(L);
  const size_t per = (size_t)L->batch * L->seq;
  if ((int)L->slots.size() != depth) {
    for (auto& s : L->slots) {
      if (s.host) cudaFreeHost(s.host);
      if (s.copied) cudaEventDestroy(s.copied);
    }
    L->slots.assign(depth, {});
    for (auto& s : L->slots) {
      if (cudaHostAlloc(&s.host, 2 * per * sizeof(int32_t), cudaHostAllocDefault) != cudaSuccess ||
          cudaEventCreateWithFlags(&s.copied, cudaEventDisableTiming) != cudaSuccess)
        return zl::set_error(ZL_ENOMEM, "loader: pinned buffers");
    }
  }
  L->running = true;
  L->worker = std::thread([L, per]() {
    cudaSetDevice(L->dev);
    for (;;) {
      zl_loader::Slot* s = nullptr;
      {
        std::unique_lock<std::mutex> g(L->mu);
        L->cv.wait(g, [&] {
          if (L->stop) return true;
          zl_loader::Slot& c = L->slots[L->next_fill % L->slots.size()];
          return c.state != 1;  // free, or its copy may be complete
        });
        if (L->stop) return;
        s = &L->slots[L->next_fill % L->slots.size()];
      }
      if (s->state == 2) cudaEventSynchronize(s->copied);  // the consumer's copy has read this buffer
      const int n = fill_batch(L, s->host, s->host + per);
      {
        std::lock_guard<std::mutex> g(L->mu);
        s->count = n;
        s->state = 1;
        ++L->next_fill;
      }
      L->cv.notify_all();
      if (n == 0) return;  // end of the epoch: an empty batch marks it
    }
  });
  return ZL_OK;
}

extern "C" zl_status zl_loader_next_device(zl_loader* L, int32_t* d_ids, int32_t* d_targets, int* count,
                                           zl_stream stream) {
  if (!L || !d_ids || !d_targets || !count) return zl::set_error(ZL_EINVAL, "loader: null argument");
  if (!L->running) return zl::set_error(ZL_ESTATE, "loader: zl_loader_start first");
  zl_loader::Slot* s = nullptr;
  {
    std::unique_lock<std::mutex> g(L->mu);
    L->cv.wait(g, [&] { return L->next_use < L->next_fill; });
    s = &L->slots[L->next_use % L->slots.size()];
  }
  *count = s->count;
  cudaError_t e = cudaSuccess;
  if (s->count > 0) {
    const size_t per = (size_t)L->batch * L->seq, n = (size_t)s->count * L->seq;
    e = cudaMemcpyAsync(d_ids, s->host, n * sizeof(int32_t), cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(d_targets, s->host + per, n * sizeof(int32_t), cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaEventRecord(s->copied, (cudaStream_t)stream);
  }
  {
    std::lock_guard<std::mutex> g(L->mu);
    s->state = s->count > 0 ? 2 : 0;
    ++L->next_use;
  }
  L->cv.notify_all();
  if (e != cudaSuccess) return zl::set_error(ZL_ECUDA, "loader: %s", cudaGetErrorString(e));
  if (s->count == 0) L->running = false;  // epoch over: the worker has returned
  return ZL_OK;
}
