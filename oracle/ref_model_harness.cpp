// ref_model_harness.cpp -- C entry points over the reference's own model code.
//
// TEST INFRASTRUCTURE ONLY.  Compiled with the unmodified reference sources
// (src/model/zerollm.cpp, src/layer/*.cpp, src/loss/cross_entropy.cpp,
// src/optimizer/*.cpp, src/utils/async_logger.cpp and src/kernel/cuda/*.cu,
// where they lie; Makefile target `refmodel`) into oracle/_ref/libzlrefmodel.so.
// GPU tests use it to have the reference itself write and read checkpoints
// (ZeroLLM::save / ZeroLLM::load, src/model/zerollm.cpp:334-425) and compute
// its forward loss (ZeroLLM::forward, zerollm.cpp:101-190, then
// CrossEntropyLoss::forward, src/loss/cross_entropy.cpp:23-79), so the
// library's checkpoint format and its reference-topology loss are pinned
// against the reference's own code.  Every function returns 0 on success,
// 1 if the reference threw, 2 on a CUDA error.
#include <cuda_runtime.h>

#include <exception>
#include <stdexcept>
#include <vector>

#include "cross_entropy.hpp"
#include "zerollm.hpp"
#include "zerollm_config.hpp"

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
// A reference model (forward only: with_grad = false) with the reference's own initialisation.
int zlrefm_create(int vocab, int dim, int layers, int heads, int ffn, int max_seq, void** out) {
  *out = nullptr;
  return run([&] { *out = new ZeroLLM(ZeroLLMConfig(vocab, dim, layers, heads, ffn, max_seq, false)); });
}
void zlrefm_destroy(void* m) { delete static_cast<ZeroLLM*>(m); }
int zlrefm_save(void* m, const char* dir) { return run([&] { static_cast<ZeroLLM*>(m)->save(dir); }); }
int zlrefm_load(void* m, const char* dir) { return run([&] { static_cast<ZeroLLM*>(m)->load(dir); }); }
// Mean cross-entropy of the model's logits on host ids / targets ([B * S] each).
int zlrefm_forward_loss(void* m, const int* ids, const int* targets, int B, int S, int vocab, float* loss) {
  int* d_ids = nullptr;
  int* d_tg = nullptr;
  float* d_logits = nullptr;
  const size_t T = (size_t)B * S;
  int rc = run([&] {
    if (cudaMalloc(&d_ids, T * sizeof(int)) != cudaSuccess || cudaMalloc(&d_tg, T * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&d_logits, T * vocab * sizeof(float)) != cudaSuccess)
      throw std::runtime_error("harness: cudaMalloc failed");
    cudaMemcpy(d_ids, ids, T * sizeof(int), cudaMemcpyHostToDevice);
    cudaMemcpy(d_tg, targets, T * sizeof(int), cudaMemcpyHostToDevice);
    static_cast<ZeroLLM*>(m)->forward(d_logits, d_ids, B, S);
    CrossEntropyLoss ce;
    *loss = ce.forward(d_logits, d_tg, (int)T, vocab);
  });
  cudaFree(d_ids);
  cudaFree(d_tg);
  cudaFree(d_logits);
  return rc;
}
}
