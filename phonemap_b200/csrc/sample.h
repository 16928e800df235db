// sample.h -- on-device sampling of a token from logits (sample.cu).
//
// The computation of ss_sample (SlipStream/src/core/tensor.c:363-451) for one
// logits vector, in one kernel launch on the caller's stream.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace ss {

struct SampleArgs {
  const float* logits = nullptr;  // [n], device
  int n = 0;
  float temperature = 0.0f, top_p = 1.0f;
  int top_k = 0;
  unsigned long long* rng = nullptr;  // device RNG state, advanced once when temperature > 0
  int* token = nullptr;               // device result
  // decode loop (seq_tokens null: no write): the token also goes to
  // seq_tokens[*d_pos] when *fixed_until <= *d_pos < ctx, and to seq_tokens[ctx]
  int* seq_tokens = nullptr;
  const int* d_pos = nullptr;
  const int* fixed_until = nullptr;
  int ctx = 0;
  void* scratch = nullptr;  // sample_scratch_bytes(n), device
  // several independent draws in one launch, one CTA each (seq_tokens must be
  // null): draw b reads logits + b * logits_stride, advances rng[b], writes
  // token[b * token_stride] and uses scratch + b * scratch_stride bytes
  int batch = 1;
  size_t logits_stride = 0;
  int token_stride = 0;
  size_t scratch_stride = 0;
};

// Device scratch one draw over n logits needs (probabilities and two key
// arrays of the sort).
size_t sample_scratch_bytes(int n);
// Largest n the kernel takes.
constexpr int kSampleMaxN = 1 << 24;
// Launches the sampler; returns the launch's error.
cudaError_t sample_launch(const SampleArgs& a, cudaStream_t s);

}  // namespace ss
