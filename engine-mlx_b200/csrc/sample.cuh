// sample.cuh — temperature / top-k / top-p sampling on the device.
//
// Replaces the host sampler the served engine runs for temperature > 0
// (sample_from_logits + sample_token + SimpleRng,
// crates/serve/src/sampler.rs:50-202; called from generate.rs:53-60 and
// decode_eager.rs:179-185): no logits readback, no host sort.
#pragma once
#include "common.cuh"

namespace emx {

struct SampleArgs {
  const bf16* logits;  // [n] (the lm_head output)
  int n;
  float temperature;   // >= 1e-6 (below that the engine keeps the in-graph argmax)
  float top_p;         // in [0, 1]
  int top_k;           // 0: off
  unsigned long long* rng;  // xorshift64* state, advanced by one draw
  float* scratch;      // [n] probabilities
  int* tok_out;
  int* hist;           // optional: hist[*hist_n] = token, (*hist_n)++ (below hist_cap)
  int* hist_n;
  int hist_cap;
};

// SimpleRng::new (sampler.rs:56-59): seed 0 is replaced by a fixed constant.
inline unsigned long long sample_rng_seed(unsigned long long seed) { return seed ? seed : 0x9E3779B97F4A7C15ull; }

cudaError_t sample_launch(const SampleArgs& a, cudaStream_t st);

}  // namespace emx
