// sampler.h — next-token sampling on the host, as the reference samples.
//
// Restates packages/rust/crates/oxbitnet/src/sampling.rs:4-77 over the f32
// logits of the last position: repetition penalty over the recent window
// (llama.cpp style: divide positive logits, multiply the others; a token that
// occurs several times in the window is penalised that many times), then
// temperature (multiply by 1 / T), then top-k (every logit below the k-th
// largest becomes -inf; ties at the threshold stay), then softmax with the
// max subtracted and a draw r = u * sum, u uniform in [0, 1), returning the
// first index whose running sum reaches r (the last index if none does).
//
// Two deliberate differences: the uniform draw comes from a seedable
// generator (xoshiro128+, seeded per model) where the reference uses the
// thread RNG, and temperature <= 0 picks the arg-max (the reference's
// arithmetic turns every probability into NaN there and returns the last id).
#pragma once

#include <cstddef>
#include <cstdint>

namespace obn {

class Sampler {
 public:
  explicit Sampler(uint64_t seed = 0x0B17E7u) { reseed(seed); }
  void reseed(uint64_t seed);
  // Next uniform float in [0, 1) with 24 random bits.
  float uniform();

  // Samples from `logits` [vocab] (modified in place). `recent` holds the
  // window of previously generated ids (duplicates allowed).
  uint32_t sample(float* logits, size_t vocab, float temperature, size_t top_k,
                  float repeat_penalty, const uint32_t* recent, size_t n_recent);

 private:
  uint32_t s_[4];
};

// Index of the largest logit (the first one among equal maxima).
uint32_t argmax(const float* logits, size_t vocab);

// One sampling step with the uniform draw u in [0, 1) supplied.
uint32_t sample_logits(float* logits, size_t vocab, float temperature, size_t top_k,
                       float repeat_penalty, const uint32_t* recent, size_t n_recent, float u);

}  // namespace obn
