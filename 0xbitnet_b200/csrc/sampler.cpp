// sampler.cpp — host-side next-token sampling (sampler.h).
#include "sampler.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <vector>

namespace obn {

void Sampler::reseed(uint64_t seed) {
  // splitmix64 expands the seed into the four state words (never all zero).
  for (int i = 0; i < 4; ++i) {
    seed += 0x9E3779B97F4A7C15ull;
    uint64_t z = seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    s_[i] = static_cast<uint32_t>((z ^ (z >> 31)) >> 16);
  }
  if ((s_[0] | s_[1] | s_[2] | s_[3]) == 0) s_[0] = 1;
}

float Sampler::uniform() {
  // xoshiro128+ (Blackman & Vigna); the top 24 bits of the sum give the float.
  const uint32_t result = s_[0] + s_[3];
  const uint32_t t = s_[1] << 9;
  s_[2] ^= s_[0];
  s_[3] ^= s_[1];
  s_[1] ^= s_[2];
  s_[0] ^= s_[3];
  s_[2] ^= t;
  s_[3] = (s_[3] << 11) | (s_[3] >> 21);
  return static_cast<float>(result >> 8) * (1.0f / 16777216.0f);
}

uint32_t argmax(const float* logits, size_t vocab) {
  size_t best = 0;
  for (size_t i = 1; i < vocab; ++i)
    if (logits[i] > logits[best]) best = i;
  return static_cast<uint32_t>(best);
}

uint32_t sample_logits(float* logits, size_t vocab, float temperature, size_t top_k,
                       float repeat_penalty, const uint32_t* recent, size_t n_recent, float u) {
  if (vocab == 0) return 0;
  if (repeat_penalty != 1.0f && n_recent > 0) {  // sampling.rs:14-27
    for (size_t k = 0; k < n_recent; ++k) {
      const size_t idx = recent[k];
      if (idx < vocab) {
        if (logits[idx] > 0.0f)
          logits[idx] /= repeat_penalty;
        else
          logits[idx] *= repeat_penalty;
      }
    }
  }
  if (!(temperature > 0.0f)) return argmax(logits, vocab);
  if (temperature != 1.0f) {  // sampling.rs:29-35
    const float inv_temp = 1.0f / temperature;
    for (size_t i = 0; i < vocab; ++i) logits[i] *= inv_temp;
  }
  bool masked = false;
  if (top_k > 0 && top_k < vocab) {  // sampling.rs:37-60: keep logits >= the k-th largest
    // A min-heap of the k largest values seen so far; its root is the threshold.
    std::vector<float> heap(logits, logits + top_k);
    std::make_heap(heap.begin(), heap.end(), std::greater<float>());
    for (size_t i = top_k; i < vocab; ++i) {
      if (logits[i] > heap.front()) {
        std::pop_heap(heap.begin(), heap.end(), std::greater<float>());
        heap.back() = logits[i];
        std::push_heap(heap.begin(), heap.end(), std::greater<float>());
      }
    }
    const float threshold = heap.front();
    for (size_t i = 0; i < vocab; ++i)
      if (logits[i] < threshold) logits[i] = -std::numeric_limits<float>::infinity();
    masked = true;
  }
  // sampling.rs:62-76: softmax (unnormalised) and the cumulative draw. A masked
  // logit's exp is exactly 0 (max_val is finite), so it is written without a call.
  float max_val = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < vocab; ++i) max_val = std::fmax(max_val, logits[i]);
  const bool finite_max = std::isfinite(max_val);
  float sum = 0.0f;
  for (size_t i = 0; i < vocab; ++i) {
    if (masked && finite_max && logits[i] == -std::numeric_limits<float>::infinity())
      logits[i] = 0.0f;
    else
      logits[i] = std::exp(logits[i] - max_val);
    sum += logits[i];
  }
  const float r = u * sum;
  float cumsum = 0.0f;
  for (size_t i = 0; i < vocab; ++i) {
    cumsum += logits[i];
    if (cumsum >= r) return static_cast<uint32_t>(i);
  }
  return static_cast<uint32_t>(vocab - 1);
}

uint32_t Sampler::sample(float* logits, size_t vocab, float temperature, size_t top_k,
                         float repeat_penalty, const uint32_t* recent, size_t n_recent) {
  return sample_logits(logits, vocab, temperature, top_k, repeat_penalty, recent, n_recent,
                       uniform());
}

}  // namespace obn
