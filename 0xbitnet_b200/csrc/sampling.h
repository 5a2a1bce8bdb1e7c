// sampling.h — device-side top-k selection for next-token sampling (sampling.cu).
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace obn {

// Applies the repetition penalty of `recent` [n_recent] (device ids) to `logits`
// [V] in place, then writes every (index, value) whose value x — the logit
// times 1 / temperature (the logit itself when temperature is 1 or <= 0) — is
// at least the k-th largest x. Up to `cap` pairs (index, float bits of x) land
// in `out` in no particular order; *count (device) gets their full number, or
// cap + 1 when the ties at one slice's cut did not fit the candidate buffer
// (then the caller samples from the logits, which carry the penalty). Two
// launches; `scratch` holds select_topk_scratch_bytes(V) bytes.
size_t select_topk_scratch_bytes(int V);
cudaError_t launch_select_topk(float* logits, int V, const uint32_t* recent, int n_recent,
                               float penalty, float temperature, int k, uint2* out, int cap,
                               int* count, void* scratch, cudaStream_t s);

}  // namespace obn
