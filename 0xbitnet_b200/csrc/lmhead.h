// lmhead.h — the f16 LM head GEMV behind the final RMSNorm (lmhead.cu).
#pragma once

#include <cuda_runtime.h>

namespace obn {

constexpr int kLmMaxTokensPerPass = 4;

// logits[t, v] = sum_d y[t, d] * f32(embed[v, d]) for t < n, v < V, with
// y = RMSNorm(x[t]) * gamma (gamma == nullptr: y = x). embed is [V, D] binary16,
// 16-byte aligned, D % 8 == 0; x [n, D] and logits [n, V] f32.
cudaError_t launch_lm_head_f16(const void* embed, int V, int D, const float* x,
                               const float* gamma, float eps, int n, float* logits,
                               cudaStream_t s);

}  // namespace obn
