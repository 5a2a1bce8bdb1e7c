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

// The same logits for many tokens on the tensor cores (kind::f16 with the
// hidden rows split into f16 hi + lo; f32 accumulation in the tensor core's
// order, not the shader's). workspace: lm_head_tc_workspace_bytes(n, D) bytes,
// 256-byte aligned; D % 64 == 0.
size_t lm_head_tc_workspace_bytes(int n, int D);
cudaError_t launch_lm_head_tc(const void* embed, int V, int D, const float* x, const float* gamma,
                              float eps, int n, float* logits, void* workspace, cudaStream_t s);

}  // namespace obn
