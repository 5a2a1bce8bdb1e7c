// gemm.h — prefill / batched-decode ternary GEMM on the tcgen05 tensor cores.
#pragma once

#include "kernels.h"

namespace obn {

// Smallest token count routed to the tensor-core GEMM, and to its split-K
// (thread-block cluster) form when the layer has few 128-row tiles.
constexpr int kGemmMinTokens = 16;
constexpr int kGemmMinSplitTokens = 4;

// True when launch_gemm handles this shape (otherwise the dp4a path runs).
bool gemm_supported(const WeightView& W, int n);

// y[t, m] (or exact int32 acc when acc != nullptr) for t < n, m < out_dim.
cudaError_t launch_gemm(const WeightView& W, const int8_t* q, const float* s_x,
                        const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                        cudaStream_t s);

}  // namespace obn
