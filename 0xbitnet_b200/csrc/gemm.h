// gemm.h — prefill / batched-decode ternary GEMM on the tcgen05 tensor cores.
#pragma once

#include <cuda.h>

#include "kernels.h"

namespace obn {

// Smallest token count routed to the tensor-core GEMM, and to its split-K
// (thread-block cluster) form when the layer has few 128-row tiles.
constexpr int kGemmMinTokens = 16;
constexpr int kGemmMinSplitTokens = 4;

// Output of a tensor-parallel (output-feature split) GEMM: this rank computes
// columns [col0, col0 + out_dim) of an [n][ldy] f32 output that every rank
// holds, and writes them into all of those outputs from its epilogue: one
// multimem store through `mc` (an NVLS multicast address bound to every rank's
// buffer) or, when mc is null, one store per rank through `ranks` (each rank's
// buffer as mapped on this device: peer stores over NVLink).
constexpr int kMaxGatherRanks = 8;
struct GatherOut {
  float* mc = nullptr;
  float* ranks[kMaxGatherRanks] = {};
  int world = 0;
  int ldy = 0;
  int col0 = 0;
  int vec4 = 0;  // ldy, col0, out_dim multiples of 4 and every base 16-byte aligned
};

// cuTensorMapEncodeTiled from the driver (null when unavailable).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();

// True when launch_gemm handles this shape (otherwise the dp4a path runs).
bool gemm_supported(const WeightView& W, int n);

// y[t, m] (or exact int32 acc when acc != nullptr) for t < n, m < out_dim.
cudaError_t launch_gemm(const WeightView& W, const int8_t* q, const float* s_x,
                        const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                        cudaStream_t s);

// The tensor-parallel gather form of the GEMM (n >= kGemmMinTokens).
cudaError_t launch_gemm_gather(const WeightView& W, const int8_t* q, const float* s_x,
                               const int32_t* qsum, int n, int order, const GatherOut& go,
                               cudaStream_t s);

}  // namespace obn
