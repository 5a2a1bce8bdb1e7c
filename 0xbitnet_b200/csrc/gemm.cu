// gemm.cu — tcgen05 int8 GEMM (not yet enabled: every shape runs the dp4a path).
#include "gemm.h"
#include "obn_common.cuh"

namespace obn {

bool gemm_supported(const WeightView&, int) { return false; }

cudaError_t launch_gemm(const WeightView&, const int8_t*, const float*, const int32_t*, int,
                        float*, int32_t*, int, cudaStream_t) {
  return cudaErrorNotSupported;
}

cudaError_t read_and_clear_dev_error_gemm(uint32_t* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_dev_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(uint32_t));
}

}  // namespace obn
