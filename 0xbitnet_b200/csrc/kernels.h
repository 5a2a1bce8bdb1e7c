// kernels.h — internal C++ launchers for the sm_100a kernels (not part of the C ABI).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace obn {

// Epilogue rounding order, as the two reference shaders write it.
enum EpilogueOrder : int {
  kOrderGemv = 0,  // (f32(acc) * s_w[m]) * s_x[t]      ternary_gemv.wgsl:95
  kOrderGemm = 1,  // f32(acc) * (s_w[m] * s_x[t])      ternary_gemm.wgsl:132-133
  // OR-ed into the order: y += the result (the residual add that follows the
  // layer in the reference, elementwise.wgsl op 0), y = y + val rounded once.
  kOutAccumulate = 2,
  // OR-ed into the order (k_gemm only): the weight rows are gated pairs (2i gate,
  // 2i + 1 up) and y[t, i] = act(gate) * up is written, [n, rows / 2]; the
  // activation is ReLU^2, or SiLU with kOutSilu.
  kOutGated = 4,
  kOutSilu = 8,
};

struct WeightView {
  const uint8_t* w;   // T16 layout (layout.cuh)
  const float* s_w;   // [m_pad] per-row scales
  int in_dim;         // K
  int out_dim;        // M
  int m_pad;          // M rounded up to 128
};

// I2_S rows [M][K/4] -> T16 (rows >= M filled with code 1).
cudaError_t launch_repack_i2s(const uint8_t* rows, uint8_t* t256, int M, int K, int m_pad,
                              cudaStream_t s);
// T16 -> I2_S rows [M][K/4].
cudaError_t launch_export_i2s(const uint8_t* t256, uint8_t* rows, int M, int K, cudaStream_t s);

// Fused RMSNorm (norm_w may be null) + absmax int8 quantize; qsum nullable.
cudaError_t launch_rmsnorm_quant(const float* x, const float* norm_w, float eps, int n, int d,
                                 int8_t* q, float* scales, int32_t* qsum, cudaStream_t s);
cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, int d, float* y,
                           cudaStream_t s);

// Gated FFN activation over interleaved gate|up outputs (activation.wgsl, then
// elementwise.wgsl multiply): y[i] = act(gu[2i]) * gu[2i + 1] for i < n * d
// (gu: [n, 2d], y: [n, d]); act 0 = ReLU^2 (max(0, g)^2), 1 = SiLU.
cudaError_t launch_act_mul(const float* gu, int n, int d, int act, float* y, cudaStream_t s);
// y[i] = act(x[i]) for i < count (y may alias x).
cudaError_t launch_act(const float* x, size_t count, int act, float* y, cudaStream_t s);

// elementwise.wgsl op 0: y[i] = a[i] + b[i] (residual add), count elements.
cudaError_t launch_add(const float* a, const float* b, size_t count, float* y, cudaStream_t s);

// embedding.wgsl: y[t, :] = f32(table[ids[t], :]) for t < n (ids >= vocab give 0);
// table [vocab, dim] binary16.
cudaError_t launch_embed_f16(const void* table, int vocab, int dim, const int32_t* ids, int n,
                             float* y, cudaStream_t s);

// Decode-path matmul on CUDA cores (dp4a) for any n (tokens in groups of 8).
// Writes y (float, `order` rounding) or, when acc != nullptr, exact int32 sums.
cudaError_t launch_gemv(const WeightView& W, const int8_t* q, const float* s_x,
                        const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                        cudaStream_t s);
// One-token BitLinear forward in a single kernel (RMSNorm when gamma != null,
// quantize, GEMV with ternary_gemv.wgsl's epilogue order). K <= kGemvMaxK.
// act >= 0: W is a gated layer (rows 2i gate, 2i + 1 up) and y[i] = act(gate) * up
// (0 = ReLU^2, 1 = SiLU) is written instead of the rows.
cudaError_t launch_bitlinear_n1(const WeightView& W, const float* gamma, float eps,
                                const float* x, float* y, cudaStream_t s,
                                int accumulate = 0, int act = -1);

// Largest K the GEMV kernels accept.
constexpr int kGemvMaxK = 16384;

// Batched decode on the warp-level int8 MMA (gemv_mma.cu) for 2..kMmaMaxTokens
// tokens: y (kOrderGemm rounding; kOutAccumulate / kOutGated / kOutSilu as for
// the GEMM) or, when acc != nullptr, exact int32 sums.
constexpr int kMmaMaxTokens = 16;
bool mma_gemv_supported(const WeightView& W, int n);
// The whole forward (RMSNorm when gamma != null, quantize, matmul) in one launch
// on the warp MMA for 2..kFusedMaxTokens tokens, in_dim <= kFusedMaxK and at
// least kFusedMinRows weight rows; y as launch_bitlinear_n1 writes it
// (accumulate: y +=; act >= 0: gated rows).
constexpr int kFusedMaxK = 3072;
constexpr int kFusedMaxTokens = 8;
constexpr int kFusedMinRows = 8192;
bool bitlinear_mma_supported(const WeightView& W, int n);
cudaError_t launch_bitlinear_mma(const WeightView& W, const float* gamma, float eps,
                                 const float* x, int n, float* y, int accumulate, int act,
                                 cudaStream_t s);
cudaError_t launch_mma_gemv(const WeightView& W, const int8_t* q, const float* s_x,
                            const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                            cudaStream_t s);

// SM count of the current device (cached per device).
int num_sms_cached();
// Raises a kernel's dynamic shared memory limit (once per kernel and device).
cudaError_t ensure_smem(const void* fn, size_t bytes);

// Device error words (one per translation unit): read and reset.
cudaError_t read_and_clear_dev_error_kernels(uint32_t* out);
cudaError_t read_and_clear_dev_error_gemm(uint32_t* out);
cudaError_t read_and_clear_dev_error_mma(uint32_t* out);
cudaError_t read_and_clear_dev_error(uint32_t* out);

}  // namespace obn
