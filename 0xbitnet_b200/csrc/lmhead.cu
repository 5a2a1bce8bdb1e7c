// lmhead.cu — the f16 LM head GEMV (tied embedding or separate f16 head) behind
// the final RMSNorm, sm_100a.
//
// Reference: f32_matmul.wgsl:27-74 (packages/core/src/shaders/), dispatched by
// dispatch_lm_head_with after dispatch_final_norm (packages/rust/crates/
// oxbitnet/src/nn/model.rs:226-262, 393-430). Per logit the shader runs one
// 256-lane workgroup: lane t accumulates the d-pairs dh = t, t + 256, ... as
// acc += h[2dh] * e.x; acc += h[2dh+1] * e.y (two rounded products and adds per
// pair), then the halving tree partial[t] += partial[t + s], s = 128 .. 1.
//
// B200 form: one warp per embedding row, eight "virtual lanes" per real lane.
// Real lane l holds virtual lanes 4l+k and 128+4l+k (k < 4), so the words of
// virtual lanes 4l..4l+3 at pass i are one 16-byte load (u32 words
// 256i + 128h + 4l .. +3): a warp reads 512 contiguous bytes per load and the
// 5120-byte row (D = 2560) in 10 loads. The tree's strides 128, 2 and 1 stay
// inside a lane, 64 .. 4 pair lane l with lane l + 16 .. l + 1 (shuffles): the
// same pairing, so every logit is bit-identical to the shader's. The row stream
// is HBM-bound (656.7 MB per token for 128256 x 2560), read once through
// L1::no_allocate loads; the normalised hidden rows sit in shared memory and
// each CTA normalises them itself (rmsnorm.wgsl order: tree_sum_256).
#include "lmhead.h"
#include "obn_common.cuh"

#include <cuda_fp16.h>

namespace obn {
namespace {

constexpr int kLmThreads = 256;
constexpr int kLmWarps = kLmThreads / 32;

OBN_DEVINL uint4 ld_stream_v4(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

OBN_DEVINL float lo_half(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
OBN_DEVINL float hi_half(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// NT tokens per launch (ntok <= NT), their normalised rows in shared memory.
template <int NT>
__global__ __launch_bounds__(kLmThreads, 2) void k_lm_head_f16(const uint4* __restrict__ E, int V,
                                                            int D, const float* __restrict__ x,
                                                            const float* __restrict__ gamma,
                                                            float eps, int ntok,
                                                            float* __restrict__ logits) {
  extern __shared__ __align__(16) float sx[];  // [NT][D]
  __shared__ float shf[kLmThreads];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  for (int t = 0; t < ntok; ++t) {
    const float* xr = x + static_cast<size_t>(t) * D;
    float* yr = sx + static_cast<size_t>(t) * D;
    if (gamma) {  // rmsnorm.wgsl:40-62: rms = 1 / sqrt(mean(x^2) + eps); y = (x * rms) * w
      float part = 0.0f;
      for (int c = tid; c < D; c += kLmThreads) {
        const float v = xr[c];
        part = __fadd_rn(part, __fmul_rn(v, v));
      }
      const float total = tree_sum_256(part, shf);
      const float rms =
          __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(D)), eps)));
      for (int c = tid; c < D; c += kLmThreads) yr[c] = __fmul_rn(__fmul_rn(xr[c], rms), gamma[c]);
    } else {
      for (int c = tid; c < D; c += kLmThreads) yr[c] = xr[c];
    }
  }
  __syncthreads();

  const int lane = tid & 31, warp = tid >> 5;
  const int DH = D >> 1;                 // u32 words (f16 pairs) per row
  const int W4 = DH >> 2;                // 16-byte words per row
  const int nI = (DH + 255) >> 8;        // passes of 256 words
  for (int v = blockIdx.x * kLmWarps + warp; v < V; v += gridDim.x * kLmWarps) {
    const uint4* row = E + static_cast<size_t>(v) * W4;
    float a[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int j = 0; j < 8; ++j) a[t][j] = 0.0f;
    for (int i0 = 0; i0 < nI; i0 += 4) {
      // Up to 8 row loads in flight before the arithmetic that consumes them.
      uint4 w[4][2];
#pragma unroll
      for (int di = 0; di < 4; ++di)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int p0 = 256 * (i0 + di) + 128 * h + 4 * lane;
          w[di][h] = (i0 + di < nI && p0 < DH) ? ld_stream_v4(row + (p0 >> 2))
                                               : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
      for (int di = 0; di < 4; ++di)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int p0 = 256 * (i0 + di) + 128 * h + 4 * lane;
          if (i0 + di >= nI || p0 >= DH) continue;  // this virtual lane has no pair here
          const uint32_t wk[4] = {w[di][h].x, w[di][h].y, w[di][h].z, w[di][h].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float e0 = lo_half(wk[k]), e1 = hi_half(wk[k]);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t >= ntok) break;
              const float2 hv = *reinterpret_cast<const float2*>(
                  sx + static_cast<size_t>(t) * D + 2 * (p0 + k));
              float acc = a[t][h * 4 + k];
              acc = __fadd_rn(acc, __fmul_rn(hv.x, e0));
              acc = __fadd_rn(acc, __fmul_rn(hv.y, e1));
              a[t][h * 4 + k] = acc;
            }
          }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t >= ntok) break;
      float* b = a[t];
#pragma unroll
      for (int k = 0; k < 4; ++k) b[k] = __fadd_rn(b[k], b[k + 4]);  // stride 128
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1)  // strides 64 .. 4: lane l += lane l + s
#pragma unroll
        for (int k = 0; k < 4; ++k) b[k] = __fadd_rn(b[k], __shfl_down_sync(0xffffffffu, b[k], s));
      b[0] = __fadd_rn(b[0], b[2]);  // stride 2
      b[1] = __fadd_rn(b[1], b[3]);
      b[0] = __fadd_rn(b[0], b[1]);  // stride 1
      if (lane == 0) logits[static_cast<size_t>(t) * V + v] = b[0];
    }
  }
}

template <int NT>
cudaError_t launch_nt(const void* embed, int V, int D, const float* x, const float* gamma,
                      float eps, int ntok, float* logits, cudaStream_t s) {
  auto kern = k_lm_head_f16<NT>;
  const size_t smem = static_cast<size_t>(NT) * D * sizeof(float);
  if (smem + sizeof(float) * kLmThreads > 48 * 1024) {  // dynamic + the static tree buffer
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kLmThreads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int need = (V + kLmWarps - 1) / kLmWarps;
  const int grid = need < sms * per_sm ? need : sms * per_sm;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kLmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<const uint4*>(embed), V, D, x, gamma, eps,
                            ntok, logits);
}

}  // namespace

cudaError_t launch_lm_head_f16(const void* embed, int V, int D, const float* x,
                               const float* gamma, float eps, int n, float* logits,
                               cudaStream_t s) {
  // Tokens in chunks of at most 4 (each chunk streams the table once).
  for (int t0 = 0; t0 < n; t0 += kLmMaxTokensPerPass) {
    const int nt = n - t0 < kLmMaxTokensPerPass ? n - t0 : kLmMaxTokensPerPass;
    const float* xc = x + static_cast<size_t>(t0) * D;
    float* lc = logits + static_cast<size_t>(t0) * V;
    cudaError_t e = nt == 1   ? launch_nt<1>(embed, V, D, xc, gamma, eps, nt, lc, s)
                    : nt == 2 ? launch_nt<2>(embed, V, D, xc, gamma, eps, nt, lc, s)
                              : launch_nt<4>(embed, V, D, xc, gamma, eps, nt, lc, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace obn
