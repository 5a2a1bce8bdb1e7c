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
#include "gemm.h"
#include "obn_common.cuh"
#include "tc05.cuh"

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

// ---------------------------------------------------------------------------
// Batched LM head on the tensor cores (tcgen05 kind::f16), for many tokens.
//
// Swap-AB like the ternary GEMM: the MMA's M is 128 vocabulary rows (A = the
// f16 table, TMA with 128-byte swizzle, 64 elements per K block), its N is BN
// tokens. The f32 hidden rows are split into f16 hi + lo (lo = f16(y - hi)):
// a row times hi plus the same row times lo is the f32 product to 2^-22 of
// |y|, so each K block issues its 4 MMAs (K = 16) twice, once per half, into
// the same f32 accumulator. The order of the f32 sums is the tensor core's,
// not the shader's: this path is for batches (the reference only runs n = 1).
// ---------------------------------------------------------------------------
constexpr int kLmBM = 128;      // vocabulary rows per tile
constexpr int kLmBK = 64;       // f16 elements per K block (one 128-byte swizzle row)
constexpr int kLmStages = 4;
constexpr int kLmTcThreads = 256;  // warp 0 TMA, 1 MMA, 2 TMEM, 4-7 epilogue

struct LmSmem {
  uint64_t full[kLmStages];
  uint64_t empty[kLmStages];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort_flag;
};

template <int BN>
constexpr uint32_t idesc_f16() {  // D f32, A f16, B f16, both K-major
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kLmBM >> 4) << 24);
}

template <int BN>
__global__ __launch_bounds__(kLmTcThreads, 1) void k_lm_head_tc(
    const __grid_constant__ CUtensorMap tmap_e, const __grid_constant__ CUtensorMap tmap_hi,
    const __grid_constant__ CUtensorMap tmap_lo, int V, int N, int D,
    float* __restrict__ logits) {
  constexpr int kA = kLmBM * kLmBK * 2;  // 16 KB of table per stage
  constexpr int kB = BN * kLmBK * 2;     // per half
  constexpr int kStage = kA + 2 * kB;
  constexpr uint32_t kTmemCols = 2 * BN <= 128 ? 128 : 256;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  LmSmem* sm = reinterpret_cast<LmSmem*>(base + kLmStages * kStage);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int num_m = (V + kLmBM - 1) / kLmBM;
  const int tiles = num_m * ((N + BN - 1) / BN);
  const int nkb = D / kLmBK;
  if (tid == 0) {
    for (int s = 0; s < kLmStages; ++s) {
      mbar_init(&sm->full[s], 1);
      mbar_init(&sm->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm->accf[a], 1);
      mbar_init(&sm->acce[a], 4);
    }
    mbar_init(&sm->drain, 1);
    sm->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&sm->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm->tmem_base;
  pdl_launch_dependents();
  pdl_wait();  // the hi/lo rows come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !sm->abort_flag; t += gridDim.x) {
        const int mt = t % num_m, nt = t / num_m;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kLmStages;
          if (!wait_or_abort(sm, &sm->empty[s], ((it / kLmStages) & 1u) ^ 1u)) break;
          uint8_t* st = base + s * kStage;
          mbar_arrive_expect_tx(&sm->full[s], kStage);
          tma_load_2d(st, &tmap_e, kb * kLmBK, mt * kLmBM, &sm->full[s]);
          tma_load_2d(st + kA, &tmap_hi, kb * kLmBK, nt * BN, &sm->full[s]);
          tma_load_2d(st + kA + kB, &tmap_lo, kb * kLmBK, nt * BN, &sm->full[s]);
        }
      }
      // every copy this thread issued has landed before exit (bounded)
      for (int j = it > kLmStages ? it - kLmStages : 0; j < it; ++j)
        mbar_wait(&sm->full[j % kLmStages], (j / kLmStages) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t idesc = idesc_f16<BN>();
    int it = 0, ti = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok && !sm->abort_flag; t += gridDim.x, ++ti) {
      const int a = ti & 1;
      if (!wait_or_abort(sm, &sm->acce[a], ((ti >> 1) & 1u) ^ 1u)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + a * BN;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % kLmStages;
        if (!wait_or_abort(sm, &sm->full[s], (it / kLmStages) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = smem_u32(base + s * kStage);
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int kk = 0; kk < kLmBK / 16; ++kk)
              mma_f16(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sa + kA + half * kB + kk * 32),
                      idesc, (kb > 0 || half > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&sm->empty[s]);
        }
        __syncwarp();
      }
      if (ok && lane == 0) mma_commit(&sm->accf[a]);
      __syncwarp();
    }
    if (lane == 0) mma_commit(&sm->drain);
    __syncwarp();
    mbar_wait(&sm->drain, 0);
    __syncwarp();
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    int ti = 0;
    for (int t = blockIdx.x; t < tiles && !sm->abort_flag; t += gridDim.x, ++ti) {
      const int mt = t % num_m, nt = t / num_m;
      const int a = ti & 1;
      if (!wait_or_abort(sm, &sm->accf[a], (ti >> 1) & 1u)) break;
      tc_fence_after();
      const int m = mt * kLmBM + quarter * 32 + lane;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        uint32_t v[16];
        tmem_ld16(taddr + j0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = nt * BN + j0 + j;
          if (n < N && m < V) logits[static_cast<size_t>(n) * V + m] = __uint_as_float(v[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm->acce[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}

// Final RMSNorm (rmsnorm.wgsl order, as k_lm_head_f16) and the hi/lo f16 split
// of each hidden row: hi = f16(y), lo = f16(y - hi). One CTA per token.
__global__ __launch_bounds__(256) void k_lm_hilo(const float* __restrict__ x,
                                                 const float* __restrict__ gamma, float eps,
                                                 int D, __half* __restrict__ hi,
                                                 __half* __restrict__ lo) {
  __shared__ float shf[256];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const size_t t = blockIdx.x;
  const float* xr = x + t * D;
  float rms = 1.0f;
  if (gamma) {
    float part = 0.0f;
    for (int c = tid; c < D; c += 256) part = __fadd_rn(part, __fmul_rn(xr[c], xr[c]));
    const float total = tree_sum_256(part, shf);
    rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(D)), eps)));
  }
  for (int c = tid; c < D; c += 256) {
    const float y = gamma ? __fmul_rn(__fmul_rn(xr[c], rms), gamma[c]) : xr[c];
    const __half h = __float2half_rn(y);
    hi[t * D + c] = h;
    lo[t * D + c] = __float2half_rn(__fsub_rn(y, __half2float(h)));
  }
}

bool lm_map(CUtensorMap* map, const void* base, int rows, int D, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kLmBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  auto fn = tensor_map_encoder();
  return fn && fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch_tc(const void* embed, int V, int D, const __half* hi, const __half* lo, int n,
                      float* logits, cudaStream_t s) {
  CUtensorMap me, mh, ml;
  if (!lm_map(&me, embed, V, D, kLmBM) || !lm_map(&mh, hi, n, D, BN) ||
      !lm_map(&ml, lo, n, D, BN))
    return cudaErrorInvalidValue;
  constexpr size_t kStage = kLmBM * kLmBK * 2 + 2 * BN * kLmBK * 2;
  const size_t smem = 1024 + kLmStages * kStage + sizeof(LmSmem);
  auto kern = k_lm_head_tc<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((V + kLmBM - 1) / kLmBM) * ((n + BN - 1) / BN);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles < sms ? tiles : sms);
  cfg.blockDim = dim3(kLmTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, me, mh, ml, V, n, D, logits);
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

namespace obn {

size_t lm_head_tc_workspace_bytes(int n, int D) {
  const size_t half_bytes = (static_cast<size_t>(n) * D * 2 + 255) / 256 * 256;
  return 2 * half_bytes;
}

cudaError_t launch_lm_head_tc(const void* embed, int V, int D, const float* x, const float* gamma,
                              float eps, int n, float* logits, void* workspace, cudaStream_t s) {
  const size_t half_bytes = lm_head_tc_workspace_bytes(n, D) / 2;
  auto* hi = static_cast<__half*>(workspace);
  auto* lo = reinterpret_cast<__half*>(static_cast<uint8_t*>(workspace) + half_bytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_lm_hilo, x, gamma, eps, D, hi, lo);
  if (e != cudaSuccess) return e;
  return n <= 64 ? launch_tc<64>(embed, V, D, hi, lo, n, logits, s)
                 : launch_tc<128>(embed, V, D, hi, lo, n, logits, s);
}

}  // namespace obn
