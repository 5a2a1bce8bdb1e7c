// kernels.cu — repack, fused RMSNorm+quantize and the dp4a decode GEMV (sm_100a).
//
// Bit-exactness contract (against the reference shaders):
//  * RMSNorm sums squares as 256 strided lane partials followed by the halving
//    tree of rmsnorm.wgsl:41-55, with explicitly rounded __fmul_rn/__fadd_rn so
//    nvcc cannot contract them into FMAs; rms = 1 / sqrt(mean + eps) with IEEE
//    sqrt and division; y = (x * rms) * w (rmsnorm.wgsl:57-61).
//  * Quantization: absmax (order-free), scale/inv with IEEE division and the
//    absmax == 0 selects of quantize.wgsl:59,68, q = clamp(rint(y * inv))
//    with round-half-even (WGSL round(), quantize.wgsl:71).
//  * The matmul is integer: sum_k c[m,k] q[t,k] - sum_k q[t,k] with codes
//    c = w + 1 in {0,1,2}, which equals sum_k w[m,k] q[t,k] exactly (any order).
//  * The epilogue rounds in the order of the shader the reference would have
//    dispatched (kernels.h: EpilogueOrder).
#include "kernels.h"

#include <cuda_fp16.h>

#include <cstdlib>
#include "layout.cuh"
#include "obn_common.cuh"

namespace obn {

int num_sms_cached();

namespace {

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// Repack / export
// ---------------------------------------------------------------------------
// One thread per 16-byte half, enumerated in destination order so the T16
// writes are contiguous: i = ((S*KB + b)*2 + h)*16 + r, row m = 16*S + r.
__global__ void k_repack(const uint8_t* __restrict__ rows, uint8_t* __restrict__ t, int M, int K,
                         int m_pad) {
  const int KB = K / kBlockK;
  const size_t total = static_cast<size_t>(m_pad) * KB * 2;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i % 16);
    size_t j = i / 16;
    const int h = static_cast<int>(j % 2);
    j /= 2;
    const int b = static_cast<int>(j % KB);
    const int S = static_cast<int>(j / KB);
    const int m = S * kSubRows + r;
    uint4 v = make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
    if (m < M)
      v = *reinterpret_cast<const uint4*>(rows + static_cast<size_t>(m) * (K / 4) + b * 32 + h * 16);
    *reinterpret_cast<uint4*>(t + i * 16) = v;
  }
}

// One thread per 16-byte half of the I2_S rows, in row order.
__global__ void k_export(const uint8_t* __restrict__ t, uint8_t* __restrict__ rows, int M, int K) {
  const int KB = K / kBlockK;
  const size_t total = static_cast<size_t>(M) * KB * 2;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int h = static_cast<int>(i % 2);
    const int b = static_cast<int>((i / 2) % KB);
    const int m = static_cast<int>(i / (2 * static_cast<size_t>(KB)));
    *reinterpret_cast<uint4*>(rows + i * 16) =
        *reinterpret_cast<const uint4*>(t + half_offset(m, b, h, KB));
  }
}

// ---------------------------------------------------------------------------
// Block reductions for 256 threads
// Max is order-independent: any reduction order gives the shader's result.
OBN_DEVINL float block_max_256(float v, float* sh) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = sh[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) r = fmaxf(r, sh[w]);
  __syncthreads();
  return r;
}

OBN_DEVINL int block_sum_int_256(int v, int* sh) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) r += sh[w];
  __syncthreads();
  return r;
}

OBN_DEVINL float norm_mul(float x, float rms, float g) { return __fmul_rn(__fmul_rn(x, rms), g); }

// quantize.wgsl:67-72 for four values: q = clamp(round(y * inv), -127, 127) with
// WGSL round() = round half to even. For |v| < 2^22, v + 1.5 * 2^23 rounded to
// nearest-even leaves round(v) in the low mantissa bits, so the low byte of the
// sum's bit pattern is q as an int8 and (bits - 0x4B400000) is q as an int. The
// clamp never binds: |y| <= absmax and inv = 127 / absmax rounded give
// |y * inv| <= 127 * (1 + 2^-23), which rounds to at most 127. (Finite inputs;
// the magic addition runs on the FMA pipe instead of the quarter-rate conversion
// unit.)
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t kRoundMagicBits = 0x4B400000u;
OBN_DEVINL uint32_t round_bits(float v) { return __float_as_uint(__fadd_rn(v, kRoundMagic)); }

OBN_DEVINL uint32_t quant4(float4 y, float inv, int& sum) {
  const uint32_t a = round_bits(__fmul_rn(y.x, inv));
  const uint32_t b = round_bits(__fmul_rn(y.y, inv));
  const uint32_t c = round_bits(__fmul_rn(y.z, inv));
  const uint32_t d = round_bits(__fmul_rn(y.w, inv));
  sum += static_cast<int>(a + b + c + d - 4u * kRoundMagicBits);
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// ---------------------------------------------------------------------------
// Fused RMSNorm + quantize: one 256-thread CTA per token (the shaders' shape).
// ---------------------------------------------------------------------------
template <bool NORM>
__global__ __launch_bounds__(256) void k_rmsnorm_quant(const float* __restrict__ x,
                                                       const float* __restrict__ w, float eps,
                                                       int d, int8_t* __restrict__ q,
                                                       float* __restrict__ scales,
                                                       int32_t* __restrict__ qsum) {
  __shared__ float shf[256];
  __shared__ int shi[8];
  pdl_launch_dependents();
  pdl_wait();  // x may be the previous kernel's output
  const int tid = threadIdx.x;
  const size_t row = blockIdx.x;
  const float* xr = x + row * d;
  float rms = 1.0f;
  if (NORM) {
    float part = 0.0f;  // rmsnorm.wgsl:41-45, lane tid owns columns tid + 256 j
    for (int col = tid; col < d; col += 256) {
      const float v = xr[col];
      part = __fadd_rn(part, __fmul_rn(v, v));
    }
    const float total = tree_sum_256(part, shf);
    rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(d)), eps)));
  }
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const int d4 = d / 4;
  float lmax = 0.0f;
  for (int c = tid; c < d4; c += 256) {
    float4 v = x4[c];
    if (NORM) {
      const float4 g = w4[c];
      v = make_float4(norm_mul(v.x, rms, g.x), norm_mul(v.y, rms, g.y), norm_mul(v.z, rms, g.z),
                      norm_mul(v.w, rms, g.w));
    }
    lmax = fmaxf(lmax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  const float absmax = block_max_256(lmax, shf);
  const float scale = absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, 127.0f);
  const float inv = absmax == 0.0f ? 0.0f : __fdiv_rn(127.0f, absmax);
  uint32_t* q4 = reinterpret_cast<uint32_t*>(q + row * d);
  int lsum = 0;
  for (int c = tid; c < d4; c += 256) {
    float4 v = x4[c];
    if (NORM) {
      const float4 g = w4[c];
      v = make_float4(norm_mul(v.x, rms, g.x), norm_mul(v.y, rms, g.y), norm_mul(v.z, rms, g.z),
                      norm_mul(v.w, rms, g.w));
    }
    q4[c] = quant4(v, inv, lsum);
  }
  const int total_q = block_sum_int_256(lsum, shi);
  if (tid == 0) {
    scales[row] = scale;
    if (qsum) qsum[row] = total_q;
  }
}

// Single-pass variant for d <= 256 * EPT: gamma is fetched into registers
// before the PDL wait (it never depends on earlier kernels), x is loaded once
// (thread t owns columns t + 256 j, the shaders' lane mapping), and the chain
// after the wait has three block barriers: the per-thread sums of squares meet
// in shared memory once and every warp finishes the shaders' halving tree and
// the scalar divisions itself (as k_bitlinear_n1 does), the warp maxima meet
// once and every thread derives the scale, the warp code sums meet once.
// Persistent over tokens (row, row + gridDim.x, ...): the next token's x is in
// flight while the current one is reduced, and gamma is loaded once per CTA.
// The shared slots need no extra barrier between tokens: each is rewritten only
// after a barrier that every reader of its previous contents has passed.
template <int EPT, bool NORM>
__global__ __launch_bounds__(256) void k_rmsnorm_quant_reg(const float* __restrict__ x,
                                                           const float* __restrict__ w, float eps,
                                                           int d, int n, int8_t* __restrict__ q,
                                                           float* __restrict__ scales,
                                                           int32_t* __restrict__ qsum) {
  __shared__ float sh_ss[256];
  __shared__ float sh_max[8];
  __shared__ int shi[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float g[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    g[j] = (NORM && col < d) ? w[col] : 1.0f;
  }
  pdl_launch_dependents();
  pdl_wait();  // x may be the previous kernel's output
  size_t row = blockIdx.x;
  if (row >= static_cast<size_t>(n)) return;  // uniform per CTA
  float xv[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    xv[j] = col < d ? x[row * d + col] : 0.0f;
  }
  for (;;) {
  const size_t next = row + gridDim.x;
  const bool more = next < static_cast<size_t>(n);
  float xn[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    xn[j] = (more && col < d) ? x[next * d + col] : 0.0f;
  }
  if (NORM) {
    float part = 0.0f;  // rmsnorm.wgsl:41-45
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (tid + 256 * j < d) part = __fadd_rn(part, __fmul_rn(xv[j], xv[j]));
    sh_ss[tid] = part;
    __syncthreads();
    // lane l: strides 128, 64, 32 of the tree for shader lane l, then 16 .. 1
    const float* p = sh_ss + lane;
    const float b0 = __fadd_rn(__fadd_rn(p[0], p[128]), __fadd_rn(p[64], p[192]));
    const float b1 = __fadd_rn(__fadd_rn(p[32], p[160]), __fadd_rn(p[96], p[224]));
    float tsum = __fadd_rn(b0, b1);
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1)
      tsum = __fadd_rn(tsum, __shfl_down_sync(0xffffffffu, tsum, s));
    const float total = __shfl_sync(0xffffffffu, tsum, 0);
    const float rms =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(d)), eps)));
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (tid + 256 * j < d) xv[j] = norm_mul(xv[j], rms, g[j]);
  }
  float lmax = 0.0f;
#pragma unroll
  for (int j = 0; j < EPT; ++j) lmax = fmaxf(lmax, fabsf(xv[j]));
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, s));
  if (lane == 0) sh_max[warp] = lmax;
  __syncthreads();
  float absmax = sh_max[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) absmax = fmaxf(absmax, sh_max[i]);
  const float inv = absmax == 0.0f ? 0.0f : __fdiv_rn(127.0f, absmax);
  int8_t* qr = q + row * d;
  int lsum = 0;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    if (col < d) {
      const int qi = static_cast<int>(round_bits(__fmul_rn(xv[j], inv)) - kRoundMagicBits);
      qr[col] = static_cast<int8_t>(qi);
      lsum += qi;
    }
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, s);
  if (lane == 0) shi[warp] = lsum;
  __syncthreads();
  if (tid == 0) {
    int t = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += shi[i];
    scales[row] = absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, 127.0f);
    if (qsum) qsum[row] = t;
  }
  if (!more) break;
  row = next;
#pragma unroll
  for (int j = 0; j < EPT; ++j) xv[j] = xn[j];
  }
}

// Fused RMSNorm + quantize for many tokens (prefill): 64 threads (two warps) per
// token, four tokens per 256-thread CTA, persistent over tokens.
//
// Thread l of a token loads the float4 at columns 4l + 256m (m = 0, 1, ...), so
// it owns the four shader lanes L = 4l + e of rmsnorm.wgsl / quantize.wgsl
// (lane L covers columns L + 256j) with their columns in the shader's order:
// each fold of squares is local and bit-identical. The halving tree
// (rmsnorm.wgsl:50-55) then needs one exchange: after the token's threads
// publish their four partials, each of the two warps folds stride 128 (thread l
// + 32) from shared memory and strides 64 .. 4 with shuffles (lane + 16 .. + 1,
// the same pairings), strides 2 and 1 inside the lane. Barriers are named
// 64-thread barriers per token (publish partials, publish the warps' max
// |value|, publish the warps' code sums); the quantized row is stored 4 bytes
// per column quad. gamma sits in shared memory, loaded once per CTA before the
// PDL wait.
constexpr int kTokThreads = 64;
constexpr int kTokPerCta = 4;
// Up to here one CTA per token (measured on B200: rows of 2560 columns 2.9 / 3.8
// against 3.6 / 4.1 us at 384 / 512 tokens, the 64-thread form ahead from 1024;
// wide rows take the 128-thread form above 256 tokens at every count measured).
constexpr int kQuantFewTokens = 640;
constexpr int kQuantFewTokensWide = 256;  // rows of kWideMinCols columns or more

OBN_DEVINL void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ORs a predicate over its `count` threads.
OBN_DEVINL bool named_bar_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, o;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred o, %2, %3, p;\n\tselp.u32 %0, 1, 0, o;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

template <int EPT4, bool NORM>
__global__ __launch_bounds__(256) void k_rmsnorm_quant_t64(const float* __restrict__ x,
                                                           const float* __restrict__ w, float eps,
                                                           int d, int n, int8_t* __restrict__ q,
                                                           float* __restrict__ scales,
                                                           int32_t* __restrict__ qsum) {
  // dynamic: the row buffer of each token slot [kTokPerCta][d], then gamma [d] (NORM)
  extern __shared__ __align__(16) float dyn[];
  __shared__ __align__(16) float4 part_s[kTokPerCta][kTokThreads];
  __shared__ float max_s[kTokPerCta][2];
  __shared__ int sum_s[kTokPerCta][2];
  __shared__ __align__(8) uint64_t row_bar[kTokPerCta];
  const int tid = threadIdx.x, slot = tid >> 6, l = tid & 63, lane = tid & 31, half = l >> 5;
  const int bar_id = 1 + slot;
  float* row_s = dyn + static_cast<size_t>(slot) * d;
  const float* g_s = dyn + static_cast<size_t>(kTokPerCta) * d;
  if (NORM)
    for (int i = 4 * tid; i < d; i += 4 * 256)
      *reinterpret_cast<float4*>(dyn + static_cast<size_t>(kTokPerCta) * d + i) =
          *reinterpret_cast<const float4*>(w + i);
  if (tid < kTokPerCta) mbar_init(&row_bar[tid], 1);
  fence_mbar_init();
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // x may be the previous kernel's output
  const size_t stride = static_cast<size_t>(gridDim.x) * kTokPerCta;
  const uint32_t row_bytes = static_cast<uint32_t>(d) * 4;
  size_t t = static_cast<size_t>(blockIdx.x) * kTokPerCta + slot;
  // the slot's first row; every later row is requested once the current one is in registers
  if (l == 0 && t < static_cast<size_t>(n)) {
    mbar_arrive_expect_tx(&row_bar[slot], row_bytes);
    bulk_g2s(row_s, x + t * d, row_bytes, &row_bar[slot]);
  }
  uint32_t phase = 0;
  bool failed = false;  // a row copy that never landed (recorded): the slot stops
  for (; t < static_cast<size_t>(n); t += stride, phase ^= 1u) {
    const bool got = mbar_wait(&row_bar[slot], phase);
    float4 xv[EPT4];
#pragma unroll
    for (int m = 0; m < EPT4; ++m) {
      const int c = 4 * l + 256 * m;
      xv[m] = c < d ? *reinterpret_cast<const float4*>(row_s + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const size_t tn = t + stride;
    auto request_next = [&] {  // after a slot barrier: every thread has its columns
      if (l == 0 && tn < static_cast<size_t>(n)) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&row_bar[slot], row_bytes);
        bulk_g2s(row_s, x + tn * d, row_bytes, &row_bar[slot]);
      }
    };
    float rms = 1.0f;
    if (NORM) {
      float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;  // shader lanes 4l .. 4l + 3
#pragma unroll
      for (int m = 0; m < EPT4; ++m) {
        if (4 * l + 256 * m < d) {
          p0 = __fadd_rn(p0, __fmul_rn(xv[m].x, xv[m].x));
          p1 = __fadd_rn(p1, __fmul_rn(xv[m].y, xv[m].y));
          p2 = __fadd_rn(p2, __fmul_rn(xv[m].z, xv[m].z));
          p3 = __fadd_rn(p3, __fmul_rn(xv[m].w, xv[m].w));
        }
      }
      part_s[slot][l] = make_float4(p0, p1, p2, p3);
      failed = named_bar_or(bar_id, kTokThreads, !got);  // the slot agrees on a timeout
      if (failed) break;
      request_next();
      const float4 a = part_s[slot][lane], b = part_s[slot][lane + 32];  // stride 128
      float v0 = __fadd_rn(a.x, b.x), v1 = __fadd_rn(a.y, b.y);
      float v2 = __fadd_rn(a.z, b.z), v3 = __fadd_rn(a.w, b.w);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {  // strides 64 .. 4
        v0 = __fadd_rn(v0, __shfl_down_sync(0xffffffffu, v0, o));
        v1 = __fadd_rn(v1, __shfl_down_sync(0xffffffffu, v1, o));
        v2 = __fadd_rn(v2, __shfl_down_sync(0xffffffffu, v2, o));
        v3 = __fadd_rn(v3, __shfl_down_sync(0xffffffffu, v3, o));
      }
      const float total =
          __shfl_sync(0xffffffffu, __fadd_rn(__fadd_rn(v0, v2), __fadd_rn(v1, v3)), 0);
      rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(d)), eps)));
    }
    float lmax = 0.0f;
#pragma unroll
    for (int m = 0; m < EPT4; ++m) {
      const int c = 4 * l + 256 * m;
      if (c < d) {
        if (NORM) {
          const float4 g = *reinterpret_cast<const float4*>(g_s + c);
          xv[m] = make_float4(norm_mul(xv[m].x, rms, g.x), norm_mul(xv[m].y, rms, g.y),
                              norm_mul(xv[m].z, rms, g.z), norm_mul(xv[m].w, rms, g.w));
        }
        lmax = fmaxf(lmax, fmaxf(fmaxf(fabsf(xv[m].x), fabsf(xv[m].y)),
                                 fmaxf(fabsf(xv[m].z), fabsf(xv[m].w))));
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) max_s[slot][half] = lmax;
    if (NORM) {
      named_bar(bar_id, kTokThreads);
    } else {
      failed = named_bar_or(bar_id, kTokThreads, !got);
      if (failed) break;
      request_next();
    }
    const float absmax = fmaxf(max_s[slot][0], max_s[slot][1]);
    const float inv = absmax == 0.0f ? 0.0f : __fdiv_rn(127.0f, absmax);
    int lsum = 0;
    uint32_t* qr = reinterpret_cast<uint32_t*>(q + t * d);
#pragma unroll
    for (int m = 0; m < EPT4; ++m) {
      const int c = 4 * l + 256 * m;
      if (c < d) qr[c >> 2] = quant4(xv[m], inv, lsum);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) sum_s[slot][half] = lsum;
    named_bar(bar_id, kTokThreads);
    if (l == 0) {
      scales[t] = absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, 127.0f);
      if (qsum) qsum[t] = sum_s[slot][0] + sum_s[slot][1];
    }
  }
  // a slot that stopped early may still have a row copy in flight: wait for it (bounded)
  if (l == 0 && failed) mbar_wait(&row_bar[slot], phase);
}

// Fused RMSNorm + quantize for many tokens of wide rows (prefill, d > 4096):
// 128 threads per token group, three groups per CTA, each group double-buffering
// its rows in shared memory, so a row is in flight while the previous one is
// processed and a row of 6912 floats costs 54 registers per thread instead of 108.
//
// Thread l of a group owns shader lanes 2l, 2l + 1 (float2 at columns 2l + 256m),
// each lane folding its columns in the shader's order. The halving tree
// (rmsnorm.wgsl:50-55): strides 128 and 64 from the group's published partials
// (every warp folds the same way, so each gets the total without another
// barrier), strides 32 .. 2 with shuffles (lane + 16 .. + 1), stride 1 inside the
// thread. Named 128-thread barriers per group: partials, the warps' max |value|,
// the warps' code sums. q is stored two bytes per column pair.
constexpr int kWideThreads = 128;
constexpr int kWideGroups = 3;
constexpr int kWideMinCols = 4097;  // narrower rows keep the 64-thread form

template <int EPT2, bool NORM>
__global__ __launch_bounds__(kWideThreads* kWideGroups, 1) void k_rmsnorm_quant_w128(
    const float* __restrict__ x, const float* __restrict__ w, float eps, int d, int n,
    int8_t* __restrict__ q, float* __restrict__ scales, int32_t* __restrict__ qsum) {
  // dynamic: two row buffers per group [kWideGroups][2][d], then gamma [d] (NORM)
  extern __shared__ __align__(16) float dyn[];
  __shared__ __align__(16) float2 part_s[kWideGroups][kWideThreads];
  __shared__ float max_s[kWideGroups][4];
  __shared__ int sum_s[kWideGroups][4];
  __shared__ __align__(8) uint64_t row_bar[kWideGroups][2];
  const int tid = threadIdx.x, grp = tid / kWideThreads, l = tid % kWideThreads;
  const int lane = tid & 31, wq = l >> 5;
  const int bar_id = 1 + grp;
  float* rows = dyn + static_cast<size_t>(2 * grp) * d;
  const float* g_s = dyn + static_cast<size_t>(2 * kWideGroups) * d;
  if (NORM)
    for (int i = 4 * tid; i < d; i += 4 * kWideThreads * kWideGroups)
      *reinterpret_cast<float4*>(dyn + static_cast<size_t>(2 * kWideGroups) * d + i) =
          *reinterpret_cast<const float4*>(w + i);
  if (tid < 2 * kWideGroups) mbar_init(&row_bar[tid >> 1][tid & 1], 1);
  fence_mbar_init();
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // x may be the previous kernel's output
  const size_t stride = static_cast<size_t>(gridDim.x) * kWideGroups;
  const uint32_t row_bytes = static_cast<uint32_t>(d) * 4;
  size_t t = static_cast<size_t>(blockIdx.x) * kWideGroups + grp;
  // the group's first two rows; each later row is requested into the buffer the
  // row two steps earlier has left (once every thread holds that row's columns)
  if (l == 0)
    for (int b = 0; b < 2; ++b) {
      const size_t tb = t + b * stride;
      if (tb < static_cast<size_t>(n)) {
        mbar_arrive_expect_tx(&row_bar[grp][b], row_bytes);
        bulk_g2s(rows + static_cast<size_t>(b) * d, x + tb * d, row_bytes, &row_bar[grp][b]);
      }
    }
  int i = 0;
  bool failed = false;  // a row copy that never landed (recorded): the group stops
  for (; t < static_cast<size_t>(n); t += stride, ++i) {
    const int b = i & 1;
    const uint32_t ph = static_cast<uint32_t>(i >> 1) & 1u;
    const bool got = mbar_wait(&row_bar[grp][b], ph);
    const float* row = rows + static_cast<size_t>(b) * d;
    float2 xv[EPT2];
#pragma unroll
    for (int m = 0; m < EPT2; ++m) {
      const int c = 2 * l + 256 * m;
      xv[m] = c < d ? *reinterpret_cast<const float2*>(row + c) : make_float2(0.f, 0.f);
    }
    const size_t tn = t + 2 * stride;
    auto request_next = [&] {  // after a group barrier: every thread has its columns
      if (l == 0 && tn < static_cast<size_t>(n)) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&row_bar[grp][b], row_bytes);
        bulk_g2s(rows + static_cast<size_t>(b) * d, x + tn * d, row_bytes, &row_bar[grp][b]);
      }
    };
    float rms = 1.0f;
    if (NORM) {
      float p0 = 0.f, p1 = 0.f;  // shader lanes 2l, 2l + 1
#pragma unroll
      for (int m = 0; m < EPT2; ++m) {
        if (2 * l + 256 * m < d) {
          p0 = __fadd_rn(p0, __fmul_rn(xv[m].x, xv[m].x));
          p1 = __fadd_rn(p1, __fmul_rn(xv[m].y, xv[m].y));
        }
      }
      part_s[grp][l] = make_float2(p0, p1);
      failed = named_bar_or(bar_id, kWideThreads, !got);  // the group agrees on a timeout
      if (failed) break;
      request_next();
      // stride 128: lanes 2j + e += lanes 2j + e + 128 (thread j + 64), for the
      // lanes of threads lane and lane + 32; stride 64 then folds the second pair
      const float2 a = part_s[grp][lane], a2 = part_s[grp][lane + 64];
      const float2 c = part_s[grp][lane + 32], c2 = part_s[grp][lane + 96];
      float v0 = __fadd_rn(a.x, a2.x), v1 = __fadd_rn(a.y, a2.y);
      const float w0 = __fadd_rn(c.x, c2.x), w1 = __fadd_rn(c.y, c2.y);
      v0 = __fadd_rn(v0, w0);
      v1 = __fadd_rn(v1, w1);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {  // strides 32 .. 2
        v0 = __fadd_rn(v0, __shfl_down_sync(0xffffffffu, v0, o));
        v1 = __fadd_rn(v1, __shfl_down_sync(0xffffffffu, v1, o));
      }
      const float total = __shfl_sync(0xffffffffu, __fadd_rn(v0, v1), 0);  // stride 1
      rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(d)), eps)));
    }
    float lmax = 0.0f;
#pragma unroll
    for (int m = 0; m < EPT2; ++m) {
      const int c = 2 * l + 256 * m;
      if (c < d) {
        if (NORM) {
          const float2 g = *reinterpret_cast<const float2*>(g_s + c);
          xv[m] = make_float2(norm_mul(xv[m].x, rms, g.x), norm_mul(xv[m].y, rms, g.y));
        }
        lmax = fmaxf(lmax, fmaxf(fabsf(xv[m].x), fabsf(xv[m].y)));
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) max_s[grp][wq] = lmax;
    if (NORM) {
      named_bar(bar_id, kWideThreads);
    } else {
      failed = named_bar_or(bar_id, kWideThreads, !got);
      if (failed) break;
      request_next();
    }
    const float absmax =
        fmaxf(fmaxf(max_s[grp][0], max_s[grp][1]), fmaxf(max_s[grp][2], max_s[grp][3]));
    const float inv = absmax == 0.0f ? 0.0f : __fdiv_rn(127.0f, absmax);
    int lsum = 0;
    uint16_t* qr = reinterpret_cast<uint16_t*>(q + t * d);
#pragma unroll
    for (int m = 0; m < EPT2; ++m) {
      const int c = 2 * l + 256 * m;
      if (c < d) {
        const uint32_t qa = round_bits(__fmul_rn(xv[m].x, inv));
        const uint32_t qb = round_bits(__fmul_rn(xv[m].y, inv));
        lsum += static_cast<int>(qa + qb - 2u * kRoundMagicBits);
        qr[c >> 1] = static_cast<uint16_t>(__byte_perm(qa, qb, 0x0040));
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) sum_s[grp][wq] = lsum;
    named_bar(bar_id, kWideThreads);
    if (l == 0) {
      scales[t] = absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, 127.0f);
      if (qsum) qsum[t] = (sum_s[grp][0] + sum_s[grp][1]) + (sum_s[grp][2] + sum_s[grp][3]);
    }
  }
  // a group that stopped early may still have row copies in flight: wait for them (bounded)
  if (l == 0 && failed) {
    mbar_wait(&row_bar[grp][i & 1], static_cast<uint32_t>(i >> 1) & 1u);
    if (t + stride < static_cast<size_t>(n))
      mbar_wait(&row_bar[grp][(i + 1) & 1], static_cast<uint32_t>((i + 1) >> 1) & 1u);
  }
}

// rmsnorm.wgsl alone.
__global__ __launch_bounds__(256) void k_rmsnorm(const float* __restrict__ x,
                                                 const float* __restrict__ w, float eps, int d,
                                                 float* __restrict__ y) {
  __shared__ float shf[256];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const size_t row = blockIdx.x;
  const float* xr = x + row * d;
  float part = 0.0f;
  for (int col = tid; col < d; col += 256) {
    const float v = xr[col];
    part = __fadd_rn(part, __fmul_rn(v, v));
  }
  const float total = tree_sum_256(part, shf);
  const float rms =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(d)), eps)));
  float* yr = y + row * d;
  for (int col = tid; col < d; col += 256) yr[col] = norm_mul(xr[col], rms, w[col]);
}

// ---------------------------------------------------------------------------
// Decode GEMV on CUDA cores.
//
// CTA = one 16-row subtile x NT tokens, kGemvWarps warps. Before waiting on
// the previous kernel (PDL), warp 0 bulk-copies the subtile's KB x 512 bytes
// of packed weights into shared memory: the weights never depend on earlier
// kernels, so their HBM stream overlaps the tail of the producer of q. Lane
// (h = lane/16, r = lane%16) owns row r's half h of every block; warps split
// the blocks. Per 16 bytes of weights and per token: 4 broadcast 16-byte
// activation loads and 16 dp4a, in two independent accumulation chains.
// ---------------------------------------------------------------------------
constexpr int kGemvWarps = 8;

// Accumulates sum_k c[r,k] q[t,k] for this lane's row r = lane%16 and half
// h = lane/16 over blocks first, first + stride, ... (codes c = w + 1).
//
// Group g of a packed byte sits at bits (6-2g); instead of shifting it down,
// the word is only masked (one LOP3) and fed to dp4a as unsigned bytes
// c_g << (6-2g). Each group keeps its own accumulator, an exact multiple of
// 4^(3-g), and the shifts are applied once at the end (exact; |acc| stays
// below 3*64*127*16384 < 2^31 for K <= 16384).
template <int NT>
OBN_DEVINL void subtile_dot(uint32_t w_s, uint32_t q_s, int ldq, int KB, int first, int stride,
                            int lane, int (&acc)[NT]) {
  int a[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int g = 0; g < 4; ++g) a[t][g] = 0;
  const uint32_t wbase = w_s + lane * 16;
  const uint32_t qbase = q_s + (lane >> 4) * 16;
#pragma unroll 2
  for (int b = first; b < KB; b += stride) {
    const uint4 wv = lds128(wbase + b * kSubtileBytes);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t mask = 0xC0C0C0C0u >> (2 * g);
      const uint32_t c0 = wv.x & mask, c1 = wv.y & mask, c2 = wv.z & mask, c3 = wv.w & mask;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint4 xa = lds128(qbase + t * ldq + b * kBlockK + 32 * g);
        a[t][g] = dp4a_us(c3, xa.w, dp4a_us(c2, xa.z, dp4a_us(c1, xa.y, dp4a_us(c0, xa.x, a[t][g]))));
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t)
    acc[t] += (a[t][0] >> 6) + (a[t][1] >> 4) + (a[t][2] >> 2) + a[t][3];
}

// Issues the bulk copy of subtile S's KB blocks (one contiguous KB*512-byte
// run) on `bar` (lane 0 of the calling warp), announcing `extra_bytes` more for
// copies the caller adds.
OBN_DEVINL void prefetch_subtile(uint8_t* w_s, const uint8_t* W, int S, int KB, uint64_t* bar,
                                 uint32_t extra_bytes, int lane) {
  if (lane == 0) {
    const uint32_t bytes = static_cast<uint32_t>(KB) * kSubtileBytes;
    mbar_arrive_expect_tx(bar, bytes + extra_bytes);
    bulk_g2s_hint(w_s, W + subtile_offset(S, 0, KB), bytes, bar, policy_evict_first());
  }
  __syncwarp();
}

template <int NT, bool ACC>
__global__ __launch_bounds__(kGemvWarps * 32) void k_gemv(
    const uint8_t* __restrict__ W, const float* __restrict__ s_w, const int8_t* __restrict__ q,
    const float* __restrict__ s_x, const int32_t* __restrict__ qsum, float* __restrict__ y,
    int32_t* __restrict__ acc_out, int M, int K, int n, int order) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int red[kGemvWarps][NT][16];
  __shared__ float sx_s[NT];
  __shared__ int qs_s[NT];

  const int KB = K / kBlockK;
  const int S = blockIdx.x;
  const int t0 = blockIdx.y * NT;
  const int nt = min(NT, n - t0);
  uint8_t* w_s = smem;
  uint8_t* q_s = smem + KB * kSubtileBytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) prefetch_subtile(w_s, W, S, KB, &bar, 0, lane);
  pdl_launch_dependents();
  pdl_wait();  // q / s_x / qsum come from the quantize kernel

  const int kc = K / 16;  // 16-byte chunks per token
  for (int i = tid; i < NT * kc; i += kGemvWarps * 32) {
    const int t = i / kc, c = i - t * kc;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < nt) v = reinterpret_cast<const uint4*>(q + static_cast<size_t>(t0 + t) * K)[c];
    reinterpret_cast<uint4*>(q_s)[i] = v;
  }
  if (tid < NT) {
    sx_s[tid] = (!ACC && tid < nt) ? s_x[t0 + tid] : 0.0f;  // s_x is null in ACC mode
    qs_s[tid] = tid < nt ? qsum[t0 + tid] : 0;
  }
  __syncthreads();

  const bool ok = mbar_wait(&bar, 0);
  if (!ok) mbar_wait(&bar, 0);  // copies may still be in flight: wait once more, bounded
  int acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0;
  if (ok) subtile_dot<NT>(smem_u32(w_s), smem_u32(q_s), K, KB, warp, kGemvWarps, lane, acc);
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], 16);
  if (lane < 16) {
#pragma unroll
    for (int t = 0; t < NT; ++t) red[warp][t][lane] = acc[t];
  }
  __syncthreads();
  if (tid < 16 * NT) {
    const int t = tid >> 4, r = tid & 15;
    const int m = S * kSubRows + r;
    if (ok && t < nt && m < M) {
      int a = -qs_s[t];
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) a += red[w][t][r];
      const size_t o = static_cast<size_t>(t0 + t) * M + m;
      if (ACC) {
        acc_out[o] = a;
      } else {
        const float fa = static_cast<float>(a);
        const float sw = s_w[m], sx = sx_s[t];
        const float val = (order & 1) == kOrderGemv ? __fmul_rn(__fmul_rn(fa, sw), sx)
                                                    : __fmul_rn(fa, __fmul_rn(sw, sx));
        y[o] = (order & kOutAccumulate) ? __fadd_rn(y[o], val) : val;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Single-token BitLinear in one kernel: RMSNorm + quantize + GEMV.
//
// One decode token leaves no work to share, so every CTA normalises and
// quantizes the token itself and the whole BitLinear is one launch and one
// dependent round trip. The grid spreads the layer's 16-row subtiles evenly over
// at most one CTA per SM (a CTA takes a contiguous run of up to NSUB subtiles,
// one bulk copy in the T16 layout), so every SM streams weights. Before the PDL
// wait a CTA fetches everything that does not depend on earlier kernels: its
// packed weights (bulk copy into shared memory), its row scales and, in
// registers, the RMSNorm gamma of the columns each thread owns. The grid keeps
// shared memory near a third of an SM, so the next launches' CTAs become
// resident, and start their own weight copies, while this one runs.
//
// After the wait the kernel is a chain of dependent steps with three block
// barriers:
//   A  thread t loads the columns t + 256j (the lane mapping of rmsnorm.wgsl /
//      quantize.wgsl), folds its sum of squares in the shader's order and
//      publishes it; every warp then finishes the shader's halving tree itself
//      (lane l folds strides 128, 64, 32 from eight partials, shuffles do 16..1)
//      and derives 1/rms, so no broadcast barrier follows;
//   B  each thread normalises its columns into shared memory and publishes its
//      warp's max |value|; after the barrier every thread derives the scale;
//   -  warp w then quantizes only the 128-column blocks b = w, w + 8, ... that
//      its own dot product consumes (the normalised values of those columns are
//      in shared memory since B), so the int8 row needs no block barrier, only
//      a warp sync; the warp's code sum is kept for the epilogue;
//   D  each warp's row partials (all of the CTA's subtiles over its blocks) meet
//      in shared memory; one thread per row sums them, subtracts the code sum
//      and applies ternary_gemv.wgsl:95's epilogue.
// Integer sums are exact in any order; every float step rounds as the shaders.
// ---------------------------------------------------------------------------
constexpr int kN1MaxCtaSmem = 100 * 1024;  // two launches' CTAs resident per SM

// Dynamic shared memory of k_bitlinear_n1 with room for `wslots` subtiles of
// packed weights, then the normalised row (f32) and the quantized row (int8).
inline size_t n1_smem_bytes(int K, int nsub) {
  return static_cast<size_t>(nsub) * (K / kBlockK) * kSubtileBytes + 5 * static_cast<size_t>(K);
}

template <int EPT, int NSUB>
__global__ __launch_bounds__(256) void k_bitlinear_n1(
    const uint8_t* __restrict__ W, const float* __restrict__ s_w,
    const float* __restrict__ gamma, float eps, const float* __restrict__ x,
    float* __restrict__ y, int M, int K, int accumulate, int act, int wslots) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float sh_ss[256];          // per thread: sum of squares of its columns
  __shared__ float sh_max[8];           // per warp: max |normalised x|
  __shared__ int red_q[8];              // per warp: code sum of its blocks
  __shared__ int red[8][NSUB][16];      // per warp: row partials

  const int KB = K / kBlockK;
  const int S_total = (M + kSubRows - 1) / kSubRows;
  const int s0 = static_cast<int>(static_cast<long long>(blockIdx.x) * S_total / gridDim.x);
  const int s1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * S_total / gridDim.x);
  const int ns = s1 - s0;  // 1 .. NSUB (the launcher sizes the grid)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool geom_ok = ns >= 1 && ns <= wslots && wslots <= NSUB;
  if (tid == 0 && !geom_ok) record_error(DEVERR_BAD_LAUNCH);
  if (!geom_ok) {  // uniform per CTA; still ordered after the preceding grid
    pdl_wait();
    return;
  }
  uint8_t* w_s = smem;                                                         // wslots * KB * 512
  float* xn_s = reinterpret_cast<float*>(smem + wslots * KB * kSubtileBytes);  // K floats
  uint8_t* q_s = reinterpret_cast<uint8_t*>(xn_s + K);                       // K bytes

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {  // the CTA's subtiles are one contiguous run in the T16 layout
    const uint32_t wbytes = static_cast<uint32_t>(ns * KB) * kSubtileBytes;
    mbar_arrive_expect_tx(&bar, wbytes);
    bulk_g2s_hint(w_s, W + subtile_offset(s0, 0, KB), wbytes, &bar, policy_evict_first());
  }
  const int row = s0 * kSubRows + tid;  // epilogue: thread t < 16 * ns owns row s0*16 + t
  const bool row_thread = tid < ns * kSubRows && row < M;
  const float sw = row_thread ? s_w[row] : 0.0f;
  float gv[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    gv[j] = (gamma != nullptr && col < K) ? gamma[col] : 1.0f;
  }
  pdl_launch_dependents();
  pdl_wait();  // x, and y when accumulating, may be the previous kernel's output

  float xv[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    xv[j] = col < K ? x[col] : 0.0f;
  }
  const float y_old = (accumulate && row_thread) ? y[row] : 0.0f;  // x != y (host check)

  // ---- A: sum of squares -> 1/rms
  float rms = 1.0f;
  if (gamma) {
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < EPT; ++j)
      if (tid + 256 * j < K) part = __fadd_rn(part, __fmul_rn(xv[j], xv[j]));
    sh_ss[tid] = part;
    __syncthreads();
    const float* p = sh_ss + lane;
    const float b0 = __fadd_rn(__fadd_rn(p[0], p[128]), __fadd_rn(p[64], p[192]));
    const float b1 = __fadd_rn(__fadd_rn(p[32], p[160]), __fadd_rn(p[96], p[224]));
    float tsum = __fadd_rn(b0, b1);
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1)
      tsum = __fadd_rn(tsum, __shfl_down_sync(0xffffffffu, tsum, s));
    const float total = __shfl_sync(0xffffffffu, tsum, 0);
    rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), eps)));
  }
  // ---- B: normalised row into shared memory, max |value|
  float lmax = 0.0f;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int col = tid + 256 * j;
    if (col < K) {
      const float v = gamma ? norm_mul(xv[j], rms, gv[j]) : xv[j];
      xn_s[col] = v;
      lmax = fmaxf(lmax, fabsf(v));
    }
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, s));
  if (lane == 0) sh_max[warp] = lmax;
  __syncthreads();
  float absmax = sh_max[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) absmax = fmaxf(absmax, sh_max[w]);
  const float inv = absmax == 0.0f ? 0.0f : __fdiv_rn(127.0f, absmax);

  // ---- the warp's own blocks: quantize (lane = 4 columns), warp sync
  int qpart = 0;
  for (int b = warp; b < KB; b += 8) {
    const float4 v = *reinterpret_cast<const float4*>(xn_s + b * kBlockK + 4 * lane);
    *reinterpret_cast<uint32_t*>(q_s + b * kBlockK + 4 * lane) = quant4(v, inv, qpart);
  }
  __syncwarp();

  // ---- dot: per block, the lane's 16-byte q chunks once, then every subtile
  int a[NSUB][4];
#pragma unroll
  for (int s = 0; s < NSUB; ++s)
#pragma unroll
    for (int g = 0; g < 4; ++g) a[s][g] = 0;
  const bool ok = mbar_wait(&bar, 0);  // the weights (normally landed long ago)
  if (!ok) mbar_wait(&bar, 0);         // copies may still be in flight: once more, bounded
  if (ok) {
    const uint32_t wl = smem_u32(w_s) + lane * 16;
    const uint32_t qb = smem_u32(q_s) + (lane >> 4) * 16;
    for (int b = warp; b < KB; b += 8) {
      uint4 xq[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) xq[g] = lds128(qb + b * kBlockK + 32 * g);
#pragma unroll
      for (int s = 0; s < NSUB; ++s) {
        if (s < ns) {
          const uint4 wv = lds128(wl + (s * KB + b) * kSubtileBytes);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t mask = 0xC0C0C0C0u >> (2 * g);
            a[s][g] = dp4a_us(wv.w & mask, xq[g].w, dp4a_us(wv.z & mask, xq[g].z,
                      dp4a_us(wv.y & mask, xq[g].y, dp4a_us(wv.x & mask, xq[g].x, a[s][g]))));
          }
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < NSUB; ++s) {
    if (s < ns) {
      int acc = (a[s][0] >> 6) + (a[s][1] >> 4) + (a[s][2] >> 2) + a[s][3];
      acc += __shfl_xor_sync(0xffffffffu, acc, 16);  // the two halves of the row
      if (lane < 16) red[warp][s][lane] = acc;
    }
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) qpart += __shfl_xor_sync(0xffffffffu, qpart, s);
  if (lane == 0) red_q[warp] = qpart;
  __syncthreads();

  // ---- D: one thread per row (rows of a gated pair are adjacent lanes)
  if (tid < NSUB * kSubRows) {
    float val = 0.0f;
    if (row_thread && ok) {
      const int sb = tid >> 4, r = tid & 15;
      int acc = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) acc += red[w][sb][r] - red_q[w];
      const float scale = absmax == 0.0f ? 1.0f : __fdiv_rn(absmax, 127.0f);
      // ternary_gemv.wgsl:95 order: (f32(acc) * s_w) * s_x
      val = __fmul_rn(__fmul_rn(static_cast<float>(acc), sw), scale);
    }
    if (act < 0) {
      if (row_thread && ok) y[row] = accumulate ? __fadd_rn(y_old, val) : val;
    } else {
      // Gated layer (rows 2i = gate, 2i + 1 = up of feature i, an even row count):
      // the even lane forms act(gate) * up as the separate activation pass would.
      const float up = __shfl_down_sync(0xffffffffu, val, 1);
      if (row_thread && ok && (tid & 1) == 0) y[row >> 1] = __fmul_rn(gate_act(act, val), up);
    }
  }
}

}  // namespace

// Raises a kernel's dynamic shared memory limit once per (kernel, device) to the
// largest size requested so far.
struct SmemCfg {
  const void* fn;
  int dev;
  size_t bytes;
};
cudaError_t ensure_smem(const void* fn, size_t bytes) {
  static SmemCfg table[256];
  static int used = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  for (int i = 0; i < used; ++i)
    if (table[i].fn == fn && table[i].dev == dev) {
      if (table[i].bytes >= bytes) return cudaSuccess;
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
      if (e == cudaSuccess) table[i].bytes = bytes;
      return e;
    }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess && used < 256) table[used++] = SmemCfg{fn, dev, bytes};
  return e;
}

namespace {

template <int NT, bool ACC>
cudaError_t gemv_nt(const WeightView& W, const int8_t* q, const float* s_x, const int32_t* qsum,
                    int n, float* y, int32_t* acc, int order, cudaStream_t s) {
  const int K = W.in_dim;
  const size_t smem = static_cast<size_t>(K / kBlockK) * kSubtileBytes + static_cast<size_t>(NT) * K;
  auto kern = k_gemv<NT, ACC>;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  dim3 grid((W.out_dim + kSubRows - 1) / kSubRows, (n + NT - 1) / NT);
  return launch_pdl(kern, grid, dim3(kGemvWarps * 32), smem, s, W.w, W.s_w, q, s_x, qsum, y, acc,
                    W.out_dim, K, n, order);
}

template <int EPT, int NSUB>
cudaError_t bitlinear_n1_run(const WeightView& W, const float* gamma, float eps, const float* x,
                             float* y, int accumulate, int act, int grid, int wslots,
                             cudaStream_t s) {
  const int K = W.in_dim;
  const size_t smem = n1_smem_bytes(K, wslots);
  auto kern = k_bitlinear_n1<EPT, NSUB>;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(grid), dim3(256), smem, s, W.w, W.s_w, gamma, eps, x, y,
                    W.out_dim, K, accumulate, act, wslots);
}

// Grid of the single-token kernel: the layer's 16-row subtiles spread evenly over
// one CTA per SM (more CTAs only when a CTA's share would not fit its shared
// memory budget); subtiles per CTA <= 2 or <= 8 picks the kernel's register tile.
template <int EPT>
cudaError_t bitlinear_n1_ept(const WeightView& W, const float* gamma, float eps, const float* x,
                             float* y, int accumulate, int act, cudaStream_t s) {
  const int K = W.in_dim;
  const int KB = K / kBlockK;
  const int S_total = (W.out_dim + kSubRows - 1) / kSubRows;
  const long long budget = kN1MaxCtaSmem - 5LL * K;
  int cap = budget > 0 ? static_cast<int>(budget / (static_cast<long long>(KB) * kSubtileBytes)) : 1;
  cap = cap < 1 ? 1 : cap > 8 ? 8 : cap;
  int grid = num_sms_cached();
  if (grid > S_total) grid = S_total;
  if ((S_total + grid - 1) / grid > cap) grid = (S_total + cap - 1) / cap;
  const int per_cta = (S_total + grid - 1) / grid;  // the most subtiles any CTA takes
  if (per_cta <= 2)
    return bitlinear_n1_run<EPT, 2>(W, gamma, eps, x, y, accumulate, act, grid, per_cta, s);
  return bitlinear_n1_run<EPT, 8>(W, gamma, eps, x, y, accumulate, act, grid, per_cta, s);
}

template <bool ACC>
cudaError_t gemv_dispatch(const WeightView& W, const int8_t* q, const float* s_x,
                          const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                          cudaStream_t s) {
  switch (n) {
    case 1: return gemv_nt<1, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    case 2: return gemv_nt<2, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    case 3: return gemv_nt<3, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    case 4: return gemv_nt<4, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    case 5: return gemv_nt<5, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    case 6: return gemv_nt<6, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    case 7: return gemv_nt<7, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
    default: return gemv_nt<8, ACC>(W, q, s_x, qsum, n, y, acc, order, s);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
static int grid_for(size_t work, int block) {
  size_t g = (work + block - 1) / block;
  if (g > 148 * 32) g = 148 * 32;
  return static_cast<int>(g < 1 ? 1 : g);
}

cudaError_t launch_repack_i2s(const uint8_t* rows, uint8_t* t256, int M, int K, int m_pad,
                              cudaStream_t s) {
  const size_t work = static_cast<size_t>(m_pad) * (K / kBlockK) * 2;
  k_repack<<<grid_for(work, 256), 256, 0, s>>>(rows, t256, M, K, m_pad);
  return cudaGetLastError();
}

cudaError_t launch_export_i2s(const uint8_t* t256, uint8_t* rows, int M, int K, cudaStream_t s) {
  const size_t work = static_cast<size_t>(M) * (K / kBlockK) * 2;
  k_export<<<grid_for(work, 256), 256, 0, s>>>(t256, rows, M, K);
  return cudaGetLastError();
}

// SM count of the current device (cached per device).
int num_sms_cached() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] ? sms[dev] : 148;
}

template <int EPT>
cudaError_t rmsnorm_quant_ept(const float* x, const float* norm_w, float eps, int n, int d,
                              int8_t* q, float* scales, int32_t* qsum, cudaStream_t s) {
  auto kern = norm_w ? k_rmsnorm_quant_reg<EPT, true> : k_rmsnorm_quant_reg<EPT, false>;
  // One CTA per token up to the resident capacity, then persistent CTAs.
  static int cap[2] = {0, 0};
  int& c = cap[norm_w ? 1 : 0];
  if (c == 0) {
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0);
    if (e != cudaSuccess) return e;
    c = (per_sm > 0 ? per_sm : 1) * num_sms_cached();
  }
  const int grid = n < c ? n : c;
  return launch_pdl(kern, dim3(grid), dim3(256), 0, s, x, norm_w, eps, d, n, q, scales, qsum);
}

template <int EPT4>
cudaError_t rmsnorm_quant_t64(const float* x, const float* norm_w, float eps, int n, int d,
                              int8_t* q, float* scales, int32_t* qsum, cudaStream_t s) {
  auto kern = norm_w ? k_rmsnorm_quant_t64<EPT4, true> : k_rmsnorm_quant_t64<EPT4, false>;
  const size_t smem = sizeof(float) * static_cast<size_t>(d) * (kTokPerCta + (norm_w ? 1 : 0));
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  // four tokens per CTA up to the resident capacity, then persistent CTAs
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem);
  if (e != cudaSuccess) return e;
  const int cap = (per_sm > 0 ? per_sm : 1) * num_sms_cached();
  const int want = (n + kTokPerCta - 1) / kTokPerCta;
  return launch_pdl(kern, dim3(want < cap ? want : cap), dim3(256), smem, s, x, norm_w, eps, d, n,
                    q, scales, qsum);
}

template <int EPT2>
cudaError_t rmsnorm_quant_w128(const float* x, const float* norm_w, float eps, int n, int d,
                               int8_t* q, float* scales, int32_t* qsum, cudaStream_t s) {
  auto kern = norm_w ? k_rmsnorm_quant_w128<EPT2, true> : k_rmsnorm_quant_w128<EPT2, false>;
  const size_t smem = sizeof(float) * static_cast<size_t>(d) * (2 * kWideGroups + (norm_w ? 1 : 0));
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWideThreads * kWideGroups, smem);
  if (e != cudaSuccess) return e;
  const int cap = (per_sm > 0 ? per_sm : 1) * num_sms_cached();
  const int want = (n + kWideGroups - 1) / kWideGroups;
  return launch_pdl(kern, dim3(want < cap ? want : cap), dim3(kWideThreads * kWideGroups), smem, s,
                    x, norm_w, eps, d, n, q, scales, qsum);
}

// Rows from this many columns (and whose double-buffered groups fit in shared
// memory) take the 128-thread form for many tokens: kWideMinCols, or
// OBN_QUANT_WIDE_MIN=<columns>; OBN_QUANT_WIDE=0 keeps every row on the 64-thread
// form. Read once per process.
int quant_wide_min_cols() {
  static const int v = [] {
    const char* e = std::getenv("OBN_QUANT_WIDE");
    if (e && e[0] == '0') return 1 << 30;
    const char* m = std::getenv("OBN_QUANT_WIDE_MIN");
    const int c = m ? std::atoi(m) : 0;
    return c > 0 ? c : kWideMinCols;
  }();
  return v;
}
constexpr int kWideMaxCols = 7936;  // (2 * 3 + 1) rows of floats within 227 KB

cudaError_t launch_rmsnorm_quant(const float* x, const float* norm_w, float eps, int n, int d,
                                 int8_t* q, float* scales, int32_t* qsum, cudaStream_t s) {
  // Few tokens (decode): one 256-thread CTA per token keeps each token's chain short.
  const int ept = (d + 255) / 256;
  static const int few = [] {  // OBN_QUANT_FEW=<tokens> moves the switch (A/B measurements)
    const char* e = std::getenv("OBN_QUANT_FEW");
    const int v = e ? std::atoi(e) : 0;
    return v;
  }();
  if (n <= (few > 0 ? few : d >= kWideMinCols ? kQuantFewTokensWide : kQuantFewTokens)) {
    if (ept <= 2) return rmsnorm_quant_ept<2>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 4) return rmsnorm_quant_ept<4>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 8) return rmsnorm_quant_ept<8>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 12) return rmsnorm_quant_ept<12>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 16) return rmsnorm_quant_ept<16>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 24) return rmsnorm_quant_ept<24>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 28) return rmsnorm_quant_ept<28>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 36) return rmsnorm_quant_ept<36>(x, norm_w, eps, n, d, q, scales, qsum, s);
  }
  if (d >= quant_wide_min_cols() && d <= kWideMaxCols) {
    if (ept <= 8) return rmsnorm_quant_w128<8>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 12) return rmsnorm_quant_w128<12>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 16) return rmsnorm_quant_w128<16>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 24) return rmsnorm_quant_w128<24>(x, norm_w, eps, n, d, q, scales, qsum, s);
    if (ept <= 28) return rmsnorm_quant_w128<28>(x, norm_w, eps, n, d, q, scales, qsum, s);
    return rmsnorm_quant_w128<32>(x, norm_w, eps, n, d, q, scales, qsum, s);
  }
  // Many tokens (prefill): 64 threads per token, packed 4-byte stores.
  const int ept4 = ept;  // float4 column quads per thread
  if (ept4 <= 1) return rmsnorm_quant_t64<1>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 2) return rmsnorm_quant_t64<2>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 4) return rmsnorm_quant_t64<4>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 6) return rmsnorm_quant_t64<6>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 8) return rmsnorm_quant_t64<8>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 10) return rmsnorm_quant_t64<10>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 12) return rmsnorm_quant_t64<12>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 16) return rmsnorm_quant_t64<16>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 20) return rmsnorm_quant_t64<20>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 24) return rmsnorm_quant_t64<24>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 28) return rmsnorm_quant_t64<28>(x, norm_w, eps, n, d, q, scales, qsum, s);
  if (ept4 <= 36) return rmsnorm_quant_t64<36>(x, norm_w, eps, n, d, q, scales, qsum, s);
  // larger rows: the three-pass kernel re-reads x instead of holding it in registers
  if (norm_w)
    return launch_pdl(k_rmsnorm_quant<true>, dim3(n), dim3(256), 0, s, x, norm_w, eps, d, q,
                      scales, qsum);
  return launch_pdl(k_rmsnorm_quant<false>, dim3(n), dim3(256), 0, s, x, norm_w, eps, d, q, scales,
                    qsum);
}

namespace {
// activation.wgsl:28-33 then elementwise.wgsl:31-32: the activation of a gate
// value, ReLU^2 (act 0: max(0, x)^2) or SiLU (act 1: x / (1 + exp(-x))).
template <int ACT>
OBN_DEVINL float activation(float x) {
  return gate_act(ACT, x);
}

// act(gate) * up over interleaved (gate, up) pairs: two outputs per thread from
// one 16-byte load of (gate, up, gate, up).
template <int ACT>
__global__ __launch_bounds__(256) void k_act_mul(const float4* __restrict__ gu,
                                                 const float* __restrict__ gu1, size_t pairs2,
                                                 size_t total, float* __restrict__ y) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < pairs2) {
    const float4 v = gu[i];
    y[2 * i] = __fmul_rn(activation<ACT>(v.x), v.y);
    y[2 * i + 1] = __fmul_rn(activation<ACT>(v.z), v.w);
  } else if (i == pairs2 && 2 * pairs2 < total) {  // odd element count: the last output
    const size_t j = 2 * pairs2;
    y[j] = __fmul_rn(activation<ACT>(gu1[2 * j]), gu1[2 * j + 1]);
  }
}

// activation.wgsl alone (FFN::forward_simple, ffn.rs:82-92): y[i] = act(x[i]).
template <int ACT>
__global__ __launch_bounds__(256) void k_act(const float* x, size_t count, float* y) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < count) y[i] = activation<ACT>(x[i]);
}
}  // namespace

namespace {
__global__ __launch_bounds__(256) void k_add(const float4* __restrict__ a,
                                             const float4* __restrict__ b, size_t n4,
                                             const float* __restrict__ a1,
                                             const float* __restrict__ b1, size_t count,
                                             float4* __restrict__ y4, float* __restrict__ y1) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n4) {
    const float4 u = a[i], v = b[i];
    y4[i] = make_float4(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y), __fadd_rn(u.z, v.z),
                        __fadd_rn(u.w, v.w));
  } else if (i - n4 < count - 4 * n4) {  // the tail of a count not divisible by 4
    const size_t j = 4 * n4 + (i - n4);
    y1[j] = __fadd_rn(a1[j], b1[j]);
  }
}

__global__ __launch_bounds__(256) void k_embed_f16(const unsigned short* __restrict__ table,
                                                   int vocab, int dim,
                                                   const int32_t* __restrict__ ids, size_t total,
                                                   float* __restrict__ y) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const size_t t = i / dim, c = i % dim;
  const int id = ids[t];
  y[i] = (id >= 0 && id < vocab)
             ? __half2float(__ushort_as_half(table[static_cast<size_t>(id) * dim + c]))
             : 0.0f;
}
}  // namespace

cudaError_t launch_add(const float* a, const float* b, size_t count, float* y, cudaStream_t s) {
  const bool vec = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                     reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const size_t n4 = vec ? count / 4 : 0;
  const size_t threads = n4 + (count - 4 * n4);
  if (threads == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  return launch_pdl(k_add, dim3(blocks), dim3(256), 0, s, reinterpret_cast<const float4*>(a),
                    reinterpret_cast<const float4*>(b), n4, a, b, count,
                    reinterpret_cast<float4*>(y), y);
}

cudaError_t launch_embed_f16(const void* table, int vocab, int dim, const int32_t* ids, int n,
                             float* y, cudaStream_t s) {
  const size_t total = static_cast<size_t>(n) * dim;
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  return launch_pdl(k_embed_f16, dim3(blocks), dim3(256), 0, s,
                    static_cast<const unsigned short*>(table), vocab, dim, ids, total, y);
}

cudaError_t launch_act_mul(const float* gu, int n, int d, int act, float* y, cudaStream_t s) {
  const size_t total = static_cast<size_t>(n) * d;
  const size_t pairs2 = total / 2;
  const size_t threads = pairs2 + 1;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  auto kern = act == 0 ? k_act_mul<0> : k_act_mul<1>;
  return launch_pdl(kern, dim3(blocks), dim3(256), 0, s, reinterpret_cast<const float4*>(gu), gu,
                    pairs2, total, y);
}

cudaError_t launch_act(const float* x, size_t count, int act, float* y, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((count + 255) / 256);
  auto kern = act == 0 ? k_act<0> : k_act<1>;
  return launch_pdl(kern, dim3(blocks), dim3(256), 0, s, x, count, y);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int n, int d, float* y,
                           cudaStream_t s) {
  return launch_pdl(k_rmsnorm, dim3(n), dim3(256), 0, s, x, w, eps, d, y);
}

cudaError_t launch_bitlinear_n1(const WeightView& W, const float* gamma, float eps,
                                const float* x, float* y, cudaStream_t s, int accumulate,
                                int act) {
  const int ept = (W.in_dim + 255) / 256;
  if (ept <= 1) return bitlinear_n1_ept<1>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 2) return bitlinear_n1_ept<2>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 4) return bitlinear_n1_ept<4>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 8) return bitlinear_n1_ept<8>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 12) return bitlinear_n1_ept<12>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 16) return bitlinear_n1_ept<16>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 20) return bitlinear_n1_ept<20>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 24) return bitlinear_n1_ept<24>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 28) return bitlinear_n1_ept<28>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 32) return bitlinear_n1_ept<32>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 40) return bitlinear_n1_ept<40>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 48) return bitlinear_n1_ept<48>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 56) return bitlinear_n1_ept<56>(W, gamma, eps, x, y, accumulate, act, s);
  if (ept <= 64) return bitlinear_n1_ept<64>(W, gamma, eps, x, y, accumulate, act, s);
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const WeightView& W, const int8_t* q, const float* s_x,
                        const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                        cudaStream_t s) {
  if (acc) return gemv_dispatch<true>(W, q, s_x, qsum, n, nullptr, acc, order, s);
  return gemv_dispatch<false>(W, q, s_x, qsum, n, y, nullptr, order, s);
}

cudaError_t read_and_clear_dev_error_kernels(uint32_t* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_dev_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(uint32_t));
}

cudaError_t read_and_clear_dev_error(uint32_t* out) {
  uint32_t a = 0, b = 0, c = 0;
  cudaError_t e = read_and_clear_dev_error_kernels(&a);
  if (e == cudaSuccess) e = read_and_clear_dev_error_gemm(&b);
  if (e == cudaSuccess) e = read_and_clear_dev_error_mma(&c);
  *out = a ? a : b ? b : c;
  return e;
}

}  // namespace obn
