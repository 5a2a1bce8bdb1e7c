// gemv_mma.cu — batched-decode ternary matmul (2..16 tokens) on mma.sync.
//
// Out[t, m] = f32(sum_k w[m,k] q[t,k]) * (s_w[m] * s_x[t])   (ternary_gemm.wgsl:132-133)
//
// Why mma.sync here and tcgen05 for prefill: on B200 one tcgen05.mma kind::i8
// (M = 128, K = 32) costs a near-flat ~102-106 cycles for every N from 8 to 128
// (143 at N = 256; obn_measure_mma_rate, 64-MMA bursts on every SM, one commit),
// so at decode widths the tensor-core path pays for columns it does not use:
// 310 MACs per cycle per SM at N = 8, 1280 at N = 32, 2560 at N = 64. The
// warp-level m16n8k32 u8 x s8 MMA sustains ~1850 MACs per cycle per SM with
// N = 8, so it wins up to ~32 tokens; the tcgen05 GEMMs (gemm.cu) serve 17
// tokens and up, where this kernel's per-block activation loads from L2 also
// leave it latency-bound.
//
// Work split: like the single-token kernel, the layer's 16-row subtiles are
// spread evenly over at most one CTA per SM (a contiguous run, one bulk copy of
// the T16 layout into shared memory, issued before the PDL wait). Warp w takes
// the 128-column K blocks b = w, w + 8, ... for all of the CTA's subtiles and all
// token groups of 8; its partial sums meet the other warps' in shared memory
// through integer atomics (exact in any order), then one thread per output
// forms the epilogue.
//
// K permutation: the MMA sums over its 32 K slots in any order, so A and B only
// have to agree on which real column each slot holds. Per 64-column chunk c of a
// block and k-step s (0, 1), slot tig*4 + e (b0 / a0, a1) holds real column
// 64c + 16 tig + 8s + e and slot 16 + tig*4 + e (b1 / a2, a3) holds
// 64c + 16 tig + 8s + 4 + e (tig = lane % 4, e = 0..3). Then
//   B: thread (gid = lane / 4, tig) reads the 16 bytes q[token gid][64c + 16 tig ..]
//      once: word 2s is b0 and word 2s + 1 is b1 of k-step s;
//   A: those columns sit in T16 half h = tig % 2 of the block, group
//      g = 2c + tig / 2, bytes 8s .. 8s + 7 of the row's 16-byte half, so a0 / a2
//      are words 2s / 2s + 1 of row gid's half shifted by 6 - 2g and masked to
//      one 2-bit code per byte (a1 / a3: row gid + 8). Codes c = w + 1; the
//      epilogue subtracts the per-token code sum (exact).
#include "kernels.h"

#include "layout.cuh"
#include "obn_common.cuh"

namespace obn {

namespace {

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_mma(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
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

OBN_DEVINL void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

OBN_DEVINL uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// quantize.wgsl:67-72 for four values (round half to even): adding 1.5 * 2^23
// leaves round(v) in the low mantissa bits for |v| < 2^22, so the low byte of
// the bit pattern is the int8 and bits - 0x4B400000 the int. |y * inv| <=
// 127 * (1 + 2^-23) for |y| <= absmax, so the shader's clamp never binds.
OBN_DEVINL uint32_t quant4_rn(float4 y, float inv, int& sum) {
  const uint32_t a = __float_as_uint(__fadd_rn(__fmul_rn(y.x, inv), 12582912.0f));
  const uint32_t b = __float_as_uint(__fadd_rn(__fmul_rn(y.y, inv), 12582912.0f));
  const uint32_t c = __float_as_uint(__fadd_rn(__fmul_rn(y.z, inv), 12582912.0f));
  const uint32_t d = __float_as_uint(__fadd_rn(__fmul_rn(y.w, inv), 12582912.0f));
  sum += static_cast<int>(a + b + c + d - 4u * 0x4B400000u);
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Epilogue kinds, fixed per launch.
enum : int { kMmaAcc = 0, kMmaStore = 1, kMmaAdd = 2, kMmaRelu2 = 3, kMmaSilu = 4 };

constexpr int kMmaWarps = 8;
constexpr int kMmaMaxCtaSmem = 100 * 1024;

// Dynamic shared memory: `wslots` subtiles of packed weights, then the partial
// sums red[wslots * 16 rows][NT * 8 tokens] (int32).
inline size_t mma_smem_bytes(int K, int wslots, int nt) {
  return static_cast<size_t>(wslots) * (K / kBlockK) * kSubtileBytes +
         static_cast<size_t>(wslots) * kSubRows * nt * 8 * sizeof(int32_t);
}

// The MMA phase and epilogue shared by both kernels: warp w accumulates the
// blocks b = w, w + 8, ... of the CTA's ns subtiles for every token group, the
// warps' partials meet in `red` (integer atomics, exact), and one thread per
// output applies the epilogue of kind KIND. q holds the int8 activations with
// row stride ldq, in global memory (QSMEM = false) or shared memory.
template <int NT, int NSUB, int KIND, bool QSMEM>
OBN_DEVINL void mma_phase(const uint8_t* w_s, uint64_t* bar, int32_t* red, const float* sw_s,
                          const float* sx_s, const int* qs_s, const int8_t* q, int ldq,
                          float* __restrict__ y, int32_t* __restrict__ acc_out, int M, int K, int n,
                          int ns, int m0) {
  constexpr int NTOK = NT * 8;
  const int KB = K / kBlockK;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  // B fragments of every token group for block b: 16 bytes per 64-column chunk
  auto load_b = [&](int b, uint4 (&bq)[NT][2]) {
#pragma unroll
    for (int tg = 0; tg < NT; ++tg) {
      const int t = tg * 8 + gid;
#pragma unroll
      for (int c = 0; c < 2; ++c)
        bq[tg][c] = t >= n ? make_uint4(0u, 0u, 0u, 0u)
                    : QSMEM ? lds128(smem_u32(q + t * ldq + b * kBlockK + 64 * c + 16 * tig))
                            : ldg_nc_v4(q + static_cast<size_t>(t) * ldq + b * kBlockK + 64 * c +
                                        16 * tig);
    }
  };
  int acc[NSUB][NT][4];
#pragma unroll
  for (int sub = 0; sub < NSUB; ++sub)
#pragma unroll
    for (int tg = 0; tg < NT; ++tg)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[sub][tg][i] = 0;

  uint4 bq[NT][2], bn[NT][2];
  int b = warp;
  if (b < KB) load_b(b, bq);
  const bool ok = mbar_wait(bar, 0);  // the weights (normally landed long ago)
  if (!ok) mbar_wait(bar, 0);         // copies may still be in flight: once more, bounded
  const uint32_t wrow = smem_u32(w_s) + (tig & 1) * 256 + gid * 16;  // row gid of half tig % 2
  if (ok) {
    for (; b < KB; b += kMmaWarps) {
      const int bnext = b + kMmaWarps;
      if (bnext < KB) load_b(bnext, bn);
#pragma unroll
      for (int sub = 0; sub < NSUB; ++sub) {
        if (sub < ns) {
          const uint32_t base = wrow + (sub * KB + b) * kSubtileBytes;
          const uint4 r0 = lds128(base), r1 = lds128(base + 128);  // rows gid and gid + 8
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int sh = 6 - 4 * c - 2 * (tig >> 1);  // group g = 2c + tig / 2
#pragma unroll
            for (int s = 0; s < 2; ++s) {
              const uint32_t a0 = ((s ? r0.z : r0.x) >> sh) & 0x03030303u;
              const uint32_t a2 = ((s ? r0.w : r0.y) >> sh) & 0x03030303u;
              const uint32_t a1 = ((s ? r1.z : r1.x) >> sh) & 0x03030303u;
              const uint32_t a3 = ((s ? r1.w : r1.y) >> sh) & 0x03030303u;
#pragma unroll
              for (int tg = 0; tg < NT; ++tg)
                mma_u8s8(acc[sub][tg], a0, a1, a2, a3, s ? bq[tg][c].z : bq[tg][c].x,
                         s ? bq[tg][c].w : bq[tg][c].y);
            }
          }
        }
      }
      if (bnext < KB) {
#pragma unroll
        for (int tg = 0; tg < NT; ++tg) {
          bq[tg][0] = bn[tg][0];
          bq[tg][1] = bn[tg][1];
        }
      }
    }
  }

  // ---- partial sums of all warps (C fragment: rows gid / gid + 8, tokens 2 tig, 2 tig + 1)
#pragma unroll
  for (int sub = 0; sub < NSUB; ++sub) {
    if (sub < ns) {
#pragma unroll
      for (int tg = 0; tg < NT; ++tg) {
        int32_t* r0 = red + (sub * kSubRows + gid) * NTOK + tg * 8 + 2 * tig;
        int32_t* r1 = r0 + 8 * NTOK;
        atomicAdd(r0, acc[sub][tg][0]);
        atomicAdd(r0 + 1, acc[sub][tg][1]);
        atomicAdd(r1, acc[sub][tg][2]);
        atomicAdd(r1 + 1, acc[sub][tg][3]);
      }
    }
  }
  __syncthreads();
  if (!ok) return;

  // ---- epilogue: consecutive threads take consecutive rows of one token
  const int rows = ns * kSubRows;
  if constexpr (KIND >= kMmaRelu2) {
    // gated pairs (rows 2i gate, 2i + 1 up; subtiles start on even rows):
    // act(gate) * up, each in ternary_gemm.wgsl:132-133's order
    const int pairs = rows >> 1;
    const size_t Mh = static_cast<size_t>(M) >> 1;
    for (int i = tid; i < pairs * n; i += kMmaWarps * 32) {
      const int t = i / pairs, p = i - t * pairs;
      const int r = 2 * p, m = m0 + r;
      if (m + 1 >= M) continue;
      const float sx = sx_s[t];
      const float g = __fmul_rn(static_cast<float>(red[r * NTOK + t] - qs_s[t]),
                                __fmul_rn(sw_s[r], sx));
      const float u = __fmul_rn(static_cast<float>(red[(r + 1) * NTOK + t] - qs_s[t]),
                                __fmul_rn(sw_s[r + 1], sx));
      y[static_cast<size_t>(t) * Mh + (m >> 1)] = __fmul_rn(gate_act(KIND - kMmaRelu2, g), u);
    }
  } else {
    for (int i = tid; i < rows * n; i += kMmaWarps * 32) {
      const int t = i / rows, r = i - t * rows;
      const int m = m0 + r;
      if (m >= M) continue;
      const int a = red[r * NTOK + t] - qs_s[t];
      const size_t o = static_cast<size_t>(t) * M + m;
      if constexpr (KIND == kMmaAcc) {
        acc_out[o] = a;
      } else {
        const float val = __fmul_rn(static_cast<float>(a), __fmul_rn(sw_s[r], sx_s[t]));
        if constexpr (KIND == kMmaAdd)
          y[o] = __fadd_rn(y[o], val);
        else
          y[o] = val;
      }
    }
  }
}

template <int NT, int NSUB, int KIND>
__global__ __launch_bounds__(kMmaWarps * 32) void k_mma_gemv(
    const uint8_t* __restrict__ W, const float* __restrict__ s_w, const int8_t* __restrict__ q,
    const float* __restrict__ s_x, const int32_t* __restrict__ qsum, float* __restrict__ y,
    int32_t* __restrict__ acc_out, int M, int K, int n, int wslots) {
  constexpr int NTOK = NT * 8;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float sx_s[NTOK];
  __shared__ int qs_s[NTOK];
  __shared__ float sw_s[NSUB * kSubRows];

  const int KB = K / kBlockK;
  const int S_total = (M + kSubRows - 1) / kSubRows;
  const int s0 = static_cast<int>(static_cast<long long>(blockIdx.x) * S_total / gridDim.x);
  const int s1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * S_total / gridDim.x);
  const int ns = s1 - s0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool geom_ok = ns >= 1 && ns <= wslots && wslots <= NSUB && n >= 1 && n <= NTOK;
  if (tid == 0 && !geom_ok) record_error(DEVERR_BAD_LAUNCH);
  if (!geom_ok) {  // uniform per CTA; still ordered after the preceding grid
    pdl_wait();
    return;
  }
  uint8_t* w_s = smem;
  int32_t* red = reinterpret_cast<int32_t*>(smem + static_cast<size_t>(wslots) * KB * kSubtileBytes);
  const int m0 = s0 * kSubRows;

  // ---- before the wait: barrier, partial-sum buffer, weight copy, row scales
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < ns * kSubRows * NTOK; i += kMmaWarps * 32) red[i] = 0;
  if (tid < ns * kSubRows)
    sw_s[tid] = (KIND != kMmaAcc && m0 + tid < M) ? s_w[m0 + tid] : 0.0f;
  __syncthreads();
  if (tid == 0) {  // the CTA's subtiles are one contiguous run in the T16 layout
    const uint32_t wbytes = static_cast<uint32_t>(ns * KB) * kSubtileBytes;
    mbar_arrive_expect_tx(&bar, wbytes);
    bulk_g2s_hint(w_s, W + subtile_offset(s0, 0, KB), wbytes, &bar, policy_evict_first());
  }
  pdl_launch_dependents();
  pdl_wait();  // q, s_x, qsum (and y when accumulating) come from earlier kernels

  if (tid < NTOK) {
    sx_s[tid] = (KIND != kMmaAcc && tid < n) ? s_x[tid] : 0.0f;
    qs_s[tid] = tid < n ? qsum[tid] : 0;
  }
  mma_phase<NT, NSUB, KIND, false>(w_s, &bar, red, sw_s, sx_s, qs_s, q, K, y, acc_out, M, K, n,
                                    ns, m0);
}

// The whole BitLinear forward for 2..16 tokens with in_dim <= 3072: RMSNorm +
// int8 quantize of every token in each CTA (no separate quantize launch), then
// the MMA phase with its activations in shared memory. Warp w normalises tokens
// w, w + 8: lane l holds the float4 columns 4l + 128m, i.e. shader lanes
// 4l + e (m even, column round m / 2) and 128 + 4l + e (m odd), so each fold
// of squares is local and in the shader's order; stride 128 of the halving
// tree is then a local add, strides 64 .. 4 are shuffles down 16 .. 1 (the
// shader's pairings) and 2, 1 are local again: no block barrier per token.
template <int EPT4, int NT, int NSUB, int KIND>
__global__ __launch_bounds__(kMmaWarps * 32) void k_bitlinear_mma(
    const uint8_t* __restrict__ W, const float* __restrict__ s_w, const float* __restrict__ gamma,
    float eps, const float* __restrict__ x, float* __restrict__ y, int M, int K, int n,
    int wslots) {
  constexpr int NTOK = NT * 8;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float sx_s[NTOK];
  __shared__ int qs_s[NTOK];
  __shared__ float sw_s[NSUB * kSubRows];

  const int KB = K / kBlockK;
  const int S_total = (M + kSubRows - 1) / kSubRows;
  const int s0 = static_cast<int>(static_cast<long long>(blockIdx.x) * S_total / gridDim.x);
  const int s1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * S_total / gridDim.x);
  const int ns = s1 - s0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool geom_ok = ns >= 1 && ns <= wslots && wslots <= NSUB && n >= 1 && n <= NTOK &&
                       K <= EPT4 * 128;
  if (tid == 0 && !geom_ok) record_error(DEVERR_BAD_LAUNCH);
  if (!geom_ok) {  // uniform per CTA; still ordered after the preceding grid
    pdl_wait();
    return;
  }
  const int ldq = K + 16;  // padded int8 rows
  uint8_t* w_s = smem;
  int32_t* red = reinterpret_cast<int32_t*>(smem + static_cast<size_t>(wslots) * KB * kSubtileBytes);
  float* g_s = reinterpret_cast<float*>(red + wslots * kSubRows * NTOK);
  int8_t* q_s = reinterpret_cast<int8_t*>(g_s + K);
  const int m0 = s0 * kSubRows;

  // ---- before the wait: barrier, partial sums, row scales, gamma, weight copy
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < ns * kSubRows * NTOK; i += kMmaWarps * 32) red[i] = 0;
  if (tid < ns * kSubRows) sw_s[tid] = m0 + tid < M ? s_w[m0 + tid] : 0.0f;
  if (gamma)
    for (int i = 4 * tid; i < K; i += 4 * kMmaWarps * 32)
      *reinterpret_cast<float4*>(g_s + i) = *reinterpret_cast<const float4*>(gamma + i);
  __syncthreads();
  if (tid == 0) {
    const uint32_t wbytes = static_cast<uint32_t>(ns * KB) * kSubtileBytes;
    mbar_arrive_expect_tx(&bar, wbytes);
    bulk_g2s_hint(w_s, W + subtile_offset(s0, 0, KB), wbytes, &bar, policy_evict_first());
  }
  pdl_launch_dependents();
  pdl_wait();  // x (and y when accumulating) may come from earlier kernels

  // ---- RMSNorm + quantize, one warp per token
  for (int t = warp; t < n; t += kMmaWarps) {
    const float* xr = x + static_cast<size_t>(t) * K;
    float4 xv[EPT4];
#pragma unroll
    for (int m = 0; m < EPT4; ++m) {
      const int c = 4 * lane + 128 * m;
      xv[m] = c < K ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float rms = 1.0f;
    if (gamma) {
      float pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int m = 0; m < EPT4; ++m) {
        if (4 * lane + 128 * m < K) {
          if (m & 1) {
            pb[0] = __fadd_rn(pb[0], __fmul_rn(xv[m].x, xv[m].x));
            pb[1] = __fadd_rn(pb[1], __fmul_rn(xv[m].y, xv[m].y));
            pb[2] = __fadd_rn(pb[2], __fmul_rn(xv[m].z, xv[m].z));
            pb[3] = __fadd_rn(pb[3], __fmul_rn(xv[m].w, xv[m].w));
          } else {
            pa[0] = __fadd_rn(pa[0], __fmul_rn(xv[m].x, xv[m].x));
            pa[1] = __fadd_rn(pa[1], __fmul_rn(xv[m].y, xv[m].y));
            pa[2] = __fadd_rn(pa[2], __fmul_rn(xv[m].z, xv[m].z));
            pa[3] = __fadd_rn(pa[3], __fmul_rn(xv[m].w, xv[m].w));
          }
        }
      }
      float v0 = __fadd_rn(pa[0], pb[0]), v1 = __fadd_rn(pa[1], pb[1]);  // stride 128
      float v2 = __fadd_rn(pa[2], pb[2]), v3 = __fadd_rn(pa[3], pb[3]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {  // strides 64 .. 4
        v0 = __fadd_rn(v0, __shfl_down_sync(0xffffffffu, v0, o));
        v1 = __fadd_rn(v1, __shfl_down_sync(0xffffffffu, v1, o));
        v2 = __fadd_rn(v2, __shfl_down_sync(0xffffffffu, v2, o));
        v3 = __fadd_rn(v3, __shfl_down_sync(0xffffffffu, v3, o));
      }
      const float total =
          __shfl_sync(0xffffffffu, __fadd_rn(__fadd_rn(v0, v2), __fadd_rn(v1, v3)), 0);
      rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), eps)));
    }
    float lmax = 0.0f;
#pragma unroll
    for (int m = 0; m < EPT4; ++m) {
      const int c = 4 * lane + 128 * m;
      if (c < K) {
        if (gamma) {
          const float4 g = *reinterpret_cast<const float4*>(g_s + c);
          xv[m] = make_float4(__fmul_rn(__fmul_rn(xv[m].x, rms), g.x),
                              __fmul_rn(__fmul_rn(xv[m].y, rms), g.y),
                              __fmul_rn(__fmul_rn(xv[m].z, rms), g.z),
                              __fmul_rn(__fmul_rn(xv[m].w, rms), g.w));
        }
        lmax = fmaxf(lmax, fmaxf(fmaxf(fabsf(xv[m].x), fabsf(xv[m].y)),
                                 fmaxf(fabsf(xv[m].z), fabsf(xv[m].w))));
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    const float inv = lmax == 0.0f ? 0.0f : __fdiv_rn(127.0f, lmax);
    int lsum = 0;
#pragma unroll
    for (int m = 0; m < EPT4; ++m) {
      const int c = 4 * lane + 128 * m;
      if (c < K) *reinterpret_cast<uint32_t*>(q_s + t * ldq + c) = quant4_rn(xv[m], inv, lsum);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) {
      sx_s[t] = lmax == 0.0f ? 1.0f : __fdiv_rn(lmax, 127.0f);
      qs_s[t] = lsum;
    }
  }
  __syncthreads();  // every token's int8 row, scale and code sum
  mma_phase<NT, NSUB, KIND, true>(w_s, &bar, red, sw_s, sx_s, qs_s, q_s, ldq, y, nullptr, M, K,
                                   n, ns, m0);
}

template <int NT, int NSUB, int KIND>
cudaError_t mma_run(const WeightView& W, const int8_t* q, const float* s_x, const int32_t* qsum,
                    int n, float* y, int32_t* acc, int grid, int wslots, cudaStream_t s) {
  auto kern = k_mma_gemv<NT, NSUB, KIND>;
  const size_t smem = mma_smem_bytes(W.in_dim, wslots, NT);
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_mma(kern, dim3(grid), dim3(kMmaWarps * 32), smem, s, W.w, W.s_w, q, s_x,
                        qsum, y, acc, W.out_dim, W.in_dim, n, wslots);
}

template <int NT, int NSUB>
cudaError_t mma_kind(const WeightView& W, const int8_t* q, const float* s_x, const int32_t* qsum,
                     int n, float* y, int32_t* acc, int kind, cudaStream_t s) {
  // the layer's subtiles over at most one CTA per SM (more CTAs only when a CTA's
  // share would not fit its shared-memory budget or NSUB)
  const int KB = W.in_dim / kBlockK;
  const int S_total = (W.out_dim + kSubRows - 1) / kSubRows;
  const size_t per_sub = mma_smem_bytes(W.in_dim, 1, NT);
  int cap = static_cast<int>(kMmaMaxCtaSmem / per_sub);
  cap = cap < 1 ? 1 : cap > NSUB ? NSUB : cap;
  int grid = num_sms_cached();
  if (grid > S_total) grid = S_total;
  if ((S_total + grid - 1) / grid > cap) grid = (S_total + cap - 1) / cap;
  const int wslots = (S_total + grid - 1) / grid;
  (void)KB;
  switch (kind) {
    case kMmaAcc: return mma_run<NT, NSUB, kMmaAcc>(W, q, s_x, qsum, n, y, acc, grid, wslots, s);
    case kMmaAdd: return mma_run<NT, NSUB, kMmaAdd>(W, q, s_x, qsum, n, y, acc, grid, wslots, s);
    case kMmaRelu2: return mma_run<NT, NSUB, kMmaRelu2>(W, q, s_x, qsum, n, y, acc, grid, wslots, s);
    case kMmaSilu: return mma_run<NT, NSUB, kMmaSilu>(W, q, s_x, qsum, n, y, acc, grid, wslots, s);
    default: return mma_run<NT, NSUB, kMmaStore>(W, q, s_x, qsum, n, y, acc, grid, wslots, s);
  }
}


// Fused forward: shared memory = weights + partial sums (per subtile), gamma
// and the padded int8 rows of every token (fixed).
inline size_t fused_fixed_bytes(int K, int nt) {
  return sizeof(float) * static_cast<size_t>(K) + static_cast<size_t>(nt) * 8 * (K + 16);
}

template <int EPT4, int NT, int KIND>
cudaError_t fused_run(const WeightView& W, const float* gamma, float eps, const float* x, int n,
                      float* y, cudaStream_t s) {
  constexpr int NSUB = 8;
  const int S_total = (W.out_dim + kSubRows - 1) / kSubRows;
  const size_t per_sub = mma_smem_bytes(W.in_dim, 1, NT);
  const size_t fixed = fused_fixed_bytes(W.in_dim, NT);
  int cap = kMmaMaxCtaSmem > fixed ? static_cast<int>((kMmaMaxCtaSmem - fixed) / per_sub) : 1;
  cap = cap < 1 ? 1 : cap > NSUB ? NSUB : cap;
  int grid = num_sms_cached();
  if (grid > S_total) grid = S_total;
  if ((S_total + grid - 1) / grid > cap) grid = (S_total + cap - 1) / cap;
  const int wslots = (S_total + grid - 1) / grid;
  const size_t smem = per_sub * wslots + fixed;
  auto kern = k_bitlinear_mma<EPT4, NT, NSUB, KIND>;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_mma(kern, dim3(grid), dim3(kMmaWarps * 32), smem, s, W.w, W.s_w, gamma, eps,
                        x, y, W.out_dim, W.in_dim, n, wslots);
}

template <int EPT4, int NT>
cudaError_t fused_kind(const WeightView& W, const float* gamma, float eps, const float* x, int n,
                       float* y, int kind, cudaStream_t s) {
  switch (kind) {
    case kMmaAdd: return fused_run<EPT4, NT, kMmaAdd>(W, gamma, eps, x, n, y, s);
    case kMmaRelu2: return fused_run<EPT4, NT, kMmaRelu2>(W, gamma, eps, x, n, y, s);
    case kMmaSilu: return fused_run<EPT4, NT, kMmaSilu>(W, gamma, eps, x, n, y, s);
    default: return fused_run<EPT4, NT, kMmaStore>(W, gamma, eps, x, n, y, s);
  }
}

template <int EPT4>
cudaError_t fused_nt(const WeightView& W, const float* gamma, float eps, const float* x, int n,
                     float* y, int kind, cudaStream_t s) {
  if (n <= 8) return fused_kind<EPT4, 1>(W, gamma, eps, x, n, y, kind, s);
  return fused_kind<EPT4, 2>(W, gamma, eps, x, n, y, kind, s);
}
}  // namespace

bool mma_gemv_supported(const WeightView& W, int n) {
  return n >= 2 && n <= kMmaMaxTokens && W.in_dim % kBlockK == 0 &&
         mma_smem_bytes(W.in_dim, 1, 4) <= 200 * 1024;
}

cudaError_t launch_mma_gemv(const WeightView& W, const int8_t* q, const float* s_x,
                            const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                            cudaStream_t s) {
  if (n < 1 || n > kMmaMaxTokens) return cudaErrorInvalidValue;
  const int kind = acc                        ? kMmaAcc
                   : (order & kOutGated)      ? ((order & kOutSilu) ? kMmaSilu : kMmaRelu2)
                   : (order & kOutAccumulate) ? kMmaAdd
                                              : kMmaStore;
  if (n <= 8) return mma_kind<1, 8>(W, q, s_x, qsum, n, y, acc, kind, s);
  return mma_kind<2, 8>(W, q, s_x, qsum, n, y, acc, kind, s);
}

bool bitlinear_mma_supported(const WeightView& W, int n) {
  // Every CTA normalises every token again (~n * in_dim * 12 / 128 issue cycles
  // per SM): measured on B200 that pays off against the separate quantize launch
  // only when the matmul phase is long, i.e. few tokens on a layer with many rows
  // (the merged 2 x 6912-row gate|up FFN layer: 2..8 tokens 7.9-8.7 -> 6.3-7.1 us),
  // while the 2560- to 6912-row projections lose 1-15 % of step throughput.
  return n >= 2 && n <= kFusedMaxTokens && W.out_dim >= kFusedMinRows &&
         W.in_dim % kBlockK == 0 && W.in_dim <= kFusedMaxK;
}

cudaError_t launch_bitlinear_mma(const WeightView& W, const float* gamma, float eps,
                                 const float* x, int n, float* y, int accumulate, int act,
                                 cudaStream_t s) {
  if (!bitlinear_mma_supported(W, n)) return cudaErrorInvalidValue;
  const int kind = act >= 0 ? (act == 1 ? kMmaSilu : kMmaRelu2) : accumulate ? kMmaAdd : kMmaStore;
  const int ept4 = W.in_dim / kBlockK;  // float4 column quads per lane
  if (ept4 <= 8) return fused_nt<8>(W, gamma, eps, x, n, y, kind, s);
  if (ept4 <= 16) return fused_nt<16>(W, gamma, eps, x, n, y, kind, s);
  if (ept4 <= 20) return fused_nt<20>(W, gamma, eps, x, n, y, kind, s);
  return fused_nt<24>(W, gamma, eps, x, n, y, kind, s);
}

cudaError_t read_and_clear_dev_error_mma(uint32_t* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_dev_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(uint32_t));
}

}  // namespace obn
