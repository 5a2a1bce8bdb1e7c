// gemv_mma.cu — batched-decode ternary matmul (2..16 tokens) on mma.sync.
//
// Out[t, m] = f32(sum_k w[m,k] q[t,k]) * (s_w[m] * s_x[t])   (ternary_gemm.wgsl:132-133)
//
// Why mma.sync here and tcgen05 for prefill: on B200 one tcgen05.mma kind::i8
// (M = 128, K = 32) costs a flat ~168 cycles for every N from 8 to 256
// (measured: 64-MMA bursts per SM, one commit), so at decode batch sizes the
// tensor-core path pays the full N = 256 price for 8..64 token columns and is
// bound by its MMA count (rows * K / 4096 per layer). The warp-level
// m16n8k32 u8 x s8 MMA sustains ~2000 MACs per cycle per SM with N = 8, so an
// 8-token group costs 1/8 of a 64-token tcgen05 tile per MAC. The persistent
// tcgen05 GEMMs (gemm.cu) stay the path from 17 tokens up: there each CTA's
// per-block activation loads from L2 leave the warp-MMA form latency-bound.
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
  if (!geom_ok) return;  // uniform per CTA
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
  const int gid = lane >> 2, tig = lane & 3;
  // B fragments of every token group for block b: 16 bytes per 64-column chunk
  auto load_b = [&](int b, uint4 (&bq)[NT][2]) {
#pragma unroll
    for (int tg = 0; tg < NT; ++tg) {
      const int t = tg * 8 + gid;
#pragma unroll
      for (int c = 0; c < 2; ++c)
        bq[tg][c] = t < n ? ldg_nc_v4(q + static_cast<size_t>(t) * K + b * kBlockK + 64 * c + 16 * tig)
                          : make_uint4(0u, 0u, 0u, 0u);
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
  const bool ok = mbar_wait(&bar, 0);  // the weights (normally landed long ago)
  if (!ok) mbar_wait(&bar, 0);         // copies may still be in flight: once more, bounded
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

cudaError_t read_and_clear_dev_error_mma(uint32_t* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_dev_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(uint32_t));
}

}  // namespace obn
