// gemm.cu — ternary GEMM on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// Out[n, m] = f32(sum_k w[m,k] q[n,k]) * scales, for n < N tokens, m < M rows.
//
// Swap-AB formulation: the MMA's M dimension is 128 weight rows, its N
// dimension BN tokens, so D[m, n] lives in TMEM with one weight row per lane and
// the epilogue's stores of Out[n, m] are 128-byte coalesced runs over m.
//
// A pipeline stage covers KSTG 128-element K blocks (one block = one I2_S block):
//   P: the 128 rows' packed 2-bit weights, KSTG x 4 KB, one 3D TMA copy from the
//      T16 layout (box: 512 bytes x KSTG blocks x 8 subtiles);
//   B: BN tokens x KSTG*128 int8 activations, one 3D TMA copy with 128-byte
//      swizzle landing as KSTG K-major [BN][128] tiles;
//   A: P expanded to unsigned 8-bit codes c = w + 1, either in tensor memory
//      (A_TMEM: one TMEM lane per weight row, 32 columns of 4 codes, written
//      with tcgen05.st — keeps the 16 KB tile off the shared-memory port the MMA
//      reads B through) or in shared memory in the UMMA K-major 128-byte-swizzle
//      layout (row r at (r/8)*1024 + (r%8)*128, 16-byte chunk j at chunk j ^ (r%8)).
// The MMA accumulates sum_k c q = sum_k w q + sum_k q; the epilogue subtracts
// the per-token code sum qsum[n] (exact, integer).
//
// Gated layers (rows 2i = gate row i, 2i + 1 = up row i, order | kOutGated):
// the epilogue writes act(gate) * up to Out[n, i] ([N][M / 2]); the two lanes of
// a row pair swap one value per column pair, so each lane stores one column of
// the pair (64-byte runs over i per column).
//
// Warp roles (384 threads, one persistent CTA per SM):
//   warp 0      TMA / bulk-copy producer
//   warp 1      MMA issuer (one thread)
//   warp 2      TMEM allocator
//   warps 4-7   expansion P -> A (thread = weight row)
//   warps 8-11  epilogue TMEM -> registers -> global (warp%4 = TMEM lane quarter)
// Every mbarrier wait is bounded; on a timeout the CTA raises a shared abort
// flag, every role leaves its loop, in-flight copies are waited for (bounded)
// and TMEM is freed before exit.
//
// From 512 tokens the tiles are 256 weight rows x 256 tokens on a cluster of two
// CTAs (PAIR, tcgen05 cta_group::2): each CTA copies and expands its own 128
// rows and copies HALF of the token tile; the even CTA issues the 256-row MMAs,
// which read the other CTA's token half through the pair, and each CTA's TMEM
// gets its 128 accumulator rows. The single-CTA form re-reads every token tile
// from L2 once per 128 rows, and at 8192 tokens that L2 -> SM stream
// (~10 TB/s) is what held the MMA back. The odd CTA announces its codes and its
// drained accumulators with relaxed remote arrivals; the even CTA's commits
// reach both CTAs' barriers (multicast to the pair, no TMA multicast). Tiles of
// the last partial wave (or all of them, when their halves fit at once) run as
// two 128-token units each (tile_unit below).
#include <cuda.h>

#include <cstdlib>
#include <type_traits>

#include "gemm.h"
#include "layout.cuh"
#include "obn_common.cuh"
#include "tc05.cuh"

namespace obn {
namespace {

constexpr int kBM = 128;           // weight rows per tile (MMA M)
constexpr int kBK = 128;           // K elements per block (one I2_S block)
constexpr int kThreads = 384;
constexpr int kPackedBlock = kBM * 32;  // 4096 bytes of packed weights per block

struct GemmSmem {
  uint64_t full_tma[8];
  uint64_t full_a[8];
  uint64_t empty[8];
  uint64_t accf[2];
  uint64_t acce[2];
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort_flag;
};

// Instruction descriptor: D s32, A u8 (codes), B s8 (activations), both
// K-major, N = BN, M = 128.
template <int BN>
constexpr uint32_t idesc_i8() {
  return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

// ---- pieces of the paired (cta_group::2) many-token GEMM ---------------------------
// Two CTAs of a cluster share one MMA of 256 weight rows x BN tokens: each holds
// its 128 rows of codes and half of the token tile (BN / 2 rows) in shared
// memory, the even CTA issues the MMAs, and each CTA's TMEM receives its 128 rows
// of the accumulator. Every token row then crosses L2 -> SM once per 256 weight
// rows instead of once per 128.
template <int BN>
constexpr uint32_t idesc_i8_pair() {  // as idesc_i8, M = 256
  return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>((2 * kBM) >> 4) << 24);
}
// Work units of the persistent tile loop. Tiles [0, split_from) run whole (BN
// tokens); each tile from split_from on runs as two BN / 2-token halves, one unit
// each (paired kernel only). The host splits the last partial wave of tiles, or
// every tile when all the halves fit on the GPU at once, so that the pairs' work
// evens out instead of a few pairs running one more whole tile at the end.
struct TileUnit {
  int mt;    // (paired) row tile
  int tok0;  // first token
  int half;  // 1: BN / 2 tokens, else BN
};
OBN_DEVINL TileUnit tile_unit(int u, int num_m, int split_from, int bn) {
  if (u < split_from) return {u % num_m, (u / num_m) * bn, 0};
  const int h = u - split_from, t = split_from + (h >> 1);
  return {t % num_m, (t / num_m) * bn + (h & 1) * (bn / 2), 1};
}
OBN_DEVINL uint32_t pair_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
OBN_DEVINL uint32_t pair_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// Arrive on an mbarrier of another CTA of the cluster (cluster address), without
// release semantics: callers order what the arrival announces themselves.
OBN_DEVINL void arrive_cluster_relaxed(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}
OBN_DEVINL void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
OBN_DEVINL void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
OBN_DEVINL void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
OBN_DEVINL void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
OBN_DEVINL void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` (same offset) in both CTAs of the pair once every tcgen05
// operation issued so far by this thread has completed.
OBN_DEVINL void commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<unsigned short>(3))
      : "memory");
}
// wait_or_abort with cluster-scope acquire (arrivals from the other CTA).
template <class Smem>
OBN_DEVINL bool wait_or_abort_cl(Smem* sm, uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 1023u) == 1023u && sm->abort_flag) return false;
  }
  record_error(DEVERR_MBAR_TIMEOUT);
  sm->abort_flag = 1;
  return false;
}
OBN_DEVINL bool mbar_wait_cl(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  record_error(DEVERR_MBAR_TIMEOUT);
  return false;
}
template <bool PAIR, class Smem>
OBN_DEVINL bool wait_x(Smem* sm, uint64_t* bar, uint32_t parity) {
  if constexpr (PAIR)
    return wait_or_abort_cl(sm, bar, parity);
  else
    return wait_or_abort(sm, bar, parity);
}

// Output modes of k_gemm: the plain [N][M] output, or a tensor-parallel gather
// that writes this rank's columns of every rank's [N][ldy] output as it goes.
enum : int { kOutLocal = 0, kOutMulticast = 1, kOutPeers = 2 };

// One f32 store through a multicast (NVLS) address: the switch writes it into
// every rank's buffer bound to the multicast object.
OBN_DEVINL void multimem_st_f32(float* addr, float v) {
  asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}
OBN_DEVINL void multimem_st_v4(float* addr, float4 v) {
  asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Epilogue staging of the gather modes: per epilogue warp one [16 tokens][32
// rows] f32 block, so each thread can store 4 consecutive rows of one token.
constexpr int kGatherStageBytes = 4 * 16 * 32 * 4;

template <int BN, int STAGES, int KSTG, bool A_TMEM, int OUT = kOutLocal, bool PAIR = false>
__global__ __launch_bounds__(kThreads, 1) void k_gemm(const __grid_constant__ CUtensorMap tmap_q,
                                                      const __grid_constant__ CUtensorMap tmap_qh,
                                                      const __grid_constant__ CUtensorMap tmap_w,
                                                      const float* __restrict__ s_w,
                                                      const float* __restrict__ s_x,
                                                      const int32_t* __restrict__ qsum,
                                                      float* __restrict__ y,
                                                      int32_t* __restrict__ acc_out, int M, int N,
                                                      int K, int order, int split_arg,
                                                      const GatherOut go) {
  constexpr int kAStage = KSTG * kBM * kBK;      // expanded A bytes per stage (smem variant)
  // PAIR: a cluster of 2 CTAs shares each 256-row x BN-token tile (cta_group::2);
  // this CTA holds rows [128 rank, 128 rank + 128) and tokens [BN/2 rank, +BN/2).
  static_assert(!PAIR || (OUT == kOutLocal && !A_TMEM && KSTG == 1),
                "paired tiles: local output, codes in shared memory");
  constexpr int kBRows = PAIR ? BN / 2 : BN;     // token rows of B in this CTA
  constexpr int kBStage = KSTG * kBRows * kBK;   // activation bytes per stage
  constexpr int kPStage = KSTG * kPackedBlock;   // packed weight bytes per stage
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  static_assert(STAGES <= 8, "stage count");
  uint8_t* sA = base;                                  // STAGES x kAStage (A in shared memory)
  uint8_t* sB = sA + (A_TMEM ? 0 : STAGES * kAStage);  // STAGES x kBStage
  uint8_t* sP = sB + STAGES * kBStage;                 // STAGES x kPStage
  GemmSmem* sm = reinterpret_cast<GemmSmem*>(sP + STAGES * kPStage);
  float* sE = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(sm + 1) + 15) &
                                       ~static_cast<uintptr_t>(15));  // gather staging

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB = K / kBK;
  const int n_stages = (KB + KSTG - 1) / KSTG;  // a missing last block is zero-filled by TMA
  const int num_m = (M + (PAIR ? 2 : 1) * kBM - 1) / ((PAIR ? 2 : 1) * kBM);  // (paired) row tiles
  const int num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  // half tiles (tmap_qh: BN / 4 token rows per CTA) only on pairs
  const int split_from = PAIR ? (split_arg < 0 ? 0 : split_arg < tiles ? split_arg : tiles) : tiles;
  const int units = 2 * tiles - split_from;
  const uint32_t crank = PAIR ? pair_rank() : 0u;  // 0: issues the pair's MMAs
  const int t0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tstep = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // TMEM columns: two BN-wide accumulators, then (A_TMEM) 32 columns per block per stage.
  constexpr uint32_t kTmemNeed = 2 * BN + (A_TMEM ? 32 * KSTG * STAGES : 0);
  constexpr uint32_t kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128
                                 : kTmemNeed <= 256 ? 256 : 512;
  static_assert(kTmemNeed <= 512, "TMEM budget");

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm->full_tma[s], 1);
      mbar_init(&sm->full_a[s], PAIR ? 8 : 4);  // one arrival per expansion warp (both CTAs)
      mbar_init(&sm->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm->accf[a], 1);
      mbar_init(&sm->acce[a], PAIR ? 8 : 4);  // one arrival per epilogue warp (both CTAs)
    }
    mbar_init(&sm->drain, 1);
    sm->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&sm->tmem_base, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&sm->tmem_base, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) pair_sync();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = sm->tmem_base;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop (converged); one lane issues the copies.
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
      if (PAIR && split_from < tiles)
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_qh) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w) : "memory");
    }
    int it = 0;
    bool waited = false;
    for (int u = t0; u < units && !sm->abort_flag; u += tstep) {
      const TileUnit tu = tile_unit(u, num_m, split_from, BN);
      const int rowtile = PAIR ? 2 * tu.mt + static_cast<int>(crank) : tu.mt;
      const bool half = PAIR && tu.half;
      bool ok = true;
      for (int st = 0; st < n_stages; ++st, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        if (!wait_x<PAIR>(sm, &sm->empty[s], ph ^ 1u)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&sm->full_tma[s], (half ? kBStage / 2 : kBStage) + kPStage);
          tma_load_3d(sP + s * kPStage, &tmap_w, 0, st * KSTG, rowtile * (kBM / kSubRows),
                      &sm->full_tma[s]);
        }
        if (!waited) {  // q comes from the previous kernel; the weights do not
          pdl_wait();
          waited = true;
        }
        if (lane == 0) {
          // a half unit: this CTA's BN / 4 token rows land in the first half of
          // the stage (KSTG == 1 on pairs), where the N = BN / 2 MMA reads them
          if (half)
            tma_load_3d(sB + s * kBStage, &tmap_qh, 0,
                        tu.tok0 + static_cast<int>(crank) * (kBRows / 2), st * KSTG,
                        &sm->full_tma[s]);
          else
            tma_load_3d(sB + s * kBStage, &tmap_q, 0, tu.tok0 + static_cast<int>(crank) * kBRows,
                        st * KSTG, &sm->full_tma[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
    }
    if (!waited) pdl_wait();
    // Drain: wait (bounded) for every copy this warp issued before exiting.
    const int last = it;
    for (int j = (last > STAGES ? last - STAGES : 0); j < last; ++j)
      mbar_wait(&sm->full_tma[j % STAGES], (j / STAGES) & 1u);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Converged warp; one lane issues the MMAs and commits.
    pdl_wait();
    int it = 0, ti = 0;
    constexpr uint32_t kIdesc = PAIR ? idesc_i8_pair<BN>() : idesc_i8<BN>();
    constexpr uint32_t kIdescHalf = PAIR ? idesc_i8_pair<BN / 2>() : idesc_i8<BN>();
    // PAIR: the odd CTA's MMA warp issues nothing (its rows are in the even CTA's MMAs)
    for (int u = t0; u < units && !sm->abort_flag && (!PAIR || crank == 0); u += tstep, ++ti) {
      const uint32_t idesc = u >= split_from ? kIdescHalf : kIdesc;
      const int a = ti & 1;
      const uint32_t aph = (ti >> 1) & 1u;
      if (!wait_x<PAIR>(sm, &sm->acce[a], aph ^ 1u)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + a * BN;
      bool ok = true;
      for (int st = 0; st < n_stages; ++st, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        // full_a implies full_tma: the expansion warps arrive only after waiting
        // for this stage's TMA bytes (weights and activations share the barrier).
        if (!wait_x<PAIR>(sm, &sm->full_a[s], ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          // Straight-line MMA burst: descriptors are one base plus constant steps
          // (start address in 16-byte units, no carry out of its 14-bit field).
          const uint64_t bdesc0 = sw128_desc(smem_u32(sB + s * kBStage));
#pragma unroll
          for (int bb = 0; bb < KSTG; ++bb) {
            if (A_TMEM) {
              const uint32_t a_tmem = tmem + 2 * BN + (s * KSTG + bb) * 32;
#pragma unroll
              for (int kk = 0; kk < kBK / 32; ++kk)
                mma_i8_ts(d_tmem, a_tmem + kk * 8,
                          bdesc0 + static_cast<uint64_t>((bb * BN * kBK + kk * 32) >> 4), idesc,
                          (st > 0 || bb > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint32_t b_addr = smem_u32(sB + s * kBStage + bb * kBRows * kBK);
              const uint32_t a_addr = smem_u32(sA + s * kAStage + bb * kBM * kBK);
#pragma unroll
              for (int kk = 0; kk < kBK / 32; ++kk)
                if constexpr (PAIR)
                  mma_i8_pair(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32),
                              idesc, (st > 0 || bb > 0 || kk > 0) ? 1u : 0u);
                else
                  mma_i8(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                         (st > 0 || bb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          if constexpr (PAIR)
            commit_pair(&sm->empty[s]);  // both CTAs' copy stages are free again
          else
            mma_commit(&sm->empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) {
        if constexpr (PAIR)
          commit_pair(&sm->accf[a]);
        else
          mma_commit(&sm->accf[a]);
      }
      __syncwarp();
    }
    // Every MMA issued by this warp must finish before TMEM is released.
    if constexpr (PAIR) {
      if (lane == 0 && crank == 0) commit_pair(&sm->drain);
      __syncwarp();
      mbar_wait_cl(&sm->drain, 0);
    } else {
      if (lane == 0) mma_commit(&sm->drain);
      __syncwarp();
      mbar_wait(&sm->drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ expansion
    pdl_wait();
    const int r = tid - 128;  // weight row within the tile = TMEM lane
    const int sub = r >> 4, rr = r & 15;
    int it = 0;
    for (int u = t0; u < units && !sm->abort_flag; u += tstep) {
      bool ok = true;
      for (int st = 0; st < n_stages; ++st, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        if (!wait_or_abort(sm, &sm->full_tma[s], ph)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int bb = 0; bb < KSTG; ++bb) {
          // P stage layout [8 subtiles][KSTG blocks][512 B]
          const uint8_t* p = sP + s * kPStage + (sub * KSTG + bb) * kSubtileBytes + rr * 16;
          if (A_TMEM) {
            // Row r's 128 codes as 32 words, word j = codes of k = 4j .. 4j+3; the
            // 16-k chunk c = 2g + h is words 4c .. 4c+3.
            uint32_t v[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint4 w = *reinterpret_cast<const uint4*>(p + h * 256);
#pragma unroll
              for (int g = 0; g < 4; ++g) {
                const int sh = 6 - 2 * g, c = 2 * g + h;
                v[4 * c + 0] = (w.x >> sh) & 0x03030303u;
                v[4 * c + 1] = (w.y >> sh) & 0x03030303u;
                v[4 * c + 2] = (w.z >> sh) & 0x03030303u;
                v[4 * c + 3] = (w.w >> sh) & 0x03030303u;
              }
            }
            tmem_st32(tmem + (static_cast<uint32_t>(r & ~31) << 16) + 2 * BN + (s * KSTG + bb) * 32,
                      v);
          } else {
            uint8_t* arow = sA + s * kAStage + bb * kBM * kBK + (r >> 3) * 1024 + (r & 7) * 128;
            const uint32_t swz = static_cast<uint32_t>(r & 7);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint4 w = *reinterpret_cast<const uint4*>(p + h * 256);
#pragma unroll
              for (int g = 0; g < 4; ++g) {
                const int sh = 6 - 2 * g;
                uint4 c;
                c.x = (w.x >> sh) & 0x03030303u;
                c.y = (w.y >> sh) & 0x03030303u;
                c.z = (w.z >> sh) & 0x03030303u;
                c.w = (w.w >> sh) & 0x03030303u;
                const uint32_t chunk = static_cast<uint32_t>(2 * g + h) ^ swz;
                *reinterpret_cast<uint4*>(arow + chunk * 16) = c;
              }
            }
          }
        }
        if (A_TMEM) {
          tmem_st_wait();
          tc_fence_before();
        } else {
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        }
        __syncwarp();
        // PAIR: the even CTA's MMAs make each CTA's tensor core read its own
        // codes, so the odd CTA only has to tell the even one that its codes are
        // in place: a relaxed arrival, issued after this warp's writes were made
        // visible to the async proxy by the (blocking) fence above. A release at
        // cluster scope would order nothing more here and stalls the thread for
        // ~1.5 k cycles while the SM's global stores drain.
        if (lane == 0) {
          if (PAIR && crank == 1)
            arrive_cluster_relaxed(pair_map(smem_u32(&sm->full_a[s]), 0));
          else
            mbar_arrive(&sm->full_a[s]);
        }
      }
      if (!ok) break;
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int ti = 0;
    for (int u = t0; u < units && !sm->abort_flag; u += tstep, ++ti) {
      const TileUnit tu = tile_unit(u, num_m, split_from, BN);
      const int mt = tu.mt, tok0 = tu.tok0;
      const int rowtile = PAIR ? 2 * mt + static_cast<int>(crank) : mt;
      const int a = ti & 1;
      const uint32_t aph = (ti >> 1) & 1u;
      const int m = rowtile * kBM + quarter * 32 + lane;
      if constexpr (OUT == kOutLocal) {
        // The tile's per-token code sums and scales are kernel inputs: load them
        // before waiting for the accumulator, lane l holding columns l, l + 32, ...
        // (l, l + 16, ... when BN = 16), and broadcast each column by a shuffle.
        constexpr int kCols = BN < 32 ? BN : 32;  // columns per TMEM load
        constexpr int kChunks = BN / kCols;
        int qsr[kChunks];
        float sxr[kChunks];
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          const int nl = tok0 + c * kCols + (lane % kCols);
          qsr[c] = nl < N ? qsum[nl] : 0;
          sxr[c] = (nl < N && !acc_out) ? s_x[nl] : 0.0f;
        }
        const float sw = (m < M && !acc_out) ? s_w[m] : 0.0f;
        if (!wait_x<PAIR>(sm, &sm->accf[a], aph)) break;
        tc_fence_after();
        const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
        // Five store kinds, chosen once per tile so the plain store never carries
        // a (speculated) read of y: int32 accumulators, y = val, y += val, and
        // gated pairs with ReLU^2 (3) or SiLU (4) compiled in (rows 2i, 2i + 1 in
        // lanes 2i, 2i + 1: the even lane writes act(gate) * up to y[t, i], y being
        // [N][M / 2]).
        const int kind = acc_out                  ? 0
                         : (order & kOutGated)    ? ((order & kOutSilu) ? 4 : 3)
                         : (order & kOutAccumulate) ? 2
                                                    : 1;
        const bool gemv_order = (order & 1) == kOrderGemv;
        const size_t Mh = static_cast<size_t>(M) >> 1;
        // a half unit's accumulator holds BN / 2 columns
        const int width = tu.half ? BN / 2 : BN;
        const int nchunks = width / kCols;
        const bool full_tile = tok0 + width <= N && (rowtile + 1) * kBM <= M;
        auto chunk = [&](auto kind_c) {
          constexpr int K_ = decltype(kind_c)::value;
          if constexpr (K_ >= 3) {
            if (full_tile) {
              // Gated pairs: lanes 2i (gate row) and 2i + 1 (up row) swap one
              // value per column pair (2k, 2k + 1), so the even lane forms column
              // 2k and the odd lane column 2k + 1: every lane stores. The chunk
              // loop stays rolled (the column scalars shift down one chunk per
              // pass) to keep the epilogue's code small next to the other roles'.
              int qr[kChunks];
              float xr[kChunks];
#pragma unroll
              for (int c = 0; c < kChunks; ++c) {
                qr[c] = qsr[c];
                xr[c] = sxr[c];
              }
              const bool odd = (m & 1) != 0;
              float* yb = y + static_cast<size_t>(tok0 + (odd ? 1 : 0)) * Mh + (m >> 1);
#pragma unroll 1
              for (int c = 0; c < nchunks; ++c) {
                uint32_t v[kCols];
                if constexpr (kCols == 32)
                  tmem_ld32(taddr + c * 32, v);
                else
                  tmem_ld16(taddr + c * 16, v);
                int qs_v[kCols];
                float sx_v[kCols];
#pragma unroll
                for (int j = 0; j < kCols; ++j) {
                  qs_v[j] = __shfl_sync(0xffffffffu, qr[0], j);
                  sx_v[j] = __shfl_sync(0xffffffffu, xr[0], j);
                }
                tmem_ld_wait();
                float val[kCols];
#pragma unroll
                for (int j = 0; j < kCols; ++j) {
                  const float fd = static_cast<float>(static_cast<int>(v[j]) - qs_v[j]);
                  val[j] = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx_v[j])
                                      : __fmul_rn(fd, __fmul_rn(sw, sx_v[j]));
                }
#pragma unroll
                for (int k = 0; k < kCols / 2; ++k) {
                  const float r =
                      __shfl_xor_sync(0xffffffffu, odd ? val[2 * k] : val[2 * k + 1], 1);
                  const float g = odd ? r : val[2 * k];
                  const float u = odd ? val[2 * k + 1] : r;
                  yb[static_cast<size_t>(2 * k) * Mh] = __fmul_rn(gate_act(K_ - 3, g), u);
                }
                yb += static_cast<size_t>(kCols) * Mh;
#pragma unroll
                for (int k = 0; k + 1 < kChunks; ++k) {
                  qr[k] = qr[k + 1];
                  xr[k] = xr[k + 1];
                }
              }
              return;
            }
          }
          if (K_ < 3 && full_tile) {
            // Every column and row in range: branch-free chunks, the 2 * kCols
            // broadcasts first, so the conversions, products and stores of a
            // chunk issue back to back instead of one column's chain at a time.
            // The chunk loop stays rolled (column scalars shifted down a chunk
            // per pass): the unrolled epilogue's code crowded the instruction
            // cache the producer, expansion and MMA warps share.
            int qr[kChunks];
            float xr[kChunks];
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
              qr[c] = qsr[c];
              xr[c] = sxr[c];
            }
#pragma unroll 1
            for (int c = 0; c < nchunks; ++c) {
              uint32_t v[kCols];
              if constexpr (kCols == 32)
                tmem_ld32(taddr + c * 32, v);
              else
                tmem_ld16(taddr + c * 16, v);
              const size_t o0 = static_cast<size_t>(tok0 + c * kCols) * M + m;
              // y += val: every load of the chunk issues before its first store (a
              // load after a store to y would wait for the one before it)
              float yv[K_ == 2 ? kCols : 1];
              if constexpr (K_ == 2) {
#pragma unroll
                for (int j = 0; j < kCols; ++j) yv[j] = y[o0 + static_cast<size_t>(j) * M];
              }
              int qs_v[kCols];
              float sx_v[kCols];
#pragma unroll
              for (int j = 0; j < kCols; ++j) {
                qs_v[j] = __shfl_sync(0xffffffffu, qr[0], j);
                sx_v[j] = __shfl_sync(0xffffffffu, xr[0], j);
              }
#pragma unroll
              for (int k = 0; k + 1 < kChunks; ++k) {
                qr[k] = qr[k + 1];
                xr[k] = xr[k + 1];
              }
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < kCols; ++j) {
                const int d = static_cast<int>(v[j]) - qs_v[j];
                const size_t o = o0 + static_cast<size_t>(j) * M;
                if constexpr (K_ == 0) {
                  acc_out[o] = d;
                } else {
                  const float fd = static_cast<float>(d);
                  const float val = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx_v[j])
                                               : __fmul_rn(fd, __fmul_rn(sw, sx_v[j]));
                  if constexpr (K_ == 2)
                    y[o] = __fadd_rn(yv[j], val);
                  else
                    y[o] = val;
                }
              }
            }
            return;
          }
          // Partial tiles: per-column bounds checks, the chunk loop rolled as above.
          int qr[kChunks];
          float xr[kChunks];
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            qr[c] = qsr[c];
            xr[c] = sxr[c];
          }
#pragma unroll 1
          for (int c = 0; c < nchunks; ++c) {
            uint32_t v[kCols];
            if constexpr (kCols == 32)
              tmem_ld32(taddr + c * 32, v);
            else
              tmem_ld16(taddr + c * 16, v);
            const int qs_c = qr[0];
            const float sx_c = xr[0];
#pragma unroll
            for (int k = 0; k + 1 < kChunks; ++k) {
              qr[k] = qr[k + 1];
              xr[k] = xr[k + 1];
            }
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < kCols; ++j) {
              const int n = tok0 + c * kCols + j;
              const int qs_j = __shfl_sync(0xffffffffu, qs_c, j);
              const float sx_j = __shfl_sync(0xffffffffu, sx_c, j);
              if constexpr (K_ >= 3) {  // the pair's shuffle runs in every lane
                const float fd = static_cast<float>(static_cast<int>(v[j]) - qs_j);
                const float val = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx_j)
                                             : __fmul_rn(fd, __fmul_rn(sw, sx_j));
                const float up = __shfl_down_sync(0xffffffffu, val, 1);
                if (n < N && m < M && (m & 1) == 0)
                  y[static_cast<size_t>(n) * Mh + (m >> 1)] = __fmul_rn(gate_act(K_ - 3, val), up);
              } else if (n < N && m < M) {
                const int d = static_cast<int>(v[j]) - qs_j;
                const size_t o = static_cast<size_t>(n) * M + m;
                if constexpr (K_ == 0) {
                  acc_out[o] = d;
                } else {
                  const float fd = static_cast<float>(d);
                  const float val = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx_j)
                                               : __fmul_rn(fd, __fmul_rn(sw, sx_j));
                  if constexpr (K_ == 2)
                    y[o] = __fadd_rn(y[o], val);
                  else
                    y[o] = val;
                }
              }
            }
          }
        };
        if (kind == 0)
          chunk(std::integral_constant<int, 0>());
        else if (kind == 1)
          chunk(std::integral_constant<int, 1>());
        else if (kind == 2)
          chunk(std::integral_constant<int, 2>());
        else if (kind == 3)
          chunk(std::integral_constant<int, 3>());
        else
          chunk(std::integral_constant<int, 4>());
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {  // PAIR: the even CTA reuses the pair's accumulator
          if (PAIR && crank == 1)  // the TMEM reads above completed (tcgen05.wait::ld)
            arrive_cluster_relaxed(pair_map(smem_u32(&sm->acce[a]), 0));
          else
            mbar_arrive(&sm->acce[a]);
        }
        continue;
      }
      if (!wait_or_abort(sm, &sm->accf[a], aph)) break;
      tc_fence_after();
      const float sw = (m < M && !acc_out) ? s_w[m] : 0.0f;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 16) {
        uint32_t v[16];
        tmem_ld16(taddr + j0, v);
        tmem_ld_wait();
        const int n0 = tok0 + j0;
        // Column j's code sum and scale, fetched once per warp and broadcast.
        const int nl = n0 + (lane & 15);
        const int qs_l = nl < N ? qsum[nl] : 0;
        const float sx_l = (nl < N && !acc_out) ? s_x[nl] : 0.0f;
        if (OUT != kOutLocal && go.vec4) {
          // Stage the chunk as [16 tokens][32 rows], then 16-byte stores of 4
          // consecutive rows (conflict-free: 8 lanes read one token's 128 bytes).
          float* st = sE + (warp & 3) * (16 * 32);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int qs_j = __shfl_sync(0xffffffffu, qs_l, j);
            const float sx_j = __shfl_sync(0xffffffffu, sx_l, j);
            const float fd = static_cast<float>(static_cast<int>(v[j]) - qs_j);
            st[j * 32 + lane] = (order & 1) == kOrderGemv ? __fmul_rn(__fmul_rn(fd, sw), sx_j)
                                                    : __fmul_rn(fd, __fmul_rn(sw, sx_j));
          }
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int i = it * 32 + lane;
            const int jj = i >> 3, r4 = (i & 7) * 4;
            const int n = n0 + jj;
            const int mrow = mt * kBM + quarter * 32 + r4;
            if (n < N && mrow < M) {
              const float4 v4 = *reinterpret_cast<const float4*>(st + jj * 32 + r4);
              const size_t og = static_cast<size_t>(n) * go.ldy + go.col0 + mrow;
              if constexpr (OUT == kOutMulticast) {
                multimem_st_v4(go.mc + og, v4);
              } else {
#pragma unroll
                for (int p = 0; p < kMaxGatherRanks; ++p)
                  if (p < go.world) *reinterpret_cast<float4*>(go.ranks[p] + og) = v4;
              }
            }
          }
          __syncwarp();
          continue;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + j;
          const int qs_j = __shfl_sync(0xffffffffu, qs_l, j);
          const float sx_j = __shfl_sync(0xffffffffu, sx_l, j);
          if (n < N && m < M) {
            const int d = static_cast<int>(v[j]) - qs_j;
            const size_t o = static_cast<size_t>(n) * M + m;
            if (OUT == kOutLocal && acc_out) {
              acc_out[o] = d;
            } else {
              const float fd = static_cast<float>(d);
              const float val = (order & 1) == kOrderGemv ? __fmul_rn(__fmul_rn(fd, sw), sx_j)
                                                          : __fmul_rn(fd, __fmul_rn(sw, sx_j));
              if constexpr (OUT == kOutLocal) {
                y[o] = (order & kOutAccumulate) ? __fadd_rn(y[o], val) : val;
              } else {
                const size_t og = static_cast<size_t>(n) * go.ldy + go.col0 + m;
                if constexpr (OUT == kOutMulticast) {
                  multimem_st_f32(go.mc + og, val);
                } else {
#pragma unroll
                  for (int p = 0; p < kMaxGatherRanks; ++p)
                    if (p < go.world) go.ranks[p][og] = val;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm->acce[a]);
    }
    // Gathered outputs: this thread's remote stores are performed before the
    // kernel completes, so a stream-ordered barrier after it publishes them.
    if constexpr (OUT != kOutLocal) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  // PAIR: no CTA leaves (or frees TMEM) while the other may still arrive on its
  // barriers or its MMAs may still read this CTA's shared memory.
  if constexpr (PAIR) pair_sync();
  tc_fence_after();
  if (warp == 2) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, kTmemCols);
    else
      tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- split-K over a thread-block cluster ---------------------------------------------
//
// Decode-sized token counts leave too few 128-row tiles to occupy the GPU
// (20 tiles for a 2560-row layer). k_gemm_sk gives each tile a cluster of S
// CTAs (S <= 8); rank r takes the K blocks [r*KB/S, (r+1)*KB/S). A CTA's whole
// slice is in flight at once (at most sk_blocks<BN>() blocks: their
// activations, packed weights and expanded codes all fit), so no buffer is
// recycled and the MMAs end in a single tcgen05.commit:
//   - the producer issues every weight copy first, then, after the wait on the
//     previous kernel, every activation copy, with one barrier each per block;
//   - the expansion warps turn each block's weights into codes in TMEM as soon
//     as they land, overlapping the previous kernel's tail;
//   - the MMA warp issues a block's 4 MMAs once its codes and activations are in.
// Each CTA accumulates its partial in its own TMEM. The reduction is a
// reduce-scatter over distributed shared memory driven by the bulk-copy engine:
// each CTA stages its partial tile in its own shared memory, then one thread
// sends every owner rank o the rows [o*RB, o*RB+RB) (RB = ceil(128/S) rounded up
// to even, so a gated layer's gate|up row pair has one owner) with one
// cp.async.bulk shared::cta -> shared::cluster copy into slot [src] of the
// owner's buffer, completing as transaction bytes on the owner's mbarrier; the
// owner sums its S slots in rank order (integers: exact) and writes the outputs.
// A split cluster barrier (arrive early, wait late) orders the barrier inits
// before the first send and keeps every CTA's shared memory alive until no copy
// reads or writes it.
//
// One CTA per SM (shared memory is padded past half an SM): two CTAs of
// different clusters on one SM would serialise on the TMEM allocation while
// each cluster waits for all of its ranks.

OBN_DEVINL uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Relaxed arrive: nothing is published through the cluster barrier itself
// (barrier inits are released by fence.mbarrier_init, copied rows by their
// mbarrier's transaction count), and a release arrive costs about a microsecond.
OBN_DEVINL void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
OBN_DEVINL void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
OBN_DEVINL uint32_t map_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// Shared memory of this CTA -> shared memory of a CTA in the cluster (mapa
// addresses), completing `bytes` of transactions on that CTA's mbarrier.
OBN_DEVINL void bulk_s2cluster(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                               uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

OBN_DEVINL bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

constexpr int kRedRows = 140;  // >= S * RB for every S <= 8 (7 * 20)
constexpr int kSplitKDefaultCtas = 148;
constexpr size_t kSkMinSmem = 120 * 1024;

constexpr int kSkGroup = 4;  // K blocks behind one barrier (16 MMAs per burst)

template <int NB>
struct SkSmem {
  static constexpr int NG = (NB + kSkGroup - 1) / kSkGroup;
  uint64_t wfull[NG];   // packed weights of group g landed
  uint64_t afull[NG];   // activations of group g landed
  uint64_t full_a[NG];  // codes of group g in TMEM (one arrival per expanding warp)
  uint64_t accf;        // every MMA done
  uint64_t red_full;    // incoming partial rows (transaction bytes)
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort_flag;
};

// K blocks one split-K CTA holds at once: TMEM (BN accumulator columns + 32 code
// columns per block <= 512) and shared memory (4 KB of weights + BN*128 bytes
// of activations per block, next to the reduction buffer).
template <int BN>
constexpr int sk_blocks() {
  return BN <= 32 ? 15 : BN <= 64 ? 14 : 7;
}

template <int BN>
constexpr size_t sk_smem_bytes() {
  return 1024 + static_cast<size_t>(sk_blocks<BN>()) * (BN * kBK + kPackedBlock) +
         static_cast<size_t>(kRedRows) * (BN + 4) * 4 + (2 * BN + kBM) * 4 +
         sizeof(SkSmem<sk_blocks<BN>()>);
}

template <int BN>
constexpr size_t sk_smem_launch() {
  return sk_smem_bytes<BN>() < kSkMinSmem ? kSkMinSmem : sk_smem_bytes<BN>();
}

// Expansion of the groups g = set, set + 2, ... of a split-K CTA's slice by one
// of its two 4-warp sets (warps 4-7: set 0, warps 8-11: set 1). Thread = weight
// row = TMEM lane (warp % 4 selects the lane quarter); codes c = w + 1 as u8.
// All of a group's TMEM stores are in flight before one wait.
template <int BN, int NB>
OBN_DEVINL void sk_expand(SkSmem<NB>* sm, const uint8_t* sP, uint32_t tmem, int nb, int set) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = (warp & 3) * 32 + lane;
  const int sub = r >> 4, rr = r & 15;
  const int ng = (nb + kSkGroup - 1) / kSkGroup;
  for (int g = set; g < ng; g += 2) {
    if (!wait_or_abort(sm, &sm->wfull[g], 0)) break;
    const int bg = g * kSkGroup, be = min(bg + kSkGroup, nb);
    for (int b = bg; b < be; ++b) {
      const uint8_t* p = sP + b * kPackedBlock + sub * kSubtileBytes + rr * 16;
      uint32_t v[32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 w = *reinterpret_cast<const uint4*>(p + h * 256);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int sh = 6 - 2 * q, c = 2 * q + h;
          v[4 * c + 0] = (w.x >> sh) & 0x03030303u;
          v[4 * c + 1] = (w.y >> sh) & 0x03030303u;
          v[4 * c + 2] = (w.z >> sh) & 0x03030303u;
          v[4 * c + 3] = (w.w >> sh) & 0x03030303u;
        }
      }
      tmem_st32(tmem + (static_cast<uint32_t>(r & ~31) << 16) + BN + b * 32, v);
    }
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm->full_a[g]);
  }
}

template <int BN>
__global__ __launch_bounds__(kThreads, 1) void k_gemm_sk(const __grid_constant__ CUtensorMap tmap_q,
                                                         const __grid_constant__ CUtensorMap tmap_w,
                                                         const float* __restrict__ s_w,
                                                         const float* __restrict__ s_x,
                                                         const int32_t* __restrict__ qsum,
                                                         float* __restrict__ y,
                                                         int32_t* __restrict__ acc_out, int M,
                                                         int N, int K, int order) {
  constexpr int NB = sk_blocks<BN>();
  constexpr int kBBlock = BN * kBK;  // activation bytes per block
  constexpr int BNP = BN + 4;        // padded reduction row (ints): conflict-free lane strides
  constexpr uint32_t kTmemCols = 512;
  static_assert(BN + 32 * NB <= static_cast<int>(kTmemCols), "TMEM budget");
  static_assert(kBM * BNP * 4 <= NB * kBBlock, "staged partial tile fits the activation blocks");
  static_assert((BNP * 4) % 16 == 0, "bulk copies move whole 16-byte units");
  static_assert(sk_smem_bytes<BN>() <= 232448, "shared memory budget");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sB = base;                                                // NB x [BN][128], SW128
  uint8_t* sP = sB + NB * kBBlock;                                   // NB x 4 KB packed
  int32_t* red = reinterpret_cast<int32_t*>(sP + NB * kPackedBlock);  // [S][RB][BNP]
  int32_t* e_qs = red + kRedRows * BNP;                                // [BN] column code sums
  float* e_sx = reinterpret_cast<float*>(e_qs + BN);                   // [BN] column scales
  float* e_sw = e_sx + BN;                                             // [kBM] row scales
  SkSmem<NB>* sm = reinterpret_cast<SkSmem<NB>*>(e_sw + kBM);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t S = gridDim.x;  // cluster = the whole x dimension
  const uint32_t rank = cluster_ctarank();
  const int mt = blockIdx.y;
  const int KB = K / kBK;
  const int b0 = static_cast<int>(rank * KB / S);
  const int nb_slice = static_cast<int>((rank + 1) * KB / S) - b0;
  const int nb = min(nb_slice, NB);  // the host keeps every slice within NB blocks
  const int RB = (((kBM + static_cast<int>(S) - 1) / static_cast<int>(S)) + 1) & ~1;
  // The owner reduce below decodes row blocks for 1 or 2 blocks of 32 rows (RB <= 64),
  // which holds for 2 <= S <= 8; any other launch records an error and skips it.
  const bool geom_ok = nb_slice <= NB && S >= 2 && S <= 8 && RB <= 64;
  if (tid == 0 && !geom_ok) record_error(DEVERR_BAD_LAUNCH);

  const int ng = (nb + kSkGroup - 1) / kSkGroup;
  if (tid == 0) {
    for (int g = 0; g < ng; ++g) {
      mbar_init(&sm->wfull[g], 1);
      mbar_init(&sm->afull[g], 1);
      mbar_init(&sm->full_a[g], 4);
    }
    mbar_init(&sm->accf, 1);
    mbar_init(&sm->red_full, 1);
    mbar_init(&sm->drain, 1);
    sm->abort_flag = 0;
    fence_mbar_init();
    // Armed before this CTA's cluster arrive: no peer sends before its wait.
    const int own_rows = min(RB, kBM - static_cast<int>(rank) * RB);
    mbar_arrive_expect_tx(&sm->red_full, S * static_cast<uint32_t>(own_rows) * BNP * 4);
  }
  if (warp == 2) {
    tmem_alloc(&sm->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  // Cluster barrier, phase 0: published barrier inits. Only the epilogue's sends
  // depend on it, so every thread arrives now and waits when it must.
  cluster_arrive();
  tc_fence_after();
  const uint32_t tmem = sm->tmem_base;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The weights do not depend on the previous kernel; the activations do.
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_w) : "memory");
      for (int g = 0; g < ng; ++g) {
        const int bg = g * kSkGroup, ne = min(kSkGroup, nb - bg);
        mbar_arrive_expect_tx(&sm->wfull[g], ne * kPackedBlock);
        for (int b = bg; b < bg + ne; ++b)
          tma_load_3d(sP + b * kPackedBlock, &tmap_w, 0, b0 + b, mt * (kBM / kSubRows),
                      &sm->wfull[g]);
      }
    }
    __syncwarp();
    pdl_wait();
    if (lane == 0)
      for (int g = 0; g < ng; ++g) {
        const int bg = g * kSkGroup, ne = min(kSkGroup, nb - bg);
        mbar_arrive_expect_tx(&sm->afull[g], ne * kBBlock);
        for (int b = bg; b < bg + ne; ++b)
          tma_load_3d(sB + b * kBBlock, &tmap_q, 0, 0, b0 + b, &sm->afull[g]);
      }
    __syncwarp();
    // Every copy has landed before the CTA exits (immediate unless it aborted).
    for (int g = 0; g < ng; ++g) {
      mbar_wait(&sm->wfull[g], 0);
      mbar_wait(&sm->afull[g], 0);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_i8<BN>();
    bool ok = true;
    // One wait pair per group, then a straight burst of its MMAs (a wait costs
    // about as much as two MMAs even when its phase completed long ago).
    for (int g = 0; g < ng; ++g) {
      if (!wait_or_abort(sm, &sm->full_a[g], 0) || !wait_or_abort(sm, &sm->afull[g], 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const int bg = g * kSkGroup, be = min(bg + kSkGroup, nb);
        for (int b = bg; b < be; ++b) {
          const uint32_t b_addr = smem_u32(sB + b * kBBlock);
          const uint32_t a_tmem = tmem + BN + b * 32;
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            mma_i8_ts(tmem, a_tmem + kk * 8, sw128_desc(b_addr + kk * 32), idesc,
                      (b > 0 || kk > 0) ? 1u : 0u);
        }
      }
      __syncwarp();
    }
    if (lane == 0) {
      if (ok) mma_commit(&sm->accf);
      mma_commit(&sm->drain);
    }
    __syncwarp();
    mbar_wait(&sm->drain, 0);
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ expansion
    sk_expand<BN, NB>(sm, sP, tmem, nb, 0);
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    // First the odd expansion groups (no dependence on the previous kernel).
    sk_expand<BN, NB>(sm, sP, tmem, nb, 1);
    pdl_wait();
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // tile row = TMEM lane
    // Scalars for the owned rows' outputs, fetched while the MMAs run and
    // published by the epilogue barrier below.
    const int t = tid - 256;
    if (t < BN) {
      e_qs[t] = t < N ? qsum[t] : 0;
      e_sx[t] = (t < N && !acc_out) ? s_x[t] : 0.0f;
    }
    {
      const int m = mt * kBM + t;
      e_sw[t] = (m < M && !acc_out) ? s_w[m] : 0.0f;
    }
    bool have = nb > 0 && wait_or_abort(sm, &sm->accf, 0);
    tc_fence_after();
    // Stage the partial tile locally; the activation blocks are free once every
    // MMA has completed (accf).
    int32_t* part = reinterpret_cast<int32_t*>(sB);
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
    for (int j0 = 0; j0 < BN; j0 += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + j0, v);
      tmem_ld_wait();
      if (!have) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0;  // no K stages here: contribute zero
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(part + r * BNP + j0 + 4 * i) =
            make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    tc_fence_before();
    fence_proxy_async_smem();  // generic stores -> visible to the bulk-copy engine
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
    cluster_wait();  // phase 0: every peer's red_full is initialised and armed
    if (tid == 256) {
      for (uint32_t o = 0; o < S; ++o) {
        const int rows_o = min(RB, kBM - static_cast<int>(o) * RB);
        if (rows_o <= 0) continue;
        bulk_s2cluster(map_rank(smem_u32(red + static_cast<int>(rank) * RB * BNP), o),
                       smem_u32(part + static_cast<int>(o) * RB * BNP),
                       static_cast<uint32_t>(rows_o) * BNP * 4, map_rank(smem_u32(&sm->red_full), o));
      }
    }
  }

  // ---------------------------------------------------------------- owner reduce
  // All 12 warps: a single warp per SM sub-partition leaves the dependent
  // load-add-scale-store chains exposed. The epilogue warps published the
  // column and row scalars before their barrier; the others finish phase 0 now.
  if (warp < 8) cluster_wait();
  __syncthreads();
  bool ok = false;
  for (uint32_t i = 0; i < kWaitLimit && !ok; ++i) ok = mbar_try_wait_cluster(&sm->red_full, 0);
  if (!ok && tid == 0) record_error(DEVERR_MBAR_TIMEOUT);
  __syncwarp();
  // Phase 1: this CTA's incoming copies are complete (so are the peers' reads
  // behind them); the wait before exit makes that true cluster-wide.
  cluster_arrive();
  // Work item (row block of 32, 4-column group) per warp; lane = row, so the
  // stores run over consecutive m. One 16-byte load per source rank, all issued
  // before the sums (a 4-word run of red is conflict-free across 8 lanes).
  const int row0 = static_cast<int>(rank) * RB;
  const int nrows = (row0 + RB <= kBM ? RB : kBM - row0);
  const int nrb = (nrows + 31) >> 5;  // 1 or 2 row blocks (RB <= 64)
  const int ngrp = (min(BN, N) + 7) >> 3;  // 8-column groups
  // The store kind (int32 accumulators, y = val, y += val, gated pairs) is fixed
  // per launch and compiled separately, so a plain store never carries a
  // speculated read of y. Gated pairs: row blocks start on even rows (RB is
  // even), so rows 2i and 2i + 1 sit in lanes 2i and 2i + 1 of one warp.
  const int kind = acc_out                    ? 0
                   : (order & kOutGated)      ? ((order & kOutSilu) ? 4 : 3)
                   : (order & kOutAccumulate) ? 2
                                              : 1;
  const bool gemv_order = (order & 1) == kOrderGemv;
  const size_t Mh = static_cast<size_t>(M) >> 1;
  auto reduce = [&](auto kind_c) {
    constexpr int K_ = decltype(kind_c)::value;
    for (int item = warp; item < nrb * ngrp; item += kThreads / 32) {
      const int rb = item & (nrb - 1), grp = item >> (nrb - 1);  // nrb is 1 or 2
      int rr = rb * 32 + lane;
      const int m = mt * kBM + row0 + rr;
      const bool valid = rr < nrows && m < M;
      if constexpr (K_ >= 3) {
        rr = valid ? rr : 0;  // every lane reaches the pair shuffle, on a real row
      } else {
        if (!valid) continue;
      }
      const int j0 = 8 * grp;
      // Every source rank's two 16-byte runs and the column scalars in flight
      // before the first sum.
      uint4 pa[8], pb[8];
#pragma unroll
      for (uint32_t src = 0; src < 8; ++src)
        if (src < S) {
          const int32_t* rp = red + (src * RB + rr) * BNP + j0;
          pa[src] = *reinterpret_cast<const uint4*>(rp);
          pb[src] = *reinterpret_cast<const uint4*>(rp + 4);
        }
      const int4 qa = *reinterpret_cast<const int4*>(e_qs + j0);
      const int4 qb = *reinterpret_cast<const int4*>(e_qs + j0 + 4);
      const float4 xa = *reinterpret_cast<const float4*>(e_sx + j0);
      const float4 xb = *reinterpret_cast<const float4*>(e_sx + j0 + 4);
      const float sw = e_sw[row0 + rr];
      int sum[8] = {-qa.x, -qa.y, -qa.z, -qa.w, -qb.x, -qb.y, -qb.z, -qb.w};
#pragma unroll
      for (uint32_t src = 0; src < 8; ++src)
        if (src < S) {
          sum[0] += static_cast<int>(pa[src].x);
          sum[1] += static_cast<int>(pa[src].y);
          sum[2] += static_cast<int>(pa[src].z);
          sum[3] += static_cast<int>(pa[src].w);
          sum[4] += static_cast<int>(pb[src].x);
          sum[5] += static_cast<int>(pb[src].y);
          sum[6] += static_cast<int>(pb[src].z);
          sum[7] += static_cast<int>(pb[src].w);
        }
      const float sx[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      auto put = [&](int c) {
        const size_t o = static_cast<size_t>(j0 + c) * M + m;
        if constexpr (K_ == 0) {
          acc_out[o] = sum[c];
        } else {
          const float fd = static_cast<float>(sum[c]);
          const float val = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx[c])
                                       : __fmul_rn(fd, __fmul_rn(sw, sx[c]));
          if constexpr (K_ == 2)
            y[o] = __fadd_rn(y[o], val);
          else
            y[o] = val;
        }
      };
      if constexpr (K_ >= 3) {
        // lanes 2i (gate) and 2i + 1 (up) swap one value per column pair: the even
        // lane forms column 2k, the odd lane column 2k + 1
        float val[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float fd = static_cast<float>(sum[c]);
          val[c] = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx[c])
                              : __fmul_rn(fd, __fmul_rn(sw, sx[c]));
        }
        const int odd = m & 1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float r = __shfl_xor_sync(0xffffffffu, odd ? val[2 * k] : val[2 * k + 1], 1);
          const float g = odd ? r : val[2 * k];
          const float u = odd ? val[2 * k + 1] : r;
          const int col = j0 + 2 * k + odd;
          if (valid && col < N)
            y[static_cast<size_t>(col) * Mh + (m >> 1)] = __fmul_rn(gate_act(K_ - 3, g), u);
        }
      } else if (j0 + 8 <= N) {
        if constexpr (K_ == 2) {  // y += val: the 8 loads first, then the stores
          float yv[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) yv[c] = y[static_cast<size_t>(j0 + c) * M + m];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float fd = static_cast<float>(sum[c]);
            const float val = gemv_order ? __fmul_rn(__fmul_rn(fd, sw), sx[c])
                                         : __fmul_rn(fd, __fmul_rn(sw, sx[c]));
            y[static_cast<size_t>(j0 + c) * M + m] = __fadd_rn(yv[c], val);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) put(c);
        }
      } else {
        for (int c = 0; c < 8 && j0 + c < N; ++c) put(c);
      }
    }
  };
  if (ok && geom_ok) {
    if (kind == 0)
      reduce(std::integral_constant<int, 0>());
    else if (kind == 1)
      reduce(std::integral_constant<int, 1>());
    else if (kind == 2)
      reduce(std::integral_constant<int, 2>());
    else if (kind == 3)
      reduce(std::integral_constant<int, 3>());
    else
      reduce(std::integral_constant<int, 4>());
  }

  tc_fence_before();
  __syncthreads();
  cluster_wait();  // phase 1: no copy still reads or writes any CTA's shared memory
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}


// ---- host side ------------------------------------------------------------------
EncodeTiledFn encode_fn() { return tensor_map_encoder(); }

template <int BN, int STAGES, int KSTG, bool A_TMEM, int OUT = kOutLocal, bool PAIR = false>
size_t gemm_smem_bytes() {
  return 1024 +
         static_cast<size_t>(STAGES) * ((A_TMEM ? 0 : KSTG * kBM * kBK) +
                                        KSTG * (PAIR ? BN / 2 : BN) * kBK + KSTG * kPackedBlock) +
         sizeof(GemmSmem) + (OUT == kOutLocal ? 0 : 16 + kGatherStageBytes);
}

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] ? sms[dev] : 148;
}

// Activations q [n][K] int8 viewed as 3D {128 bytes of a block, n tokens, KB blocks}
// so one box brings KSTG K-major [BN][128] tiles; 128-byte swizzle for the MMA.
bool make_q_map(CUtensorMap* map, const int8_t* q, int n, int K, int BN, int KSTG) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kBK), static_cast<cuuint64_t>(n),
                              static_cast<cuuint64_t>(K / kBK)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(kBK)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(BN),
                             static_cast<cuuint32_t>(KSTG)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(q), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// T16 weights viewed as 3D u32 {128 words of a subtile block, KB blocks, m_pad/16
// subtiles}; one box = KSTG blocks of 8 subtiles (a 128-row tile), no swizzle.
bool make_w_map(CUtensorMap* map, const WeightView& W, int KSTG) {
  const int KB = W.in_dim / kBK;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kSubtileBytes / 4),
                              static_cast<cuuint64_t>(KB),
                              static_cast<cuuint64_t>(W.m_pad / kSubRows)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kSubtileBytes),
                                 static_cast<cuuint64_t>(KB) * kSubtileBytes};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kSubtileBytes / 4),
                             static_cast<cuuint32_t>(KSTG),
                             static_cast<cuuint32_t>(kBM / kSubRows)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(W.w), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// First tile of the paired GEMM that runs as two half-width units (tiles when
// none does), for `pairs` co-resident pairs: every tile when all the halves fit
// in one wave, else the last partial wave when its halves fit in one; not when
// the last token tile's second half would be empty. OBN_GEMM_HALVES=0 disables.
int pair_split_from(int tiles, int pairs, int n, int bn) {
  static const bool on = [] {
    const char* e = std::getenv("OBN_GEMM_HALVES");
    return !(e && e[0] == '0');
  }();
  if (!on || pairs <= 0) return tiles;
  const int tail = n % bn;
  if (tail != 0 && tail <= bn / 2) return tiles;
  if (2 * tiles <= pairs) return 0;
  if (tiles <= pairs) return tiles;
  const int rem = tiles % pairs;
  return rem > 0 && 2 * rem <= pairs ? tiles - rem : tiles;
}

template <int BN, int STAGES, int KSTG, bool A_TMEM, int OUT = kOutLocal, bool PAIR = false>
cudaError_t gemm_bn(const WeightView& W, const int8_t* q, const float* s_x, const int32_t* qsum,
                    int n, float* y, int32_t* acc, int order, cudaStream_t s,
                    const GatherOut& go = GatherOut{}) {
  if (!encode_fn()) return cudaErrorNotSupported;
  CUtensorMap qmap, qhmap, wmap;
  if (!make_q_map(&qmap, q, n, W.in_dim, PAIR ? BN / 2 : BN, KSTG) || !make_w_map(&wmap, W, KSTG))
    return cudaErrorInvalidValue;
  if (PAIR && !make_q_map(&qhmap, q, n, W.in_dim, BN / 4, KSTG)) return cudaErrorInvalidValue;
  if (!PAIR) qhmap = qmap;
  const size_t smem = gemm_smem_bytes<BN, STAGES, KSTG, A_TMEM, OUT, PAIR>();
  auto kern = k_gemm<BN, STAGES, KSTG, A_TMEM, OUT, PAIR>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  const int rows = PAIR ? 2 * kBM : kBM;
  const int tiles = ((W.out_dim + rows - 1) / rows) * ((n + BN - 1) / BN);
  // PAIR: clusters of 2 CTAs, one pair per unit (an even grid)
  const int cap = PAIR ? (num_sms() & ~1) : num_sms();
  const int split_from = PAIR ? pair_split_from(tiles, cap / 2, n, BN) : tiles;
  const int units = 2 * tiles - split_from;
  const int grid = (PAIR ? 2 * units : units) < cap ? (PAIR ? 2 * units : units) : cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = PAIR ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, qmap, qhmap, wmap, W.s_w, s_x, qsum, y, acc, W.out_dim,
                            n, W.in_dim, order, split_from, go);
}

template <int BN>
cudaError_t gemm_sk(const WeightView& W, const int8_t* q, const float* s_x, const int32_t* qsum,
                    int n, float* y, int32_t* acc, int order, int S, cudaStream_t s) {
  CUtensorMap qmap, wmap;
  if (!make_q_map(&qmap, q, n, W.in_dim, BN, 1) || !make_w_map(&wmap, W, 1))
    return cudaErrorInvalidValue;
  const size_t smem = sk_smem_launch<BN>();
  auto kern = k_gemm_sk<BN>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  const int num_m = (W.out_dim + kBM - 1) / kBM;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, num_m);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = S;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, qmap, wmap, W.s_w, s_x, qsum, y, acc, W.out_dim, n,
                            W.in_dim, order);
}

// Clusters of S CTAs of k_gemm_sk<BN> that fit on the device at once (cached per
// device and S). Clusters must sit inside one GPC, so this falls off faster than
// num_sms / S (B200: 74 for S = 2, 33 for 4, 22 for 6, 15 for 8).
template <int BN>
int sk_max_clusters(int S) {
  static int cache[64][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || S < 2 || S > 8) return 0;
  if (cache[dev][S]) return cache[dev][S] > 0 ? cache[dev][S] : 0;
  auto kern = k_gemm_sk<BN>;
  const size_t smem = sk_smem_launch<BN>();
  int count = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&count, kern, &cfg) != cudaSuccess) count = 0;
  }
  cudaGetLastError();  // a refused query only disables split-K
  cache[dev][S] = count > 0 ? count : -1;
  return count;
}

// Upper bound on the CTAs of one split-K launch; OBN_GEMM_SPLIT_K=<n> overrides
// it (0 disables split-K). Read once per process.
int split_k_cta_cap() {
  static const int cap = [] {
    const char* e = std::getenv("OBN_GEMM_SPLIT_K");
    return e ? std::atoi(e) : kSplitKDefaultCtas;
  }();
  return cap;
}

// Cluster size for split-K: the largest S <= 8 whose K slices fit one CTA
// (<= sk_blocks<BN>() blocks) and for which one cluster per 128-row tile fits on
// the device in a single wave within the CTA cap; 1 (no split) otherwise.
template <int BN>
int split_k_factor(const WeightView& W) {
  const int num_m = (W.out_dim + kBM - 1) / kBM;
  const int cap = split_k_cta_cap();
  const int KB = W.in_dim / kBK;
  for (int S = KB < 8 ? KB : 8; S >= 2; --S) {
    if ((KB + S - 1) / S > sk_blocks<BN>()) break;  // a smaller S only lengthens the slices
    if (S * num_m <= cap && num_m <= sk_max_clusters<BN>(S)) return S;
  }
  return 1;
}

}  // namespace

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool gemm_supported(const WeightView& W, int n) {
  if (W.in_dim % kBK != 0 || W.m_pad % kBM != 0 || encode_fn() == nullptr) return false;
  // From 4 tokens the tensor cores beat the dp4a GEMV when they get most SMs:
  // through split-K on layers with few row tiles, or directly on layers with
  // more row tiles than half the SMs (measured on B200).
  if (n >= kGemmMinTokens) return true;
  if (n < kGemmMinSplitTokens) return false;
  return split_k_factor<16>(W) > 1 || 2 * (W.m_pad / kBM) > num_sms();
}

// The paired (cta_group::2) tiles for many tokens; OBN_GEMM_PAIR=0 turns them
// off (read once per process).
constexpr int kPairMinTokens = 512;
bool pair_tiles_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("OBN_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

cudaError_t launch_gemm(const WeightView& W, const int8_t* q, const float* s_x,
                        const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                        cudaStream_t s) {
  // Few 128-row tiles: split K over a cluster per tile.
  int S = 1;
  if (n <= 16 && (S = split_k_factor<16>(W)) > 1)
    return gemm_sk<16>(W, q, s_x, qsum, n, y, acc, order, S, s);
  if (n > 16 && n <= 32 && (S = split_k_factor<32>(W)) > 1)
    return gemm_sk<32>(W, q, s_x, qsum, n, y, acc, order, S, s);
  if (n > 32 && n <= 64 && (S = split_k_factor<64>(W)) > 1)
    return gemm_sk<64>(W, q, s_x, qsum, n, y, acc, order, S, s);
  if (n > 64 && n <= 128 && (S = split_k_factor<128>(W)) > 1)
    return gemm_sk<128>(W, q, s_x, qsum, n, y, acc, order, S, s);
  // Small token tiles: 4-block stages (16 MMAs per commit) amortise the commit cost.
  if (n <= 16) return gemm_bn<16, 3, 4, true>(W, q, s_x, qsum, n, y, acc, order, s);
  if (n <= 32) return gemm_bn<32, 3, 4, true>(W, q, s_x, qsum, n, y, acc, order, s);
  if (n <= 64) return gemm_bn<64, 3, 4, true>(W, q, s_x, qsum, n, y, acc, order, s);
  if (n <= 128) return gemm_bn<128, 4, 2, true>(W, q, s_x, qsum, n, y, acc, order, s);
  // From 512 tokens: 256-row tiles on CTA pairs (cta_group::2), each CTA loading
  // half of the token tile; below, the single-CTA 256-token tile.
  if (n >= kPairMinTokens && pair_tiles_enabled())
    return gemm_bn<256, 6, 1, false, kOutLocal, true>(W, q, s_x, qsum, n, y, acc, order, s);
  return gemm_bn<256, 4, 1, false>(W, q, s_x, qsum, n, y, acc, order, s);
}

cudaError_t launch_gemm_gather(const WeightView& W, const int8_t* q, const float* s_x,
                               const int32_t* qsum, int n, int order, const GatherOut& go,
                               cudaStream_t s) {
  if (go.world < 1 || go.world > kMaxGatherRanks) return cudaErrorInvalidValue;
  if (go.mc) {
    if (n <= 128) return gemm_bn<128, 4, 2, true, kOutMulticast>(W, q, s_x, qsum, n, nullptr, nullptr, order, s, go);
    return gemm_bn<256, 4, 1, false, kOutMulticast>(W, q, s_x, qsum, n, nullptr, nullptr, order, s, go);
  }
  if (n <= 128) return gemm_bn<128, 4, 2, true, kOutPeers>(W, q, s_x, qsum, n, nullptr, nullptr, order, s, go);
  return gemm_bn<256, 4, 1, false, kOutPeers>(W, q, s_x, qsum, n, nullptr, nullptr, order, s, go);
}

cudaError_t read_and_clear_dev_error_gemm(uint32_t* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_dev_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(uint32_t));
}

}  // namespace obn
