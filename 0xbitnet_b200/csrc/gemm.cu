// gemm.cu — ternary GEMM on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// Out[n, m] = f32(sum_k w[m,k] q[n,k]) * scales, for n < N tokens, m < M rows.
//
// Swap-AB formulation: the MMA's M dimension is 128 weight rows, its N
// dimension BN tokens, so D[m, n] lives in TMEM with one weight row per lane and
// the epilogue's stores of Out[n, m] are 128-byte coalesced runs over m.
//
// Per 128-element K block (one I2_S block) a pipeline stage holds:
//   P: the 128 rows' packed 2-bit weights, 4 KB, one contiguous bulk copy
//      (T256 layout: a half panel of one block is contiguous);
//   B: BN tokens x 128 int8 activations, TMA 2D tile, 128-byte swizzle;
//   A: P expanded to unsigned 8-bit codes c = w + 1 in the UMMA K-major
//      128-byte-swizzle layout (row r at (r/8)*1024 + (r%8)*128, 16-byte chunk
//      j stored at chunk j ^ (r%8)).
// The MMA accumulates sum_k c q = sum_k w q + sum_k q; the epilogue subtracts
// the per-token code sum qsum[n] (exact, integer).
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
#include <cuda.h>

#include "gemm.h"
#include "layout.cuh"
#include "obn_common.cuh"

namespace obn {
namespace {

constexpr int kBM = 128;           // weight rows per tile (MMA M)
constexpr int kBK = 128;           // K elements per stage (one I2_S block)
constexpr int kThreads = 384;
constexpr int kPackedStage = kBM * 32;  // 4096 bytes of packed weights per stage

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

// ---- tcgen05 wrappers --------------------------------------------------------
OBN_DEVINL void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
OBN_DEVINL void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
OBN_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
OBN_DEVINL void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
OBN_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

OBN_DEVINL void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
OBN_DEVINL void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

OBN_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
OBN_DEVINL void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 2D tiled TMA load (no multicast) completing on `bar`.
OBN_DEVINL void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes stacked contiguously (SBO = 1024), Blackwell version 1.
OBN_DEVINL uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                    // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;            // SBO
  d |= static_cast<uint64_t>(1u) << 46;                    // version
  d |= static_cast<uint64_t>(2u) << 61;                    // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D s32, A u8 (codes), B s8 (activations), both
// K-major, N = BN, M = 128.
template <int BN>
constexpr uint32_t idesc_i8() {
  return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

// Bounded wait that gives up at once after another role aborted.
OBN_DEVINL bool wait_or_abort(GemmSmem* sm, uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && sm->abort_flag) return false;
  }
  record_error(DEVERR_MBAR_TIMEOUT);
  sm->abort_flag = 1;
  return false;
}

template <int BN, int STAGES>
__global__ __launch_bounds__(kThreads, 1) void k_gemm(const __grid_constant__ CUtensorMap tmap_q,
                                                      const uint8_t* __restrict__ W,
                                                      const float* __restrict__ s_w,
                                                      const float* __restrict__ s_x,
                                                      const int32_t* __restrict__ qsum,
                                                      float* __restrict__ y,
                                                      int32_t* __restrict__ acc_out, int M, int N,
                                                      int K, int order) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = base;                                   // STAGES x 16 KB
  uint8_t* sB = sA + STAGES * kBM * kBK;                // STAGES x BN*128
  uint8_t* sP = sB + STAGES * BN * kBK;                 // STAGES x 4 KB
  GemmSmem* sm = reinterpret_cast<GemmSmem*>(sP + STAGES * kPackedStage);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB = K / kBK;
  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  constexpr uint32_t kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm->full_tma[s], 1);
      mbar_init(&sm->full_a[s], 128);
      mbar_init(&sm->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm->accf[a], 1);
      mbar_init(&sm->acce[a], 128);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
      const uint64_t pol = policy_evict_last();  // weights are re-read by every token tile
      int it = 0;
      bool waited = false;
      for (int t = blockIdx.x; t < tiles && !sm->abort_flag; t += gridDim.x) {
        const int mt = t % num_m, nt = t / num_m;
        const uint8_t* wsrc = W + (static_cast<size_t>(mt >> 1) * KB * 16 + (mt & 1) * 8) *
                                      kSubtileBytes;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!wait_or_abort(sm, &sm->empty[s], ph ^ 1u)) break;
          mbar_arrive_expect_tx(&sm->full_tma[s], BN * kBK + kPackedStage);
          bulk_g2s_hint(sP + s * kPackedStage, wsrc + static_cast<size_t>(kb) * 16 * kSubtileBytes,
                        kPackedStage, &sm->full_tma[s], pol);
          if (!waited) {  // q comes from the previous kernel; the weights do not
            pdl_wait();
            waited = true;
          }
          tma_load_2d(sB + s * BN * kBK, &tmap_q, kb * kBK, nt * BN, &sm->full_tma[s]);
        }
      }
      if (!waited) pdl_wait();
      // Drain: wait (bounded) for every copy this thread issued before exiting.
      const int last = it;
      for (int j = (last > STAGES ? last - STAGES : 0); j < last; ++j)
        mbar_wait(&sm->full_tma[j % STAGES], (j / STAGES) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    pdl_wait();
    if (lane == 0) {
      int it = 0, ti = 0;
      constexpr uint32_t idesc = idesc_i8<BN>();
      for (int t = blockIdx.x; t < tiles && !sm->abort_flag; t += gridDim.x, ++ti) {
        const int a = ti & 1;
        const uint32_t aph = (ti >> 1) & 1u;
        if (!wait_or_abort(sm, &sm->acce[a], aph ^ 1u)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + a * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!wait_or_abort(sm, &sm->full_tma[s], ph) || !wait_or_abort(sm, &sm->full_a[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * kBM * kBK);
          const uint32_t b_addr = smem_u32(sB + s * BN * kBK);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            mma_i8(d_tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc,
                   (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&sm->empty[s]);
        }
        if (!ok) break;
        mma_commit(&sm->accf[a]);
      }
      // Every MMA issued by this thread must finish before TMEM is released.
      mma_commit(&sm->drain);
      mbar_wait(&sm->drain, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ expansion
    pdl_wait();
    const int r = tid - 128;  // weight row within the tile
    const int sub = r >> 4, rr = r & 15;
    const uint32_t swz = static_cast<uint32_t>(r & 7);
    int it = 0;
    for (int t = blockIdx.x; t < tiles && !sm->abort_flag; t += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        if (!wait_or_abort(sm, &sm->full_tma[s], ph)) {
          ok = false;
          break;
        }
        const uint8_t* p = sP + s * kPackedStage + sub * kSubtileBytes + rr * 16;
        uint8_t* arow = sA + s * kBM * kBK + (r >> 3) * 1024 + (r & 7) * 128;
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
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        mbar_arrive(&sm->full_a[s]);
      }
      if (!ok) break;
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int ti = 0;
    for (int t = blockIdx.x; t < tiles && !sm->abort_flag; t += gridDim.x, ++ti) {
      const int mt = t % num_m, nt = t / num_m;
      const int a = ti & 1;
      const uint32_t aph = (ti >> 1) & 1u;
      if (!wait_or_abort(sm, &sm->accf[a], aph)) break;
      tc_fence_after();
      const int m = mt * kBM + quarter * 32 + lane;
      const float sw = (m < M && !acc_out) ? s_w[m] : 0.0f;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + a * BN;
#pragma unroll 1
      for (int j0 = 0; j0 < BN; j0 += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + j0, v);
        tmem_ld_wait();
        const int n0 = nt * BN + j0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = n0 + j;
          if (n < N && m < M) {
            const int d = static_cast<int>(v[j]) - qsum[n];
            const size_t o = static_cast<size_t>(n) * M + m;
            if (acc_out) {
              acc_out[o] = d;
            } else {
              const float fd = static_cast<float>(d);
              const float sx = s_x[n];
              y[o] = order == kOrderGemv ? __fmul_rn(__fmul_rn(fd, sw), sx)
                                         : __fmul_rn(fd, __fmul_rn(sw, sx));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sm->acce[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}

// ---- host side ------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

template <int BN, int STAGES>
size_t gemm_smem_bytes() {
  return 1024 + static_cast<size_t>(STAGES) * (kBM * kBK + BN * kBK + kPackedStage) +
         sizeof(GemmSmem);
}

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] ? sms[dev] : 148;
}

template <int BN, int STAGES>
cudaError_t gemm_bn(const WeightView& W, const int8_t* q, const float* s_x, const int32_t* qsum,
                    int n, float* y, int32_t* acc, int order, cudaStream_t s) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(W.in_dim), static_cast<cuuint64_t>(n)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(W.in_dim)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(BN)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const size_t smem = gemm_smem_bytes<BN, STAGES>();
  auto kern = k_gemm<BN, STAGES>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  const int tiles = ((W.out_dim + kBM - 1) / kBM) * ((n + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, map, W.w, W.s_w, s_x, qsum, y, acc, W.out_dim, n,
                            W.in_dim, order);
}

}  // namespace

bool gemm_supported(const WeightView& W, int n) {
  return n >= kGemmMinTokens && W.in_dim % kBK == 0 && encode_fn() != nullptr;
}

cudaError_t launch_gemm(const WeightView& W, const int8_t* q, const float* s_x,
                        const int32_t* qsum, int n, float* y, int32_t* acc, int order,
                        cudaStream_t s) {
  if (n <= 32) return gemm_bn<32, 8>(W, q, s_x, qsum, n, y, acc, order, s);
  if (n <= 64) return gemm_bn<64, 6>(W, q, s_x, qsum, n, y, acc, order, s);
  if (n <= 128) return gemm_bn<128, 5>(W, q, s_x, qsum, n, y, acc, order, s);
  return gemm_bn<256, 4>(W, q, s_x, qsum, n, y, acc, order, s);
}

cudaError_t read_and_clear_dev_error_gemm(uint32_t* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_dev_error, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  const uint32_t zero = 0;
  return cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(uint32_t));
}

}  // namespace obn
