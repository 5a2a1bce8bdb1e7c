// mma_rate.cu — measurement of the integer multiply-accumulate rates that decide
// which kernel serves which batch size (no counterpart in the reference).
//
// One CTA per SM issues a burst of back-to-back operations and times it with
// clock64; the slowest SM's count is reported as MACs per cycle per SM:
//   form 0: tcgen05.mma.cta_group::1.kind::i8, M = 128, K = 32, A in TMEM,
//           B in shared memory (128-byte swizzle), N = n, one commit at the end;
//   form 1: the same with A in shared memory;
//   form 2: mma.sync.aligned.m16n8k32.s32.u8.s8 (4 independent chains per warp,
//           4 warps per SM);
//   form 3: dp4a.u32.s32 (8 independent chains per thread, 256 threads per SM).
// Operand values are arbitrary (the rate does not depend on them); every wait is
// bounded and TMEM is released before exit.
#include <cuda.h>

#include "../../include/obn.h"
#include "tc05.cuh"

namespace obn {
int report_error(int code, const char* message);
}  // namespace obn

namespace {
using namespace obn;

__global__ __launch_bounds__(128, 1) void k_rate_tc05(int n, int nmma, int ss, long long* out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sB = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  uint8_t* sA = sB + 256 * 128;
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int i = tid; i < (256 + 128) * 128 / 4; i += 128)
    reinterpret_cast<uint32_t*>(sB)[i] = 0x01010101u * (i & 3);
  if (tid == 0) {
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tbase, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;
  {
    uint32_t v[32];
    for (int j = 0; j < 32; ++j) v[j] = 0x01010101u;
    tmem_st32(tmem + (static_cast<uint32_t>(warp * 32) << 16), v);  // A codes, columns 0..31
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  long long cycles = 0;
  if (tid == 0) {
    const uint32_t idesc = (2u << 4) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
                           (static_cast<uint32_t>(128 >> 4) << 24);
    const uint64_t b0 = sw128_desc(smem_u32(sB)), a0 = sw128_desc(smem_u32(sA));
    const long long t0 = clock64();
    for (int i = 0; i < nmma; ++i) {
      const int kk = i & 3;
      if (ss)
        mma_i8(tmem + 32, a0 + static_cast<uint64_t>((kk * 32) >> 4),
               b0 + static_cast<uint64_t>((kk * 32) >> 4), idesc, i > 0 ? 1u : 0u);
      else
        mma_i8_ts(tmem + 32, tmem + kk * 8, b0 + static_cast<uint64_t>((kk * 32) >> 4), idesc,
                  i > 0 ? 1u : 0u);
    }
    mma_commit(&done);
    const bool ok = mbar_wait(&done, 0);
    cycles = ok ? clock64() - t0 : -1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
  if (tid == 0) out[blockIdx.x] = cycles;
}

__global__ void k_rate_imma(int iters, int* sink, long long* out) {
  uint32_t a0 = threadIdx.x, a1 = a0 * 3, a2 = a0 * 5, a3 = a0 * 7, b0 = a0 ^ 0x55u, b1 = a0 ^ 0x33u;
  int c[4][4] = {};
  const long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      asm volatile(
          "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
          "{%8,%9}, {%0,%1,%2,%3};"
          : "+r"(c[k][0]), "+r"(c[k][1]), "+r"(c[k][2]), "+r"(c[k][3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  const long long t1 = clock64();
  int s = 0;
  for (int k = 0; k < 4; ++k)
    for (int j = 0; j < 4; ++j) s += c[k][j];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) out[blockIdx.x] = t1 - t0;
}

__global__ void k_rate_dp4a(int iters, int* sink, long long* out) {
  const uint32_t a = threadIdx.x, b = a * 7;
  int c[8] = {};
  const long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      asm volatile("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(c[k]) : "r"(a + k), "r"(b));
  }
  const long long t1 = clock64();
  int s = 0;
  for (int k = 0; k < 8; ++k) s += c[k];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) out[blockIdx.x] = t1 - t0;
}

}  // namespace

extern "C" int obn_measure_mma_rate(int form, int n, int count, double* macs_per_cycle_per_sm) {
  if (!macs_per_cycle_per_sm || form < 0 || form > 3 || count < 1 || count > (1 << 16))
    return obn::report_error(OBN_ERR_INVALID_ARGUMENT, "obn_measure_mma_rate: bad argument");
  if (form <= 1 && (n < 8 || n > 256 || n % 8 != 0))
    return obn::report_error(OBN_ERR_INVALID_ARGUMENT,
                             "obn_measure_mma_rate: tcgen05 N must be a multiple of 8 in 8..256");
  int sms = 0, dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return obn::report_error(OBN_ERR_CUDA, "obn_measure_mma_rate: no device");
  long long* cyc = nullptr;
  int* sink = nullptr;
  e = cudaMalloc(&cyc, sizeof(long long) * sms);
  if (e == cudaSuccess) e = cudaMalloc(&sink, sizeof(int) * sms * 256);
  double macs = 0.0;
  if (e == cudaSuccess) {
    if (form <= 1) {
      const int smem = 60 * 1024;
      e = cudaFuncSetAttribute(k_rate_tc05, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e == cudaSuccess) {
        k_rate_tc05<<<sms, 128, smem>>>(n, count, form, cyc);
        e = cudaGetLastError();
      }
      macs = 128.0 * n * 32 * count;
    } else if (form == 2) {
      k_rate_imma<<<sms, 128>>>(count, sink, cyc);
      e = cudaGetLastError();
      macs = 4.0 * 4 * 16 * 8 * 32 * count;  // 4 warps x 4 chains x m16n8k32
    } else {
      k_rate_dp4a<<<sms, 256>>>(count, sink, cyc);
      e = cudaGetLastError();
      macs = 256.0 * 8 * 4 * count;
    }
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  long long worst = 0;
  bool timed_out = false;
  if (e == cudaSuccess) {
    long long* h = new long long[sms];
    e = cudaMemcpy(h, cyc, sizeof(long long) * sms, cudaMemcpyDeviceToHost);
    for (int i = 0; e == cudaSuccess && i < sms; ++i) {
      if (h[i] < 0) timed_out = true;
      else if (h[i] > worst) worst = h[i];
    }
    delete[] h;
  }
  cudaFree(cyc);
  cudaFree(sink);
  if (e != cudaSuccess) return obn::report_error(OBN_ERR_CUDA, cudaGetErrorString(e));
  if (timed_out || worst <= 0)
    return obn::report_error(OBN_ERR_DEVICE_TIMEOUT, "obn_measure_mma_rate: a bounded wait gave up");
  *macs_per_cycle_per_sm = macs / static_cast<double>(worst);
  return OBN_OK;
}
