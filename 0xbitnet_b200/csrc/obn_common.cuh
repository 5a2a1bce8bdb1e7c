// obn_common.cuh — shared device helpers for the sm_100a ternary BitLinear kernels.
//
// Inline PTX wrappers for mbarriers, bulk (TMA) copies, programmatic dependent
// launch (PDL) and bounded waits. Every wait in this library is bounded: when
// the bound is hit the kernel records OBN_DEVERR_* in obn_dev_error and moves on
// without touching the data the wait guarded; the host reads the word with
// obn_check_device_errors().
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define OBN_DEVINL __device__ __forceinline__

namespace obn {

// Device-side error word (one per device context): 0 = ok, else the first
// failure code recorded by a bounded wait.
enum : uint32_t {
  DEVERR_NONE = 0,
  DEVERR_MBAR_TIMEOUT = 1,
  DEVERR_BAD_LAUNCH = 2,  // launch geometry outside what the kernel was built for
};
// Internal linkage: every translation unit (built without -rdc) owns its own
// copy and exposes it through a host reader (kernels.h).
static __device__ uint32_t g_dev_error = 0;

// Spin bound for mbarrier waits. try_wait suspends the thread for a
// hardware-chosen interval per attempt, so this bounds the wait at well under
// a second for any sane data movement while still ending a stuck kernel.
constexpr uint32_t kWaitLimit = 1u << 22;

OBN_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

OBN_DEVINL void record_error(uint32_t code) { atomicCAS(&g_dev_error, 0u, code); }

// ---- mbarrier ---------------------------------------------------------------
OBN_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

OBN_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

OBN_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

OBN_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

OBN_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

OBN_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity`. Returns false (and records the error) when
// the bound is reached.
OBN_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  record_error(DEVERR_MBAR_TIMEOUT);
  return false;
}

// ---- bulk copies (non-tensor TMA) -------------------------------------------
// Global -> shared, completion signalled on `bar` as transaction bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.
OBN_DEVINL void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 eviction-priority hint (createpolicy result).
OBN_DEVINL void bulk_g2s_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

OBN_DEVINL uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

OBN_DEVINL uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- programmatic dependent launch ------------------------------------------
// Lets the next kernel in the stream (launched with the PDL attribute) start
// its prologue; it still waits for this grid's completion in pdl_wait().
OBN_DEVINL void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Blocks until every prerequisite grid has completed and its writes are visible.
OBN_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- integer dot product ------------------------------------------------------
// acc + sum_{b<4} a.byte[b] * b.byte[b], a unsigned codes, b signed int8.
OBN_DEVINL int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

OBN_DEVINL uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// ---- reductions ------------------------------------------------------------
// The exact tree of rmsnorm.wgsl:47-55: partial[tid] += partial[tid + stride]
// for stride = 128 .. 1. Strides 128 and 64 go through shared memory, 32 .. 1
// through shuffles (lane l adds lane l + stride: the same pairing).
OBN_DEVINL float tree_sum_256(float v, float* sh) {
  const int tid = threadIdx.x;
  sh[tid] = v;
  __syncthreads();
  if (tid < 128) sh[tid] = __fadd_rn(sh[tid], sh[tid + 128]);
  __syncthreads();
  if (tid < 64) sh[tid] = __fadd_rn(sh[tid], sh[tid + 64]);
  __syncthreads();
  if (tid < 32) {
    float a = __fadd_rn(sh[tid], sh[tid + 32]);
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, s));
    if (tid == 0) sh[0] = a;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}


// activation.wgsl:28-33 for a gated layer's gate value: 0 = ReLU^2 (max(0, x)^2),
// 1 = SiLU (x / (1 + exp(-x))).
OBN_DEVINL float gate_act(int act, float x) {
  if (act == 0) {
    const float r = fmaxf(0.0f, x);
    return __fmul_rn(r, r);
  }
  return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

}  // namespace obn
