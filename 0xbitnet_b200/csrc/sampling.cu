// sampling.cu — the device half of next-token sampling: repetition penalty,
// temperature and the top-k cut of sampling.rs:14-60 over the logits where the
// LM head left them, so only the k survivors (not the 128256 logits) cross to
// the host, which finishes the softmax draw in the reference's order.
//
// Two launches instead of one CTA over the whole vocabulary (4 radix passes of
// 128256 global loads, ~90 us per token):
//  * k_select_slice: CTA s owns a slice of ~1000 logits. Thread 0 applies the
//    penalty to the slice's ids in window order; the slice's keys sit in shared
//    memory for a 4-pass radix select of the slice's k-th largest value, and every
//    element at or above it (the slice's survivors) goes to the candidate buffer.
//    The slice's k-th largest value is at most the vocabulary's, so every final
//    survivor is a candidate.
//  * k_select_final: one CTA selects the vocabulary's k-th largest value among the
//    candidates and writes the survivors in the output format.
#include "sampling.h"

#include <cstdint>

#include "obn_common.cuh"

namespace obn {
namespace {

constexpr int kSliceThreads = 256;
constexpr int kSliceMax = 1024;  // logits per slice (shared-memory keys)
constexpr int kFinalThreads = 1024;

// Order-preserving key of a float for a descending selection: larger float,
// larger key. -0 is folded onto +0 (they compare equal as floats).
OBN_DEVINL uint32_t sel_key(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u & 0x7FFFFFFFu) == 0) u = 0;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Radix select over `n` keys produced by key_at(i): the key of the k-th largest
// (k <= n), 8 bits per pass from the top. hist: 256 shared counters; s: 3 shared
// words. Every thread of the CTA calls it and gets the result.
template <int THREADS, class KeyAt>
OBN_DEVINL uint32_t radix_select(KeyAt key_at, int n, int k, uint32_t* hist, uint32_t* s) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    s[0] = 0;  // prefix
    s[1] = 0;  // mask
    s[2] = static_cast<uint32_t>(k);  // still needed at or above the prefix
  }
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += THREADS) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = s[0], mask = s[1];
    for (int i = tid; i < n; i += THREADS) {
      const uint32_t key = key_at(i);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid < 32) {  // one warp scans the 256 bins from the top, 8 per lane
      const uint32_t need = s[2];
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - (8 * tid + j)];
        tot += c[j];
      }
      uint32_t incl = tot;  // inclusive prefix over lanes (bins from the top)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += v;
      }
      const uint32_t excl = incl - tot;
      const bool here = excl < need && incl >= need;
      if (here) {
        uint32_t cum = excl;
        int j = 0;
        for (; j < 7; ++j) {
          if (cum + c[j] >= need) break;
          cum += c[j];
        }
        const uint32_t b = 255u - static_cast<uint32_t>(8 * tid + j);
        s[2] = need - cum;
        s[0] = prefix | (b << shift);
        s[1] = mask | (255u << shift);
      }
    }
    __syncthreads();
  }
  return s[0];
}

__global__ __launch_bounds__(kSliceThreads) void k_select_slice(
    float* __restrict__ logits, int V, int L, const uint32_t* __restrict__ recent, int n_recent,
    float penalty, float temperature, int k, int capL, uint2* __restrict__ cand,
    int* __restrict__ cand_count) {
  __shared__ uint32_t keys[kSliceMax];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s[3];
  __shared__ int s_count;
  const int tid = threadIdx.x;
  const int i0 = blockIdx.x * L;
  const int n = min(L, V - i0);
  if (tid == 0) {
    // sampling.rs:14-27: once per occurrence in the window, in window order
    if (penalty != 1.0f)
      for (int r = 0; r < n_recent; ++r) {
        const uint32_t id = recent[r];
        if (id >= static_cast<uint32_t>(i0) && id < static_cast<uint32_t>(i0 + n)) {
          const float v = logits[id];
          logits[id] = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
        }
      }
    s_count = 0;
  }
  __syncthreads();
  const bool greedy = !(temperature > 0.0f);
  const bool scale = !greedy && temperature != 1.0f;
  const float inv_temp = scale ? __fdiv_rn(1.0f, temperature) : 1.0f;
  for (int i = tid; i < n; i += kSliceThreads) {
    const float v = logits[i0 + i];
    keys[i] = sel_key(scale ? __fmul_rn(v, inv_temp) : v);
  }
  __syncthreads();
  const int kl = min(k, n);
  const uint32_t thr =
      radix_select<kSliceThreads>([&](int i) { return keys[i]; }, n, kl, hist, s);
  for (int i = tid; i < n; i += kSliceThreads) {
    const uint32_t key = keys[i];
    if (key >= thr) {
      const int p = atomicAdd(&s_count, 1);
      if (p < capL) {
        const float v = logits[i0 + i];
        const float x = scale ? __fmul_rn(v, inv_temp) : v;
        cand[static_cast<size_t>(blockIdx.x) * capL + p] =
            make_uint2(static_cast<uint32_t>(i0 + i), __float_as_uint(x));
      }
    }
  }
  __syncthreads();
  if (tid == 0) cand_count[blockIdx.x] = s_count;  // > capL: too many ties (host path)
}

constexpr int kFinalSmemKeys = 12288;  // candidates gathered into shared memory

__global__ __launch_bounds__(kFinalThreads) void k_select_final(
    const uint2* __restrict__ cand, const int* __restrict__ cand_count, int slices, int capL,
    int k, uint2* __restrict__ out, int cap, int* __restrict__ count) {
  extern __shared__ uint32_t dyn_keys[];  // [kFinalSmemKeys] keys, then their slots
  uint32_t* g_key = dyn_keys;
  uint32_t* g_slot = dyn_keys + kFinalSmemKeys;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s[3];
  __shared__ int s_count, s_over;
  __shared__ int off[kFinalThreads + 1];  // exclusive prefix of the slices' counts
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_count = 0;
    s_over = 0;
  }
  __syncthreads();
  // per thread: a run of consecutive slices; then a block scan of the runs' sums
  const int per = (slices + kFinalThreads - 1) / kFinalThreads;
  int run = 0;
  for (int c = tid * per; c < min(slices, tid * per + per); ++c) {
    const int n = cand_count[c];
    if (n > capL) s_over = 1;
    run += min(n, capL);
  }
  off[tid + 1] = run;
  __syncthreads();
  if (s_over) {  // a slice could not hold its ties: the host samples from the logits
    if (tid == 0) *count = cap + 1;
    return;
  }
  for (int d = 1; d < kFinalThreads; d <<= 1) {  // inclusive scan of off[1..]
    const int v = tid + 1 > d ? off[tid + 1 - d] : 0;
    __syncthreads();
    off[tid + 1] += v;
    __syncthreads();
  }
  if (tid == 0) off[0] = 0;
  __syncthreads();
  const int total_valid = off[kFinalThreads];
  if (total_valid <= kFinalSmemKeys) {
    // gather the valid candidates' keys (and slots) into shared memory
    int o = off[tid];
    for (int c = tid * per; c < min(slices, tid * per + per); ++c) {
      const int n = cand_count[c];
      for (int j = 0; j < n; ++j) {
        const int e = c * capL + j;
        g_key[o + j] = sel_key(__uint_as_float(cand[e].y));
        g_slot[o + j] = static_cast<uint32_t>(e);
      }
      o += n;
    }
    __syncthreads();
    const uint32_t thr =
        radix_select<kFinalThreads>([&](int i) { return g_key[i]; }, total_valid, k, hist, s);
    for (int i = tid; i < total_valid; i += kFinalThreads) {
      if (g_key[i] >= thr) {
        const int p = atomicAdd(&s_count, 1);
        if (p < cap) out[p] = cand[g_slot[i]];
      }
    }
  } else {  // many candidates (large k): select over the slots in global memory
    const int total = slices * capL;
    auto key_at = [&](int e) -> uint32_t {  // empty slots sort below every real key
      const int c = e / capL, j = e - c * capL;
      return j < cand_count[c] ? sel_key(__uint_as_float(cand[e].y)) : 0u;
    };
    const uint32_t thr = radix_select<kFinalThreads>(key_at, total, k, hist, s);
    for (int e = tid; e < total; e += kFinalThreads) {
      const int c = e / capL, j = e - c * capL;
      if (j >= cand_count[c]) continue;
      const uint2 pr = cand[e];
      if (sel_key(__uint_as_float(pr.y)) >= thr) {
        const int p = atomicAdd(&s_count, 1);
        if (p < cap) out[p] = pr;
      }
    }
  }
  __syncthreads();
  if (tid == 0) *count = s_count;
}

}  // namespace

size_t select_topk_scratch_bytes(int V) {
  // candidates (at most one slice's length past V) and the slices' counts
  return (static_cast<size_t>(V) + kSliceMax) * sizeof(uint2) + 4096 * sizeof(int);
}

cudaError_t launch_select_topk(float* logits, int V, const uint32_t* recent, int n_recent,
                               float penalty, float temperature, int k, uint2* out, int cap,
                               int* count, void* scratch, cudaStream_t s) {
  if (V <= 0 || k <= 0 || k > V || cap <= 0 || !scratch) return cudaErrorInvalidValue;
  const int slices = (V + kSliceMax - 1) / kSliceMax;
  if (slices > 4096) return cudaErrorInvalidValue;
  const int L = (V + slices - 1) / slices;  // <= kSliceMax
  // a slice keeps at most all of its logits, so the candidates fit V pairs
  const int capL = min(L, 2 * k + 32);
  uint2* cand = static_cast<uint2*>(scratch);
  int* cand_count = reinterpret_cast<int*>(cand + static_cast<size_t>(slices) * capL);
  k_select_slice<<<slices, kSliceThreads, 0, s>>>(logits, V, L, recent, n_recent, penalty,
                                                  temperature, k, capL, cand, cand_count);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int smem = 2 * kFinalSmemKeys * static_cast<int>(sizeof(uint32_t));
  static bool configured[64] = {};  // the attribute is set per device
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(k_select_final, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  k_select_final<<<1, kFinalThreads, smem, s>>>(cand, cand_count, slices, capL, k, out, cap,
                                                count);
  return cudaGetLastError();
}

}  // namespace obn
