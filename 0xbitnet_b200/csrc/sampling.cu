// sampling.cu — the device half of next-token sampling: repetition penalty,
// temperature and the top-k cut of sampling.rs:14-60 over the logits where the
// LM head left them, so only the k survivors (not the 128256 logits) cross to
// the host, which finishes the softmax draw in the reference's order.
#include "sampling.h"

#include <cstdint>

#include "obn_common.cuh"

namespace obn {
namespace {

constexpr int kSelThreads = 1024;

// Order-preserving key of a float for a descending selection: larger float,
// larger key. -0 is folded onto +0 (they compare equal as floats).
OBN_DEVINL uint32_t sel_key(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u & 0x7FFFFFFFu) == 0) u = 0;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA. (1) Thread 0 applies the penalty to the logits in place, once per
// occurrence in the window, in window order (sampling.rs:14-27). (2) Every
// value is x = logit * (1 / T) when T != 1 (sampling.rs:29-35), or the logit
// itself when T <= 0 (arg-max, k = 1). (3) A 4-pass radix select (8 bits per
// pass, from the top) finds the key of the k-th largest x. (4) Every element
// with x >= that value is written as (index, bits of x), in no particular order;
// *count gets the number of such elements (it may exceed k when values tie,
// and exceed cap, in which case only cap are written).
__global__ __launch_bounds__(kSelThreads) void k_select_topk(
    float* __restrict__ logits, int V, const uint32_t* __restrict__ recent, int n_recent,
    float penalty, float temperature, int k, uint2* __restrict__ out, int cap,
    int* __restrict__ count) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_remaining;
  __shared__ int s_count;
  const int tid = threadIdx.x;
  if (tid == 0) {
    if (penalty != 1.0f) {
      for (int r = 0; r < n_recent; ++r) {
        const uint32_t id = recent[r];
        if (id < static_cast<uint32_t>(V)) {
          const float v = logits[id];
          logits[id] = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
        }
      }
    }
    s_prefix = 0;
    s_mask = 0;
    s_remaining = static_cast<uint32_t>(k);
    s_count = 0;
  }
  __syncthreads();
  const bool greedy = !(temperature > 0.0f);
  const bool scale = !greedy && temperature != 1.0f;
  const float inv_temp = scale ? __fdiv_rn(1.0f, temperature) : 1.0f;
  auto value = [&](int i) {
    const float v = logits[i];
    return scale ? __fmul_rn(v, inv_temp) : v;
  };
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += kSelThreads) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = tid; i < V; i += kSelThreads) {
      const uint32_t key = sel_key(value(i));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t need = s_remaining, cum = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (cum + hist[b] >= need) break;
        cum += hist[b];
      }
      s_remaining = need - cum;
      s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
      s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;  // the key of the k-th largest value
  for (int i = tid; i < V; i += kSelThreads) {
    const float x = value(i);
    if (sel_key(x) >= thr) {
      const int p = atomicAdd(&s_count, 1);
      if (p < cap) out[p] = make_uint2(static_cast<uint32_t>(i), __float_as_uint(x));
    }
  }
  __syncthreads();
  if (tid == 0) *count = s_count;
}

}  // namespace

cudaError_t launch_select_topk(float* logits, int V, const uint32_t* recent, int n_recent,
                               float penalty, float temperature, int k, uint2* out, int cap,
                               int* count, cudaStream_t s) {
  if (V <= 0 || k <= 0 || k > V || cap <= 0) return cudaErrorInvalidValue;
  k_select_topk<<<1, kSelThreads, 0, s>>>(logits, V, recent, n_recent, penalty, temperature, k,
                                           out, cap, count);
  return cudaGetLastError();
}

}  // namespace obn
