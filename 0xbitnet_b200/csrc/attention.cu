// attention.cu — decode attention for the layers around the BitLinear path, sm_100a.
//
// Reference: attention.rs:85-124 (Attention::forward), rope.wgsl, attention.wgsl
// (compute_scores, attn_v) and softmax.wgsl. The reference keeps an f32 KV cache,
// materialises the [H, N, S] score matrix and runs softmax in three passes. Here:
//
//  * k_rope_kv_append: one thread per (token row, head slot, dimension pair)
//    reads the merged QKV projection output, rotates q and k with the
//    shader's formula (theta = pos * base^(-2i/D), x0 c - x1 s, x0 s + x1 c,
//    each product and sum rounded) and writes q (f32) and the k / v of the new
//    tokens into the binary16 caches [B][S_max][Hkv][d] (half the bytes of the
//    reference's f32 cache: the decode step streams the cache).
//  * k_attn_split: one CTA per (128-key chunk, KV head, query row) — the G query
//    heads of a KV group share each K/V chunk load. Thread = key for the scores
//    (the dot over d is sequential in d, as attention.wgsl's, one fused
//    multiply-add per step, then * scale), thread = dimension for P.V
//    (sequential over the chunk's keys, fused multiply-adds); the chunk keeps
//    its own max and sum (online softmax), written as partials.
//  * k_attn_split_tc (the default): the same partials with K.q and P.V on the
//    tensor cores (mma.sync m16n8k16, binary16 operands, f32 accumulation; q
//    and P split into binary16 hi + lo so nothing is lost against f32).
//  * k_attn_combine: per (query row, head) rescales the chunks' partials to the
//    global max and divides by the global sum.
//
// Keys after a query's causal limit (k > q + (S - N), attention.wgsl:53) are
// skipped; the reference's -FLT_MAX scores give them exactly zero weight. The
// softmax is the same function in a different order of operations, so results
// agree with the reference to rounding (tests: relative 1e-4 on the same fp16
// cache contents).
#include "attention.h"
#include "obn_common.cuh"

#include <cfloat>
#include <cstdlib>

namespace obn {

int num_sms_cached();  // kernels.cu

namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxSplits = 4096 / kAttnChunk;  // combine: splits held in registers
constexpr int kKStride = kAttnHeadDim + 8;  // halves per smem K row: 16-byte rows, no conflicts

// rope.wgsl:41-55 for the pair (x0, x1) = dims (2i, 2i + 1) of a head at
// position p: theta = p * base^(-2i/d), then the rotation with products and
// sums rounded as written.
OBN_DEVINL void rope_angle(int i, int d, int p, float theta_base, float* c, float* sn) {
  const float freq_exp = __fdiv_rn(__fmul_rn(-2.0f, static_cast<float>(i)), static_cast<float>(d));
  const float theta = __fmul_rn(static_cast<float>(p), powf(theta_base, freq_exp));
  sincosf(theta, sn, c);
}
OBN_DEVINL void rope_rotate(float x0, float x1, float c, float sn, float* y0, float* y1) {
  *y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
  *y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
}
OBN_DEVINL void rope_pair(float x0, float x1, int i, int d, int p, float theta_base, float* y0,
                          float* y1) {
  float c, sn;
  rope_angle(i, d, p, theta_base, &c, &sn);
  rope_rotate(x0, x1, c, sn, y0, y1);
}

__global__ __launch_bounds__(256) void k_rope_kv_append(const float* __restrict__ qkv, int n,
                                                        int H, int Hkv, int d, int pos,
                                                        const int* __restrict__ pos_dev,
                                                        float theta_base, size_t total,
                                                        float* __restrict__ q_out,
                                                        __half* __restrict__ k_cache,
                                                        __half* __restrict__ v_cache, int S_max) {
  // No early launch of dependents: the cache rows written here are complete
  // before any later kernel starts (the decode pass reads older rows early).
  pdl_wait();
  const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int half = d >> 1;
  const int slots = H + 2 * Hkv;
  const int i = static_cast<int>(idx % half);
  const size_t rest = idx / half;
  const int j = static_cast<int>(rest % slots);  // head slot: q heads, k heads, v heads
  const size_t r = rest / slots;                 // token row b * n + t
  const int t = static_cast<int>(r % n);
  const size_t b = r / n;
  const float* src = qkv + (r * slots + j) * d + 2 * i;
  const float x0 = src[0], x1 = src[1];
  const int p = (pos_dev ? *pos_dev : pos) + t;
  if (p < 0 || p >= S_max) return;  // a device-side position past the cache writes nothing
  if (j >= H + Hkv) {  // v: stored as is
    __half* dst = v_cache + ((b * S_max + p) * Hkv + (j - H - Hkv)) * d + 2 * i;
    *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(x0, x1);
    return;
  }
  float y0, y1;
  rope_pair(x0, x1, i, d, p, theta_base, &y0, &y1);
  if (j < H) {
    float* dst = q_out + (r * H + j) * d + 2 * i;
    dst[0] = y0;
    dst[1] = y1;
  } else {
    __half* dst = k_cache + ((b * S_max + p) * Hkv + (j - H)) * d + 2 * i;
    *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(y0, y1);
  }
}

// The same append, one CTA per token row: the row's d / 2 RoPE angles are
// computed once (rope_angle, as above) and shared by all its q and k heads, so a
// row of H + Hkv rotated heads costs d / 2 pow / sincos calls instead of
// (H + Hkv) d / 2. Same values, same stores.
constexpr int kRopeRowMaxHalf = 256;  // d <= 512

__global__ __launch_bounds__(256) void k_rope_kv_append_row(
    const float* __restrict__ qkv, int n, int H, int Hkv, int d, int pos,
    const int* __restrict__ pos_dev, float theta_base, float* __restrict__ q_out,
    __half* __restrict__ k_cache, __half* __restrict__ v_cache, int S_max) {
  __shared__ float s_c[kRopeRowMaxHalf], s_s[kRopeRowMaxHalf];
  // No early launch of dependents (as k_rope_kv_append).
  pdl_wait();
  const size_t r = blockIdx.x;  // token row b * n + t
  const int t = static_cast<int>(r % n);
  const size_t b = r / n;
  const int half = d >> 1;
  const int slots = H + 2 * Hkv;
  const int p = (pos_dev ? *pos_dev : pos) + t;
  if (p < 0 || p >= S_max) return;  // a device-side position past the cache writes nothing
  for (int i = threadIdx.x; i < half; i += blockDim.x)
    rope_angle(i, d, p, theta_base, &s_c[i], &s_s[i]);
  __syncthreads();
  const float* row = qkv + r * static_cast<size_t>(slots) * d;
  const int items = slots * half;
  // eight of this thread's pairs per pass, their loads issued together
  for (int e0 = threadIdx.x; e0 < items; e0 += 8 * blockDim.x) {
    float2 xv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < items) {
        const int j = e / half, i = e - j * half;
        const float* src = row + static_cast<size_t>(j) * d + 2 * i;
        xv[u] = make_float2(src[0], src[1]);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e >= items) break;
      const int j = e / half, i = e - j * half;  // head slot: q heads, k heads, v heads
      const float x0 = xv[u].x, x1 = xv[u].y;
      if (j >= H + Hkv) {  // v: stored as is
        __half* dst = v_cache + ((b * S_max + p) * Hkv + (j - H - Hkv)) * d + 2 * i;
        *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(x0, x1);
        continue;
      }
      float y0, y1;
      rope_rotate(x0, x1, s_c[i], s_s[i], &y0, &y1);
      if (j < H) {
        float* dst = q_out + (r * H + j) * d + 2 * i;
        dst[0] = y0;
        dst[1] = y1;
      } else {
        __half* dst = k_cache + ((b * S_max + p) * Hkv + (j - H)) * d + 2 * i;
        *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(y0, y1);
      }
    }
  }
}

// 16-byte global -> shared copy that does not hold a register (cp.async, L2 only).
OBN_DEVINL void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
OBN_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// The same with a source size: bytes past src_bytes (all 16 when 0) are zero-filled.
OBN_DEVINL void cp_async16_zfill(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src), "r"(src_bytes)
               : "memory");
}
// Arrives on `bar` (without raising its pending count) once every cp.async this
// thread issued so far has completed.
OBN_DEVINL void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
template <int N>
OBN_DEVINL void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

OBN_DEVINL float warp_max(float v) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
  return v;
}
OBN_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
  return v;
}

// Where a kernel lets its dependents launch. Passes that append to the cache
// (APPENDS) do it only after their own wait: a kernel that is still waiting then
// proves every kernel before the latest appending pass complete, which is what
// lets the clustered decode pass read older cache rows before its wait.
template <bool APPENDS>
OBN_DEVINL void pdl_order() {
  if constexpr (APPENDS) {
    pdl_wait();
    pdl_launch_dependents();
  } else {
    pdl_launch_dependents();
    pdl_wait();
  }
}

// Partials layout (workspace): for row r, head h, split c:
//   acc[((r * H + h) * nsplit + c) * D + dim], then m[...] and l[...] after all acc.
// ROPE (decode, n = 1): q is the merged QKV row instead of rotated q; the CTA
// rotates its group's q heads itself (the same rope_pair as k_rope_kv_append),
// and the CTA whose chunk holds the new position also rotates the new key,
// stores key and value into the caches and places them in its shared tiles
// directly. That removes the separate RoPE launch from every decode step.
template <int G, bool ROPE = false>
__global__ __launch_bounds__(kAttnThreads) void k_attn_split(
    const float* __restrict__ q, const __half* __restrict__ k_cache,
    const __half* __restrict__ v_cache, int n, int H, int Hkv, int S_max, int seq_len,
    const int* __restrict__ pos_dev, float scale, int nsplit, float* __restrict__ part_acc,
    float* __restrict__ part_m, float* __restrict__ part_l, float theta_base) {
  constexpr int D = kAttnHeadDim;
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sK = reinterpret_cast<__half*>(smem);                       // [chunk][kKStride]
  __half* sV = sK + kAttnChunk * kKStride;                            // [chunk][D]
  float* sQ = reinterpret_cast<float*>(sV + kAttnChunk * D);          // [D][G]
  float* sP = sQ + G * D;                                             // [chunk keys][G]
  __shared__ float red[G][kAttnThreads / 32];
  pdl_order<ROPE>();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x, kvh = blockIdx.y;
  const size_t r = blockIdx.z;  // query row b * n + t
  const int t = static_cast<int>(r % n);
  const size_t b = r / n;
  const int s0 = c * kAttnChunk;
  if (pos_dev) {  // the position lives on the device (graph replay)
    seq_len = min(*pos_dev + n, S_max);
    if (s0 >= seq_len) return;  // past every query's keys: the combine skips this split
  }
  const int limit = seq_len - n + t + 1;  // keys [0, limit) are visible to this query
  const int cnt = min(kAttnChunk, limit - s0);  // may be <= 0: an empty chunk
  const size_t pbase = (r * H + static_cast<size_t>(kvh) * G) * nsplit + c;
  if (cnt <= 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      part_acc[(pbase + static_cast<size_t>(g) * nsplit) * D + tid] = 0.0f;
      if (tid == 0) {
        part_m[pbase + static_cast<size_t>(g) * nsplit] = -FLT_MAX;
        part_l[pbase + static_cast<size_t>(g) * nsplit] = 0.0f;
      }
    }
    return;
  }
  // q rows of the group's heads, and the chunk's K and V rows (16-byte loads).
  // ROPE: the new token's position (n = 1); one past the cache appends nothing
  const int p_new = ROPE ? (pos_dev ? *pos_dev : seq_len - 1) : 0;
  const int new_row =
      (ROPE && p_new < S_max && p_new >= s0 && p_new < s0 + kAttnChunk) ? p_new - s0 : -1;
  if constexpr (ROPE) {
    const int slots = H + 2 * Hkv;
    const float* qrow = q + r * static_cast<size_t>(slots) * D;
    for (int e = tid; e < G * (D / 2); e += kAttnThreads) {
      const int g = e / (D / 2), i = e % (D / 2);
      const float* src = qrow + (static_cast<size_t>(kvh) * G + g) * D + 2 * i;
      float y0, y1;
      rope_pair(src[0], src[1], i, D, p_new, theta_base, &y0, &y1);
      sQ[(2 * i) * G + g] = y0;
      sQ[(2 * i + 1) * G + g] = y1;
    }
    if (new_row >= 0) {  // append the new key (rotated) and value, keep them in the tiles
      __half* kc = const_cast<__half*>(k_cache);
      __half* vc = const_cast<__half*>(v_cache);
      const size_t cache_off = ((b * S_max + p_new) * Hkv + kvh) * D;
      if (tid < D / 2) {
        const float* src = qrow + (static_cast<size_t>(H) + kvh) * D + 2 * tid;
        float y0, y1;
        rope_pair(src[0], src[1], tid, D, p_new, theta_base, &y0, &y1);
        const __half2 h = __floats2half2_rn(y0, y1);
        *reinterpret_cast<__half2*>(kc + cache_off + 2 * tid) = h;
        *reinterpret_cast<__half2*>(sK + new_row * kKStride + 2 * tid) = h;
      } else {
        const int i = tid - D / 2;
        const float* src = qrow + (static_cast<size_t>(H) + Hkv + kvh) * D + 2 * i;
        const __half2 h = __floats2half2_rn(src[0], src[1]);
        *reinterpret_cast<__half2*>(vc + cache_off + 2 * i) = h;
        *reinterpret_cast<__half2*>(sV + new_row * D + 2 * i) = h;
      }
    }
  } else {
    for (int e = tid; e < G * D; e += kAttnThreads) {  // e = g * D + dim -> sQ[dim][g]
      const int g = e / D, dim = e % D;
      sQ[dim * G + g] = q[(r * H + static_cast<size_t>(kvh) * G) * D + e];
    }
  }
  // Asynchronous 16-byte copies (no register held): K in one group, V in a second
  // one that lands while the scores are computed.
#pragma unroll 4
  for (int e = tid; e < kAttnChunk * (D / 8); e += kAttnThreads) {
    const int key = e / (D / 8), part = e % (D / 8);
    __half* dk = sK + key * kKStride + part * 8;
    if (key == new_row) continue;  // ROPE: written above
    if (key < cnt)
      cp_async16(dk, k_cache + ((b * S_max + s0 + key) * Hkv + kvh) * D + part * 8);
    else
      *reinterpret_cast<uint4*>(dk) = make_uint4(0u, 0u, 0u, 0u);
  }
  cp_async_commit();
#pragma unroll 4
  for (int e = tid; e < kAttnChunk * (D / 8); e += kAttnThreads) {
    const int key = e / (D / 8), part = e % (D / 8);
    __half* dv = sV + key * D + part * 8;
    if (key == new_row) continue;
    if (key < cnt)
      cp_async16(dv, v_cache + ((b * S_max + s0 + key) * Hkv + kvh) * D + part * 8);
    else
      *reinterpret_cast<uint4*>(dv) = make_uint4(0u, 0u, 0u, 0u);
  }
  cp_async_commit();
  cp_async_wait_group<1>();  // K landed (V may still be in flight)
  __syncthreads();
  // Scores: thread = key, the dot sequential over d (attention.wgsl:48-51), each
  // step one fused multiply-add (the shader's q * k + sum, contracted).
  static_assert(kAttnThreads == kAttnChunk, "one thread per key");
  float sc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) sc[g] = 0.0f;
  const __half* krow = sK + tid * kKStride;
  // q of dims d and d + 1 for every head: G floats each, read as one broadcast
  // (16-byte words for G >= 4).
  auto qload = [&](int dim, float (&qv)[G]) {
    if constexpr (G % 4 == 0) {
#pragma unroll
      for (int g4 = 0; g4 < G; g4 += 4) {
        const float4 t = *reinterpret_cast<const float4*>(sQ + dim * G + g4);
        qv[g4] = t.x;
        qv[g4 + 1] = t.y;
        qv[g4 + 2] = t.z;
        qv[g4 + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) qv[g] = sQ[dim * G + g];
    }
  };
#pragma unroll 4
  for (int d8 = 0; d8 < D; d8 += 8) {
    const uint4 w = *reinterpret_cast<const uint4*>(krow + d8);
    const __half2* h2 = reinterpret_cast<const __half2*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 kf = __half22float2(h2[e]);
      float q0[G], q1[G];
      qload(d8 + 2 * e, q0);
      qload(d8 + 2 * e + 1, q1);
#pragma unroll
      for (int g = 0; g < G; ++g) {  // fused multiply-adds, in the shader's order over d
        sc[g] = fmaf(q0[g], kf.x, sc[g]);
        sc[g] = fmaf(q1[g], kf.y, sc[g]);
      }
    }
  }
  const bool valid = tid < cnt;
  float mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    sc[g] = valid ? __fmul_rn(sc[g], scale) : -FLT_MAX;
    const float wm = warp_max(sc[g]);
    if (lane == 0) red[g][warp] = wm;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    mg[g] = fmaxf(fmaxf(red[g][0], red[g][1]), fmaxf(red[g][2], red[g][3]));
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float p = valid ? expf(sc[g] - mg[g]) : 0.0f;
    sP[tid * G + g] = p;
    const float ws = warp_sum(p);
    if (lane == 0) red[g][warp] = ws;
  }
  __syncthreads();
  cp_async_wait_group<0>();  // V landed
  __syncthreads();
  // P.V: thread = dimension, sequential over the chunk's keys.
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.0f;
  for (int key = 0; key < cnt; ++key) {
    const float v = __half2float(sV[key * D + tid]);
    float pk[G];
    if constexpr (G % 4 == 0) {
#pragma unroll
      for (int g4 = 0; g4 < G; g4 += 4) {
        const float4 t = *reinterpret_cast<const float4*>(sP + key * G + g4);
        pk[g4] = t.x;
        pk[g4 + 1] = t.y;
        pk[g4 + 2] = t.z;
        pk[g4 + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) pk[g] = sP[key * G + g];
    }
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = fmaf(pk[g], v, acc[g]);
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const size_t pi = pbase + static_cast<size_t>(g) * nsplit;
    part_acc[pi * D + tid] = acc[g];
    if (tid == 0) {
      part_m[pi] = mg[g];
      part_l[pi] = (red[g][0] + red[g][1]) + (red[g][2] + red[g][3]);
    }
  }
}

// ---- tensor-core split pass ------------------------------------------------
// The same partials as k_attn_split, with the two contractions on the tensor
// cores (mma.sync m16n8k16, f16 x f16 -> f32): scores S[key][head] = K . q over
// the chunk's 128 keys and P.V out[dim][head] = sum over keys of V[key][dim] P.
// K and V are binary16 already (exact as MMA operands); q and P are f32, so each
// is split into a binary16 high part and the binary16 rounding of the remainder
// and both halves are multiplied (x = hi + lo to about 2^-22 |x|), which keeps
// the contractions at f32 accuracy. The G query heads of the KV group are the
// MMA's N = 8 columns (zero-padded above G). 4 warps: warp w takes keys
// 32w .. 32w + 31 for the scores and dimensions 32w .. 32w + 31 for P.V.
OBN_DEVINL void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
OBN_DEVINL void ldsm_x4(uint32_t addr, uint32_t (&a)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr));
}
OBN_DEVINL void ldsm_x4_t(uint32_t addr, uint32_t (&a)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr));
}
// (x0, x1) -> binary16 pairs hi and lo with x = hi + lo to about 2^-22 |x|.
OBN_DEVINL void split_h2(float x0, float x1, uint32_t* hi, uint32_t* lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const __half2 l = __floats2half2_rn(x0 - __low2float(h), x1 - __high2float(h));
  *hi = *reinterpret_cast<const uint32_t*>(&h);
  *lo = *reinterpret_cast<const uint32_t*>(&l);
}

constexpr int kVStride = kAttnHeadDim + 8;  // halves per smem V row (ldmatrix.trans, no conflicts)

// The tensor-core contractions of one chunk, shared by the split pass and the
// clustered decode pass. On entry sK / sV hold the chunk's keys and values
// (rows >= cnt zero) and sQ the group's rotated q [G][D] (f32, visible to the
// CTA); wait_k() / wait_v() are called before the first read of K / V (the K and
// V copies may still be in flight on entry). On exit o holds this thread's P.V fragments
// (dims 32 warp + 16 mt + {grp, grp + 8}, heads 2 qd, 2 qd + 1) and red_m / red_l
// every warp's max and sum per head. k_free() runs (in every thread) once no
// thread reads sK any more, before the P.V contraction.
template <int G, class WaitK, class WaitV, class KFree>
OBN_DEVINL void tc_chunk(const __half* sK, const __half* sV, const float* sQ, float* sP, int cnt,
                         float scale, float (*red_m)[4], float (*red_l)[4], float (&o)[2][4],
                         WaitK wait_k, WaitV wait_v, KFree k_free) {
  constexpr int D = kAttnHeadDim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 2, qd = lane & 3;
  // B fragments of q (column = head grp, rows = dims), split hi / lo.
  uint32_t qh[8][2], ql[8][2];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    if (grp < G) {
      const float* qc = sQ + grp * D + ks * 16 + 2 * qd;
      split_h2(qc[0], qc[1], &qh[ks][0], &ql[ks][0]);
      split_h2(qc[8], qc[9], &qh[ks][1], &ql[ks][1]);
    } else {  // padding columns
      qh[ks][0] = qh[ks][1] = ql[ks][0] = ql[ks][1] = 0u;
    }
  }
  wait_k();
  __syncthreads();
  // Scores: warp w, keys 32w + 16 mt + {grp, grp + 8}, heads 2 qd, 2 qd + 1.
  float sc[2][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[mt][i] = 0.0f;
    const int krow = 32 * warp + 16 * mt + (lane & 15);
    const uint32_t abase = smem_u32(sK + krow * kKStride + ((lane >> 4) << 3));
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4];
      ldsm_x4(abase + ks * 32, a);
      mma_16816(sc[mt], a, qh[ks][0], qh[ks][1]);
      mma_16816(sc[mt], a, ql[ks][0], ql[ks][1]);
    }
  }
  // Scale, causal validity, per-head max over the chunk.
  float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int key = 32 * warp + 16 * mt + grp + (i >= 2 ? 8 : 0);
      sc[mt][i] = key < cnt ? __fmul_rn(sc[mt][i], scale) : -FLT_MAX;
      mx[i & 1] = fmaxf(mx[i & 1], sc[mt][i]);
    }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int sft = 4; sft <= 16; sft <<= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], sft));
  if (grp == 0) {
    red_m[2 * qd][warp] = mx[0];
    red_m[2 * qd + 1][warp] = mx[1];
  }
  __syncthreads();
  float mg[2], ls[2] = {0.0f, 0.0f};
#pragma unroll
  for (int h = 0; h < 2; ++h)
    mg[h] = fmaxf(fmaxf(red_m[2 * qd + h][0], red_m[2 * qd + h][1]),
                  fmaxf(red_m[2 * qd + h][2], red_m[2 * qd + h][3]));
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int key = 32 * warp + 16 * mt + grp + (i >= 2 ? 8 : 0);
      const int h = i & 1;
      const float pv = key < cnt ? expf(sc[mt][i] - mg[h]) : 0.0f;
      ls[h] += pv;
      if (2 * qd + h < G) sP[key * G + 2 * qd + h] = pv;
    }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int sft = 4; sft <= 16; sft <<= 1) ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], sft);
  if (grp == 0) {
    red_l[2 * qd][warp] = ls[0];
    red_l[2 * qd + 1][warp] = ls[1];
  }
  wait_v();
  __syncthreads();
  k_free();
  // P.V: warp w, dims 32w + 16 mt + {grp, grp + 8}, heads 2 qd, 2 qd + 1.
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[mt][i] = 0.0f;
  // ldmatrix.trans row addresses: lanes 0-7 keys 0-7 / dims d0.., 8-15 keys 0-7 / dims
  // d0 + 8.., 16-23 keys 8-15 / d0.., 24-31 keys 8-15 / d0 + 8..
  const int vkey = (lane & 7) + ((lane >> 4) << 3);
  const int vdim = ((lane >> 3) & 1) << 3;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t ph0 = 0u, pl0 = 0u, ph1 = 0u, pl1 = 0u;
    if (grp < G) {
      const float* pc = sP + (ks * 16 + 2 * qd) * G + grp;
      split_h2(pc[0], pc[G], &ph0, &pl0);          // keys 2qd, 2qd + 1
      split_h2(pc[8 * G], pc[9 * G], &ph1, &pl1);  // keys 2qd + 8, 2qd + 9
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t a[4];
      ldsm_x4_t(smem_u32(sV + (ks * 16 + vkey) * kVStride + 32 * warp + 16 * mt + vdim), a);
      mma_16816(o[mt], a, ph0, ph1);
      mma_16816(o[mt], a, pl0, pl1);
    }
  }
}

template <int G, class WaitK, class WaitV>
OBN_DEVINL void tc_chunk(const __half* sK, const __half* sV, const float* sQ, float* sP, int cnt,
                         float scale, float (*red_m)[4], float (*red_l)[4], float (&o)[2][4],
                         WaitK wait_k, WaitV wait_v) {
  tc_chunk<G>(sK, sV, sQ, sP, cnt, scale, red_m, red_l, o, wait_k, wait_v, [] {});
}

template <int G, bool ROPE = false>
__global__ __launch_bounds__(kAttnThreads) void k_attn_split_tc(
    const float* __restrict__ q, const __half* __restrict__ k_cache,
    const __half* __restrict__ v_cache, int n, int H, int Hkv, int S_max, int seq_len,
    const int* __restrict__ pos_dev, float scale, int nsplit, float* __restrict__ part_acc,
    float* __restrict__ part_m, float* __restrict__ part_l, float theta_base) {
  constexpr int D = kAttnHeadDim;
  constexpr int C = kAttnChunk;
  static_assert(C == 128 && D == 128 && kAttnThreads == 128 && G <= 8, "tile shape");
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sK = reinterpret_cast<__half*>(smem);                 // [C][kKStride]
  __half* sV = sK + C * kKStride;                               // [C][kVStride]
  float* sQ = reinterpret_cast<float*>(sV + C * kVStride);      // [G][D] rotated q (f32)
  float* sP = sQ + G * D;                                       // [C][G] probabilities
  __shared__ float red_m[8][4], red_l[8][4];
  __shared__ __align__(8) uint64_t bar_kv[2];  // K rows, V rows
  if (threadIdx.x == 0) {
    mbar_init(&bar_kv[0], 1);
    mbar_init(&bar_kv[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_order<ROPE>();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 2, qd = lane & 3;  // MMA fragment coordinates
  const int c = blockIdx.x, kvh = blockIdx.y;
  const size_t r = blockIdx.z;  // query row b * n + t
  const int t = static_cast<int>(r % n);
  const size_t b = r / n;
  const int s0 = c * C;
  if (pos_dev) {
    seq_len = min(*pos_dev + n, S_max);
    if (s0 >= seq_len) return;
  }
  const int limit = seq_len - n + t + 1;
  const int cnt = min(C, limit - s0);
  const size_t pbase = (r * H + static_cast<size_t>(kvh) * G) * nsplit + c;
  if (cnt <= 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      part_acc[(pbase + static_cast<size_t>(g) * nsplit) * D + tid] = 0.0f;
      if (tid == 0) {
        part_m[pbase + static_cast<size_t>(g) * nsplit] = -FLT_MAX;
        part_l[pbase + static_cast<size_t>(g) * nsplit] = 0.0f;
      }
    }
    return;
  }
  const int p_new = ROPE ? (pos_dev ? *pos_dev : seq_len - 1) : 0;
  const int new_row = (ROPE && p_new < S_max && p_new >= s0 && p_new < s0 + C) ? p_new - s0 : -1;
  // One 256-byte bulk copy per K row and per V row (thread = key), K and V on
  // their own barriers so V lands while the scores run; rows past cnt zero.
  {
    int rows = cnt - (new_row >= 0 && new_row < cnt ? 1 : 0);
    if (tid == 0) {
      mbar_arrive_expect_tx(&bar_kv[0], static_cast<uint32_t>(rows) * (D * 2));
      mbar_arrive_expect_tx(&bar_kv[1], static_cast<uint32_t>(rows) * (D * 2));
    }
    if (tid < cnt && tid != new_row) {
      const size_t g = ((b * S_max + s0 + tid) * Hkv + kvh) * D;
      bulk_g2s(sK + tid * kKStride, k_cache + g, D * 2, &bar_kv[0]);
      bulk_g2s(sV + tid * kVStride, v_cache + g, D * 2, &bar_kv[1]);
    } else if (tid >= cnt) {
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        *reinterpret_cast<uint4*>(sK + tid * kKStride + 8 * j) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(sV + tid * kVStride + 8 * j) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
  // q of the group's heads (rotated here for ROPE), f32, heads above G zero.
  if constexpr (ROPE) {
    const int slots = H + 2 * Hkv;
    const float* qrow = q + r * static_cast<size_t>(slots) * D;
    for (int e = tid; e < G * (D / 2); e += kAttnThreads) {
      const int g = e / (D / 2), i = e % (D / 2);
      const float* src = qrow + (static_cast<size_t>(kvh) * G + g) * D + 2 * i;
      float y0, y1;
      rope_pair(src[0], src[1], i, D, p_new, theta_base, &y0, &y1);
      sQ[g * D + 2 * i] = y0;
      sQ[g * D + 2 * i + 1] = y1;
    }
    if (new_row >= 0) {
      __half* kc = const_cast<__half*>(k_cache);
      __half* vc = const_cast<__half*>(v_cache);
      const size_t cache_off = ((b * S_max + p_new) * Hkv + kvh) * D;
      if (tid < D / 2) {
        const float* src = qrow + (static_cast<size_t>(H) + kvh) * D + 2 * tid;
        float y0, y1;
        rope_pair(src[0], src[1], tid, D, p_new, theta_base, &y0, &y1);
        const __half2 h = __floats2half2_rn(y0, y1);
        *reinterpret_cast<__half2*>(kc + cache_off + 2 * tid) = h;
        *reinterpret_cast<__half2*>(sK + new_row * kKStride + 2 * tid) = h;
      } else {
        const int i = tid - D / 2;
        const float* src = qrow + (static_cast<size_t>(H) + Hkv + kvh) * D + 2 * i;
        const __half2 h = __floats2half2_rn(src[0], src[1]);
        *reinterpret_cast<__half2*>(vc + cache_off + 2 * i) = h;
        *reinterpret_cast<__half2*>(sV + new_row * kVStride + 2 * i) = h;
      }
    }
  } else {
    for (int e = tid; e < G * D; e += kAttnThreads)
      sQ[e] = q[(r * H + static_cast<size_t>(kvh) * G) * D + e];
  }
  __syncthreads();
  float o[2][4];
  tc_chunk<G>(
      sK, sV, sQ, sP, cnt, scale, red_m, red_l, o,
      [&] {
        if (!mbar_wait(&bar_kv[0], 0)) mbar_wait(&bar_kv[0], 0);  // bounded; error recorded
      },
      [&] {
        if (!mbar_wait(&bar_kv[1], 0)) mbar_wait(&bar_kv[1], 0);
      });
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int dim = 32 * warp + 16 * mt + grp + (i >= 2 ? 8 : 0);
      const int h = 2 * qd + (i & 1);
      if (h < G) part_acc[(pbase + static_cast<size_t>(h) * nsplit) * D + dim] = o[mt][i];
    }
  if (tid < G) {
    part_m[pbase + static_cast<size_t>(tid) * nsplit] =
        fmaxf(fmaxf(red_m[tid][0], red_m[tid][1]), fmaxf(red_m[tid][2], red_m[tid][3]));
    part_l[pbase + static_cast<size_t>(tid) * nsplit] =
        (red_l[tid][0] + red_l[tid][1]) + (red_l[tid][2] + red_l[tid][3]);
  }
}

// ---- persistent split pass (many sequences) -----------------------------------
// k_attn_split_tc's work items (128-key chunk, KV head, query row) on persistent
// CTAs, three per SM, each cycling through its items (blockIdx.x, + gridDim.x,
// ...) with one K and one V buffer that it refills as soon as they are free:
// the next item's K rows are requested once the scores are done (tc_chunk's
// k_free hook) and its V rows once P.V is, so every CTA keeps a load in flight
// while it computes instead of loading only between its start and its compute.
// The next item's q is fetched with its K rows (tc_chunk reads q first). Copies are 16-byte cp.async pieces
// (a warp moves two 256-byte cache rows per instruction) completing on the
// buffer's barrier through cp.async.mbarrier.arrive. The per-item arithmetic
// and the partials are k_attn_split_tc's (same tc_chunk, same layout), so
// k_attn_combine's result is the same bit for bit.
constexpr int kPipeCtasPerSm = 3;

template <int G>
__global__ __launch_bounds__(kAttnThreads, kPipeCtasPerSm) void k_attn_split_pipe(
    const float* __restrict__ q, const __half* __restrict__ k_cache,
    const __half* __restrict__ v_cache, int n, int H, int Hkv, int S_max, int seq_len,
    const int* __restrict__ pos_dev, float scale, int nsplit, int rows_total,
    float* __restrict__ part_acc, float* __restrict__ part_m, float* __restrict__ part_l) {
  constexpr int D = kAttnHeadDim;
  constexpr int C = kAttnChunk;
  static_assert(C == 128 && D == 128 && kAttnThreads == 128 && G <= 8, "tile shape");
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sK = reinterpret_cast<__half*>(smem);             // [C][kKStride]
  __half* sV = sK + C * kKStride;                           // [C][kVStride]
  float* sQ = reinterpret_cast<float*>(sV + C * kVStride);  // [G][D]
  float* sP = sQ + G * D;                                   // [C][G]
  __shared__ float red_m[8][4], red_l[8][4];
  __shared__ __align__(8) uint64_t bar_k, bar_v, bar_q;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 2, qd = lane & 3;  // MMA fragment coordinates
  if (tid == 0) {  // K / V: every thread arrives once per item; q: one bulk copy
    mbar_init(&bar_k, kAttnThreads);
    mbar_init(&bar_v, kAttnThreads);
    mbar_init(&bar_q, 1);
  }
  fence_mbar_init();
  __syncthreads();
  pdl_order<false>();
  if (pos_dev) seq_len = min(*pos_dev + n, S_max);
  const int nvalid = min(nsplit, (seq_len + C - 1) / C);  // chunks that hold keys
  const int items = rows_total * Hkv * nvalid;
  const int first = static_cast<int>(blockIdx.x), step = static_cast<int>(gridDim.x);
  const int count = first < items ? (items - first + step - 1) / step : 0;
  struct Item {
    size_t r;
    int kvh, c, cnt;
  };
  auto item_at = [&](int k) {
    const int it = first + k * step;
    Item x;
    x.c = it % nvalid;
    const int rest = it / nvalid;
    x.kvh = rest % Hkv;
    x.r = static_cast<size_t>(rest / Hkv);
    const int t = static_cast<int>(x.r % n);
    x.cnt = min(C, seq_len - n + t + 1 - x.c * C);  // keys of the chunk up to the causal limit
    return x;
  };
  // Item k's K (or V) rows into dst, rows past cnt zero-filled, then this
  // thread's arrival on bar once its pieces landed (a plain arrival for an empty
  // item), so the barrier's phase k & 1 completes with the copies. 16-byte piece
  // i = tid + 128 j of the chunk is row i / 16, piece i % 16.
  auto issue = [&](int k, const __half* cache, __half* dst, int stride, uint64_t* bar) {
    const Item x = item_at(k);
    const int rows = max(0, x.cnt);
    if (rows == 0) {
      mbar_arrive(bar);
      return;
    }
    const size_t g0 = ((x.r / n * S_max + static_cast<size_t>(x.c) * C) * Hkv + x.kvh) * D;
#pragma unroll 4
    for (int j = 0; j < C * D / 8 / kAttnThreads; ++j) {
      const int i = tid + kAttnThreads * j, row = i >> 4, pc = i & 15;
      const size_t go = row < rows ? g0 + static_cast<size_t>(row) * Hkv * D + pc * 8 : g0;
      cp_async16_zfill(dst + row * stride + pc * 8, cache + go, row < rows ? 16u : 0u);
    }
    cp_async_arrive(bar);
  };
  // q of item k's group (f32 [G][D]): one bulk copy (a cp.async arrival would
  // also wait for the K / V pieces issued before it), phase k & 1 of bar_q.
  auto fetch_q = [&](int k) {
    if (tid != 0) return;
    const Item x = item_at(k);
    fence_proxy_async_smem();  // the previous item's generic reads of sQ come first
    mbar_arrive_expect_tx(&bar_q, static_cast<uint32_t>(G * D * 4));
    bulk_g2s(sQ, q + (x.r * H + static_cast<size_t>(x.kvh) * G) * D, G * D * 4, &bar_q);
  };
  auto wait2 = [](uint64_t* bar, uint32_t ph) {  // bounded; the error is recorded
    if (!mbar_wait(bar, ph)) mbar_wait(bar, ph);
  };
  if (count > 0) {
    issue(0, k_cache, sK, kKStride, &bar_k);
    issue(0, v_cache, sV, kVStride, &bar_v);
    fetch_q(0);
  }
  for (int k = 0; k < count; ++k) {
    const Item x = item_at(k);
    const uint32_t ph = static_cast<uint32_t>(k) & 1u;
    wait2(&bar_q, ph);  // this item's q
    const size_t pbase = (x.r * H + static_cast<size_t>(x.kvh) * G) * nsplit + x.c;
    if (x.cnt <= 0) {  // no key of the chunk is visible to this query row
#pragma unroll
      for (int g = 0; g < G; ++g) {
        part_acc[(pbase + static_cast<size_t>(g) * nsplit) * D + tid] = 0.0f;
        if (tid == 0) {
          part_m[pbase + static_cast<size_t>(g) * nsplit] = -FLT_MAX;
          part_l[pbase + static_cast<size_t>(g) * nsplit] = 0.0f;
        }
      }
      wait2(&bar_k, ph);  // the empty item's plain arrivals
      wait2(&bar_v, ph);
      __syncthreads();  // every thread is past this item's phases
      if (k + 1 < count) {
        issue(k + 1, k_cache, sK, kKStride, &bar_k);
        issue(k + 1, v_cache, sV, kVStride, &bar_v);
        fetch_q(k + 1);
      }
      continue;
    }
    float o[2][4];
    tc_chunk<G>(
        sK, sV, sQ, sP, x.cnt, scale, red_m, red_l, o, [&] { wait2(&bar_k, ph); },
        [&] { wait2(&bar_v, ph); },
        [&] {  // the scores are done (and q is in registers): the next item's K rows and q
          if (k + 1 < count) {
            issue(k + 1, k_cache, sK, kKStride, &bar_k);
            fetch_q(k + 1);
          }
        });
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int dim = 32 * warp + 16 * mt + grp + (i >= 2 ? 8 : 0);
        const int h = 2 * qd + (i & 1);
        if (h < G) part_acc[(pbase + static_cast<size_t>(h) * nsplit) * D + dim] = o[mt][i];
      }
    if (tid < G) {
      part_m[pbase + static_cast<size_t>(tid) * nsplit] =
          fmaxf(fmaxf(red_m[tid][0], red_m[tid][1]), fmaxf(red_m[tid][2], red_m[tid][3]));
      part_l[pbase + static_cast<size_t>(tid) * nsplit] =
          (red_l[tid][0] + red_l[tid][1]) + (red_l[tid][2] + red_l[tid][3]);
    }
    __syncthreads();  // sV, sP and red_* are free again
    if (k + 1 < count) issue(k + 1, v_cache, sV, kVStride, &bar_v);
  }
}

// ---- prefill attention: one 16-row query tile per CTA ------------------------
// For chunks of many new tokens (n >= kFaMinRows) the split pass would read every
// 128-key chunk once per query row. k_attn_prefill_fa gives a CTA 16 consecutive
// query rows of one sequence and one KV head; warp w takes query head
// kvh * G + w % G for those rows (and, with KS = 2, the key blocks of parity
// w / G), so all warps share every K / V block. Keys stream
// in 64-key blocks (double-buffered 16-byte cp.async pieces); per block each
// warp computes S = Q K^T (mma.sync m16n8k16, q split into binary16 hi + lo),
// scales, masks the causal limit, updates its rows' running max and sum (online
// softmax) and accumulates O += P V (P split into hi + lo). The outputs are
// written once, divided by the sums: no partials, no combine. Numerically the
// same function as the split + combine passes in another order (the oracle
// tolerance, 1e-4 relative).
constexpr int kFaRows = 16;      // query rows per CTA (the MMA's M)
constexpr int kFaKeys = 64;      // keys per block
constexpr int kFaMinRows = 16;   // query rows per sequence from which prefill uses it
constexpr int kFaStride = kAttnHeadDim + 8;  // halves per smem K / V row

// KS = 2 (G <= 4): two warps per head, the first taking the even key blocks and
// the second the odd ones, their running max / sum / O merged at the end, which
// halves the chain of the tiles that see the most keys. Tiles are issued from
// the last (longest) one down.
template <int G, int KS>
__global__ __launch_bounds__(32 * G * KS) void k_attn_prefill_fa(
    const float* __restrict__ q, const __half* __restrict__ k_cache,
    const __half* __restrict__ v_cache, int n, int H, int Hkv, int S_max, int seq_len,
    const int* __restrict__ pos_dev, float scale, float* __restrict__ out) {
  constexpr int D = kAttnHeadDim;
  constexpr int NT = 32 * G * KS;  // threads
  static_assert(D == 128 && G >= 1 && G <= 8 && (KS == 1 || KS == 2), "tile shape");
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sKV = reinterpret_cast<__half*>(smem);  // [2 stages][KS blocks][K, V][kFaKeys][kFaStride]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 2, qd = lane & 3;
  const int hw = warp % G, kp = warp / G;  // head within the group, key-block parity
  const int t0 = (gridDim.x - 1 - blockIdx.x) * kFaRows, kvh = blockIdx.y;
  const size_t b = blockIdx.z;
  const int h = kvh * G + hw;  // this warp's query head
  pdl_launch_dependents();
  pdl_wait();
  if (pos_dev) seq_len = min(*pos_dev + n, S_max);
  if (t0 >= n) return;
  const int t_last = min(t0 + kFaRows, n) - 1;
  const int kmax = seq_len - n + t_last + 1;  // keys visible to the tile's last row
  const int nkb = (kmax + kFaKeys - 1) / kFaKeys;
  // q rows t0 + grp and t0 + grp + 8 as A fragments, split hi / lo (rows past n zero)
  uint32_t qh[8][4], ql[8][4];
  {
    const int ta = t0 + grp, tb = t0 + grp + 8;
    const float* qa = q + ((b * n + ta) * H + h) * static_cast<size_t>(D);
    const float* qb = q + ((b * n + tb) * H + h) * static_cast<size_t>(D);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d0 = 16 * ks + 2 * qd;
      const float2 a0 = ta < n ? *reinterpret_cast<const float2*>(qa + d0) : make_float2(0.f, 0.f);
      const float2 a1 = tb < n ? *reinterpret_cast<const float2*>(qb + d0) : make_float2(0.f, 0.f);
      const float2 a2 =
          ta < n ? *reinterpret_cast<const float2*>(qa + d0 + 8) : make_float2(0.f, 0.f);
      const float2 a3 =
          tb < n ? *reinterpret_cast<const float2*>(qb + d0 + 8) : make_float2(0.f, 0.f);
      split_h2(a0.x, a0.y, &qh[ks][0], &ql[ks][0]);
      split_h2(a1.x, a1.y, &qh[ks][1], &ql[ks][1]);
      split_h2(a2.x, a2.y, &qh[ks][2], &ql[ks][2]);
      split_h2(a3.x, a3.y, &qh[ks][3], &ql[ks][3]);
    }
  }
  // K and V rows of blocks KS it .. KS it + KS - 1 into stage it & 1 (rows at or
  // past kmax zero-filled)
  auto load_block = [&](int it) {
    __half* sK0 = sKV + (it & 1) * KS * 2 * kFaKeys * kFaStride;
    for (int i = tid; i < KS * kFaKeys * (D / 8); i += NT) {
      const int j = i / (kFaKeys * (D / 8)), ii = i - j * (kFaKeys * (D / 8));
      __half* sK = sK0 + j * 2 * kFaKeys * kFaStride;
      __half* sV = sK + kFaKeys * kFaStride;
      const int row = ii >> 4, pc = ii & 15, key = (KS * it + j) * kFaKeys + row;
      const size_t g = key < kmax ? ((b * S_max + key) * Hkv + kvh) * D + pc * 8
                                  : ((b * S_max) * Hkv + kvh) * D;
      const uint32_t nbytes = key < kmax ? 16u : 0u;
      cp_async16_zfill(sK + row * kFaStride + pc * 8, k_cache + g, nbytes);
      cp_async16_zfill(sV + row * kFaStride + pc * 8, v_cache + g, nbytes);
    }
    cp_async_commit();
  };
  // running max / sum of rows grp (index 0) and grp + 8 (index 1); O accumulators
  // oacc[dt]: dims 8 dt + 2 qd, + 1 of rows grp (0, 1) and grp + 8 (2, 3)
  float m_run[2] = {-FLT_MAX, -FLT_MAX}, l_run[2] = {0.0f, 0.0f};
  float oacc[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt)
#pragma unroll
    for (int i = 0; i < 4; ++i) oacc[dt][i] = 0.0f;
  const int lim0 = seq_len - n + t0 + grp;  // last key row grp may see (row grp + 8: + 8)
  const bool row_ok[2] = {t0 + grp < n, t0 + grp + 8 < n};
  const int nit = (nkb + KS - 1) / KS;
  if (nit > 0) load_block(0);
  for (int it = 0; it < nit; ++it) {
    if (it + 1 < nit) {
      load_block(it + 1);
      cp_async_wait_group<1>();  // iteration it's blocks landed (this thread's pieces)
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();  // every thread's pieces of iteration it
    const int kb = KS * it + kp;  // this warp's block
    if (kb >= nkb) {
      __syncthreads();
      continue;
    }
    const __half* sK = sKV + ((it & 1) * KS + kp) * 2 * kFaKeys * kFaStride;
    const __half* sV = sK + kFaKeys * kFaStride;
    const int key0 = kb * kFaKeys;
    // S = Q K^T: sacc[nt] holds keys key0 + 8 nt + 2 qd, + 1 of rows grp, grp + 8
    float sacc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) sacc[nt][i] = 0.0f;
      // ldmatrix x4 of keys 8 nt .. + 7: matrices d 0-7, 8-15, 16-23, 24-31 of each 32-d step
      const uint32_t kaddr =
          smem_u32(sK + (8 * nt + (lane & 7)) * kFaStride + ((lane >> 3) << 3));
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {  // 32 dims per ldmatrix.x4 = two k-steps
        uint32_t kb4[4];
        ldsm_x4(kaddr + k2 * 64, kb4);
        mma_16816(sacc[nt], qh[2 * k2], kb4[0], kb4[1]);
        mma_16816(sacc[nt], ql[2 * k2], kb4[0], kb4[1]);
        mma_16816(sacc[nt], qh[2 * k2 + 1], kb4[2], kb4[3]);
        mma_16816(sacc[nt], ql[2 * k2 + 1], kb4[2], kb4[3]);
      }
    }
    // scale, causal mask, block max per row
    float bmax[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1, key = key0 + 8 * nt + 2 * qd + (i & 1);
        const bool ok = row_ok[r] && key <= lim0 + 8 * r;
        sacc[nt][i] = ok ? __fmul_rn(sacc[nt][i], scale) : -FLT_MAX;
        bmax[r] = fmaxf(bmax[r], sacc[nt][i]);
      }
    float alpha[2], mnew[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      bmax[r] = fmaxf(bmax[r], __shfl_xor_sync(0xffffffffu, bmax[r], 1));
      bmax[r] = fmaxf(bmax[r], __shfl_xor_sync(0xffffffffu, bmax[r], 2));
      mnew[r] = fmaxf(m_run[r], bmax[r]);
      alpha[r] = expf(m_run[r] - mnew[r]);  // 1 while both are -FLT_MAX
      m_run[r] = mnew[r];
    }
    // P = exp(S - max) (masked entries 0), the rows' sums, O rescaled
    float psum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = i >> 1;
        const float p = sacc[nt][i] == -FLT_MAX ? 0.0f : expf(sacc[nt][i] - mnew[r]);
        sacc[nt][i] = p;
        psum[r] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 1);
      psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 2);
      l_run[r] = fmaf(l_run[r], alpha[r], psum[r]);
    }
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      oacc[dt][0] *= alpha[0];
      oacc[dt][1] *= alpha[0];
      oacc[dt][2] *= alpha[1];
      oacc[dt][3] *= alpha[1];
    }
    // O += P V over the block's 4 key steps of 16
    const int vkey = (lane & 7) + (((lane >> 3) & 1) << 3);
    const int vdim = (lane >> 4) << 3;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t ph[4], pl[4];
      split_h2(sacc[2 * ks][0], sacc[2 * ks][1], &ph[0], &pl[0]);
      split_h2(sacc[2 * ks][2], sacc[2 * ks][3], &ph[1], &pl[1]);
      split_h2(sacc[2 * ks + 1][0], sacc[2 * ks + 1][1], &ph[2], &pl[2]);
      split_h2(sacc[2 * ks + 1][2], sacc[2 * ks + 1][3], &ph[3], &pl[3]);
#pragma unroll
      for (int d2 = 0; d2 < 8; ++d2) {  // 16 dims per ldmatrix.x4.trans
        uint32_t vb[4];
        ldsm_x4_t(smem_u32(sV + (16 * ks + vkey) * kFaStride + 16 * d2 + vdim), vb);
        mma_16816(oacc[2 * d2], ph, vb[0], vb[1]);
        mma_16816(oacc[2 * d2], pl, vb[0], vb[1]);
        mma_16816(oacc[2 * d2 + 1], ph, vb[2], vb[3]);
        mma_16816(oacc[2 * d2 + 1], pl, vb[2], vb[3]);
      }
    }
    __syncthreads();  // stage it & 1 is read; the next load may overwrite it
  }
  if constexpr (KS == 2) {
    // the odd-block warps hand their (max, sum, O) to the even-block warps of the
    // same head through the (now idle) stage buffers; those merge them
    float* xch = reinterpret_cast<float*>(smem) + (hw * 32 + lane) * 68;
    if (kp == 1) {
      xch[0] = m_run[0];
      xch[1] = m_run[1];
      xch[2] = l_run[0];
      xch[3] = l_run[1];
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
#pragma unroll
        for (int i = 0; i < 4; ++i) xch[4 + 4 * dt + i] = oacc[dt][i];
    }
    __syncthreads();
    if (kp == 1) return;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float m1 = xch[r], l1 = xch[2 + r];
      const float mm = fmaxf(m_run[r], m1);
      const float a0 = expf(m_run[r] - mm), a1 = expf(m1 - mm);
      l_run[r] = __fadd_rn(__fmul_rn(l_run[r], a0), __fmul_rn(l1, a1));
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          oacc[dt][2 * r + e] =
              __fadd_rn(__fmul_rn(oacc[dt][2 * r + e], a0), __fmul_rn(xch[4 + 4 * dt + 2 * r + e], a1));
    }
  }
  // outputs: O / l for the tile's rows below n
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!row_ok[r]) continue;
    const int t = t0 + grp + 8 * r;
    float* o = out + ((b * n + t) * H + h) * static_cast<size_t>(D);
    const float inv_l = 1.0f / l_run[r];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
      *reinterpret_cast<float2*>(o + 8 * dt + 2 * qd) =
          make_float2(oacc[dt][2 * r] * inv_l, oacc[dt][2 * r + 1] * inv_l);
  }
}

// ---- clustered decode pass ---------------------------------------------------
// One decode token per sequence (n = 1) with RoPE, the cache append, the split
// pass and the combine in ONE launch: a cluster of CS CTAs per (sequence, KV
// head). CTA `rank` takes the chunks rank, rank + CS, ... (up to kClMaxSlots),
// runs tc_chunk on each and keeps every chunk's partial (max, sum, unnormalised
// P.V) in its own shared memory. After a cluster barrier each CTA gathers its
// G * D / CS outputs' partials from all CTAs over distributed shared memory and
// combines them with k_attn_combine's arithmetic in the same chunk order, so the
// result equals the split + combine passes bit for bit.
//
// The chunk of the first slot is copied before griddepcontrol.wait, while the
// QKV projection before this kernel still runs: its rows below pos - 1 were
// appended by earlier steps. Appending passes (this one, the RoPE append, the
// RoPE split) let their dependents launch only after their own wait or at their
// end, so while this kernel waits every kernel before the latest appending pass
// has completed; the one row that pass may still be writing is pos - 1 in a
// decode sequence (or a row at or above pos when the caller went back), and row
// pos - 1 is copied after the wait. The device position (*pos_dev) is written by
// stream-ordered copies, never by a kernel of this library.
constexpr int kClMaxSlots = 4;  // chunks per CTA

OBN_DEVINL uint32_t cl_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
OBN_DEVINL void cl_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
OBN_DEVINL void cl_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Stores into another CTA's shared memory (cluster addresses) that complete
// their bytes on that CTA's mbarrier.
OBN_DEVINL void st_async_v4(uint32_t dst, float4 v, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, "
      "[%5];" ::"r"(dst),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar)
      : "memory");
}
OBN_DEVINL void st_async_v2(uint32_t dst, float a, float b, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
          dst),
      "f"(a), "f"(b), "r"(remote_bar)
      : "memory");
}
// Bounded wait on a barrier that other CTAs of the cluster complete.
OBN_DEVINL bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
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
OBN_DEVINL void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Outputs of the group a CTA combines, and the stride of one chunk's record in
// its receive buffer: `per` partial outputs, then the chunk's (max, sum) of the
// head those outputs belong to, padded to 16 bytes.
__host__ __device__ inline int cl_per(int G, int CS) { return G * kAttnHeadDim / CS; }
__host__ __device__ inline int cl_rec(int G, int CS) { return cl_per(G, CS) + 4; }

// Dynamic shared memory: K and V tiles, q, probabilities, one chunk's partial
// [G][D] + (max, sum) per head, then the receive buffer [CS * slots][rec].
inline size_t cl_smem_bytes(int G, int CS, int slots) {
  return static_cast<size_t>(kAttnChunk) * kKStride * 2 +
         static_cast<size_t>(kAttnChunk) * kVStride * 2 + static_cast<size_t>(G) * kAttnHeadDim * 4 +
         static_cast<size_t>(kAttnChunk) * G * 4 + static_cast<size_t>(G) * kAttnHeadDim * 4 + 64 +
         static_cast<size_t>(CS) * slots * cl_rec(G, CS) * 4;
}

template <int G>
__global__ __launch_bounds__(kAttnThreads) void k_attn_decode_cl(
    const float* __restrict__ qkv, __half* __restrict__ k_cache, __half* __restrict__ v_cache,
    int H, int Hkv, int S_max, int pos, const int* __restrict__ pos_dev, float scale, int nsplit,
    int slots, float* __restrict__ out, float theta_base) {
  constexpr int D = kAttnHeadDim;
  constexpr int C = kAttnChunk;
  constexpr uint32_t kRowBytes = D * 2;
  static_assert(C == 128 && D == 128 && kAttnThreads == 128 && G <= 8, "tile shape");
  extern __shared__ __align__(16) unsigned char smem[];
  const int CS = static_cast<int>(gridDim.x);  // the cluster spans the grid's x
  const int per = cl_per(G, CS), rec = cl_rec(G, CS);
  __half* sK = reinterpret_cast<__half*>(smem);             // [C][kKStride]
  __half* sV = sK + C * kKStride;                           // [C][kVStride]
  float* sQ = reinterpret_cast<float*>(sV + C * kVStride);  // [G][D] rotated q
  float* sP = sQ + G * D;                                   // [C][G] probabilities
  float* sAcc = sP + C * G;                                 // [G][D] a chunk's partial P.V
  float* sM = sAcc + G * D;                                 // [8] its max per head
  float* sL = sM + 8;                                       // [8] its sum per head
  float* rbuf = sL + 8;                                     // [CS * slots][rec] received
  __shared__ float red_m[8][4], red_l[8][4];
  __shared__ float s_cos[D / 2], s_sin[D / 2];  // RoPE angle of dimension pair i at pos
  __shared__ __align__(8) uint64_t bar[3];      // rows before / after the wait; partials in
  const int tid = threadIdx.x;
  const int rank = static_cast<int>(blockIdx.x);
  const int kvh = blockIdx.y;
  const size_t b = blockIdx.z;
  const int p_new = pos_dev ? *pos_dev : pos;
  const int seq_len = min(p_new + 1, S_max);
  const int nvalid = min(nsplit, (seq_len + C - 1) / C);  // chunks that hold keys
  const int late = max(p_new - 1, 0);  // first row copied after the wait
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    fence_mbar_init();
  }
  if (tid < D / 2) rope_angle(tid, D, p_new, theta_base, &s_cos[tid], &s_sin[tid]);
  __syncthreads();
  cl_arrive_release();  // every CTA's barriers initialised before the first remote store
  if (tid == 0)  // the partials of every chunk for this CTA's outputs
    mbar_arrive_expect_tx(&bar[2], static_cast<uint32_t>(max(nvalid, 0) * (per + 2) * 4));

  // Bulk copies (one 256-byte K row and one V row per thread) of the chunk at s0:
  // its rows at positions [from, upto) below seq_len, except the new token's row,
  // completing on `bar_`. With zero_tail, rows past seq_len become zero.
  auto copy_rows = [&](int s0, int from, int upto, uint64_t* bar_, bool zero_tail) {
    const int a = max(s0, from), e = min(min(s0 + C, seq_len), upto);
    int rows = max(e - a, 0);
    if (p_new >= a && p_new < e) --rows;
    if (tid == 0) mbar_arrive_expect_tx(bar_, static_cast<uint32_t>(rows) * 2u * kRowBytes);
    const int p = s0 + tid;
    if (p >= a && p < e && p != p_new) {
      const size_t g = ((b * S_max + p) * Hkv + kvh) * D;
      bulk_g2s(sK + tid * kKStride, k_cache + g, kRowBytes, bar_);
      bulk_g2s(sV + tid * kVStride, v_cache + g, kRowBytes, bar_);
    } else if (zero_tail && p >= seq_len) {
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        *reinterpret_cast<uint4*>(sK + tid * kKStride + 8 * j) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(sV + tid * kVStride + 8 * j) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  auto wait_rows = [&](uint64_t* bar_, uint32_t parity) {
    if (!mbar_wait(bar_, parity)) mbar_wait(bar_, parity);  // bounded; the error is recorded
  };
  // The new token's rotated key and value: into the caches and the chunk's tiles.
  const float* qrow = qkv + b * static_cast<size_t>(H + 2 * Hkv) * D;
  auto append_new = [&](int s0) {
    if (p_new < 0 || p_new >= S_max || p_new < s0 || p_new >= s0 + C) return;
    const int row = p_new - s0;
    const size_t cache_off = ((b * S_max + p_new) * Hkv + kvh) * D;
    if (tid < D / 2) {
      const float* src = qrow + (static_cast<size_t>(H) + kvh) * D + 2 * tid;
      float y0, y1;
      rope_rotate(src[0], src[1], s_cos[tid], s_sin[tid], &y0, &y1);
      const __half2 h = __floats2half2_rn(y0, y1);
      *reinterpret_cast<__half2*>(k_cache + cache_off + 2 * tid) = h;
      *reinterpret_cast<__half2*>(sK + row * kKStride + 2 * tid) = h;
    } else {
      const int i = tid - D / 2;
      const float* src = qrow + (static_cast<size_t>(H) + Hkv + kvh) * D + 2 * i;
      const __half2 h = __floats2half2_rn(src[0], src[1]);
      *reinterpret_cast<__half2*>(v_cache + cache_off + 2 * i) = h;
      *reinterpret_cast<__half2*>(sV + row * kVStride + 2 * i) = h;
    }
  };
  // One chunk's partial -> the CTAs that combine it: CTA j receives outputs
  // [j * per, j * per + per) and the (max, sum) of their head, as record c.
  auto push_partial = [&](int c, const float (&o)[2][4]) {
    const int lane = tid & 31, warp = tid >> 5, grp = lane >> 2, qd = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int dim = 32 * warp + 16 * mt + grp + (i >= 2 ? 8 : 0);
        const int h = 2 * qd + (i & 1);
        if (h < G) sAcc[h * D + dim] = o[mt][i];
      }
    if (tid < G) {
      sM[tid] = fmaxf(fmaxf(red_m[tid][0], red_m[tid][1]), fmaxf(red_m[tid][2], red_m[tid][3]));
      sL[tid] = (red_l[tid][0] + red_l[tid][1]) + (red_l[tid][2] + red_l[tid][3]);
    }
    __syncthreads();
    const int pieces = per / 4 + 1;
    for (int e = tid; e < CS * pieces; e += kAttnThreads) {
      const int j = e / pieces, piece = e - j * pieces;
      const uint32_t rbar = cl_map(smem_u32(&bar[2]), static_cast<uint32_t>(j));
      const uint32_t dst = cl_map(smem_u32(rbuf + c * rec), static_cast<uint32_t>(j));
      if (piece < per / 4) {
        const float4 v = *reinterpret_cast<const float4*>(sAcc + j * per + 4 * piece);
        st_async_v4(dst + 16u * piece, v, rbar);
      } else {
        const int g = (j * per) / D;
        st_async_v2(dst + 4u * per, sM[g], sL[g], rbar);
      }
    }
  };

  // ---- before the wait: the first slot's rows below pos - 1, row pos - 1 into L2
  if (rank < nvalid) {
    copy_rows(rank * C, 0, late, &bar[0], true);
    if (tid == 0 && p_new >= 1 && p_new - 1 < seq_len && (p_new - 1) / C == rank) {
      const size_t g = ((b * S_max + (p_new - 1)) * Hkv + kvh) * D;
      prefetch_l2(k_cache + g, kRowBytes);
      prefetch_l2(v_cache + g, kRowBytes);
    }
  }
  cl_wait_acquire();
  pdl_wait();
  pdl_launch_dependents();

  // ---- after the wait: q, the late rows, the new row, then every slot
  for (int e = tid; e < G * (D / 2); e += kAttnThreads) {
    const int g = e / (D / 2), i = e % (D / 2);
    const float* src = qrow + (static_cast<size_t>(kvh) * G + g) * D + 2 * i;
    float y0, y1;
    rope_rotate(src[0], src[1], s_cos[i], s_sin[i], &y0, &y1);
    sQ[g * D + 2 * i] = y0;
    sQ[g * D + 2 * i + 1] = y1;
  }
  for (int slot = 0; slot < slots; ++slot) {
    const int c = rank + slot * CS;
    if (c >= nvalid) break;  // uniform per CTA
    const int s0 = c * C;
    const int cnt = min(C, seq_len - s0);
    if (slot > 0) {  // the previous slot is done with the tiles (generic writes included)
      fence_proxy_async_smem();
      __syncthreads();
    }
    copy_rows(s0, slot == 0 ? late : 0, 0x7fffffff, &bar[1], slot > 0);
    append_new(s0);
    if (slot == 0) wait_rows(&bar[0], 0);
    wait_rows(&bar[1], static_cast<uint32_t>(slot & 1));
    __syncthreads();
    float o[2][4];
    tc_chunk<G>(sK, sV, sQ, sP, cnt, scale, red_m, red_l, o, [] {}, [] {});
    push_partial(c, o);
  }

  // ---- combine: k_attn_combine's arithmetic over the records, in chunk order.
  // Every output of this CTA belongs to one head, so the chunk weights are
  // shared: lane l of each warp holds chunks l and l + 32 (nvalid <= 64) and
  // hands them out by shuffles; the max is exact in any order.
  const bool got = mbar_wait_cluster(&bar[2], 0);
  if (got && tid < ((per + 31) & ~31)) {  // whole warps
    const int lane = tid & 31;
    const bool h0 = lane < nvalid, h1 = lane + 32 < nvalid;
    const float m0 = h0 ? rbuf[lane * rec + per] : -FLT_MAX;
    const float m1 = h1 ? rbuf[(lane + 32) * rec + per] : -FLT_MAX;
    const float l0 = h0 ? rbuf[lane * rec + per + 1] : 0.0f;
    const float l1 = h1 ? rbuf[(lane + 32) * rec + per + 1] : 0.0f;
    float M = fmaxf(m0, m1);
#pragma unroll
    for (int sft = 16; sft >= 1; sft >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sft));
    const float w0 = l0 == 0.0f ? 0.0f : expf(m0 - M);
    const float w1 = l1 == 0.0f ? 0.0f : expf(m1 - M);
    const int j = tid;
    float L = 0.0f, o = 0.0f;
    // an empty chunk (l == 0) leaves L and o as they are; selects, not branches,
    // so the loads and shuffles of later chunks issue ahead of the chain
#pragma unroll 8
    for (int c = 0; c < nvalid; ++c) {
      const float l = __shfl_sync(0xffffffffu, c < 32 ? l0 : l1, c & 31);
      const float w = __shfl_sync(0xffffffffu, c < 32 ? w0 : w1, c & 31);
      const float a = j < per ? rbuf[c * rec + j] : 0.0f;
      const float Ln = fmaf(w, l, L), on = fmaf(w, a, o);
      L = l == 0.0f ? L : Ln;
      o = l == 0.0f ? o : on;
    }
    if (j < per) {
      const int oi = rank * per + j;
      const int g = oi / D, dim = oi - g * D;
      out[((b * H) + static_cast<size_t>(kvh) * G + g) * D + dim] = o / L;
    }
  }
}

// One CTA per (query row, head): thread = dimension.
__global__ __launch_bounds__(kAttnThreads) void k_attn_combine(const float* __restrict__ part_acc,
                                                               const float* __restrict__ part_m,
                                                               const float* __restrict__ part_l,
                                                               int nsplit, int n, int S_max,
                                                               const int* __restrict__ pos_dev,
                                                               float* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int D = kAttnHeadDim;
  const size_t rh = blockIdx.x;  // r * H + h
  const int tid = threadIdx.x;
  // splits that hold keys (all of them unless the position is read on the device)
  const int nvalid =
      pos_dev ? min(nsplit, (min(*pos_dev + n, S_max) + kAttnChunk - 1) / kAttnChunk) : nsplit;
  // Every split's (m, l) in shared memory, every thread's accumulator values in
  // flight before the first dependent step; then the rescaling in split order.
  __shared__ float s_m[kMaxSplits], s_l[kMaxSplits];
  const int nfast = min(nvalid, kMaxSplits);  // longer caches: the rest one by one
  for (int c = tid; c < nfast; c += kAttnThreads) {
    s_m[c] = part_m[rh * nsplit + c];
    s_l[c] = part_l[rh * nsplit + c];
  }
  float av[kMaxSplits];
#pragma unroll
  for (int c = 0; c < kMaxSplits; ++c)
    av[c] = c < nfast ? part_acc[(rh * nsplit + c) * D + tid] : 0.0f;
  __syncthreads();
  float M = -FLT_MAX;
  for (int c = 0; c < nfast; ++c) M = fmaxf(M, s_m[c]);
  for (int c = nfast; c < nvalid; ++c) M = fmaxf(M, part_m[rh * nsplit + c]);
  float L = 0.0f, o = 0.0f;
#pragma unroll
  for (int c = 0; c < kMaxSplits; ++c) {
    if (c >= nfast) break;
    const float l = s_l[c];
    if (l == 0.0f) continue;  // an empty chunk
    const float w = expf(s_m[c] - M);
    L = fmaf(w, l, L);
    o = fmaf(w, av[c], o);
  }
  for (int c = nfast; c < nvalid; ++c) {
    const float l = part_l[rh * nsplit + c];
    if (l == 0.0f) continue;
    const float w = expf(part_m[rh * nsplit + c] - M);
    L = fmaf(w, l, L);
    o = fmaf(w, part_acc[(rh * nsplit + c) * D + tid], o);
  }
  out[rh * D + tid] = o / L;
}

template <int G, bool ROPE>
cudaError_t launch_split(const float* q, const __half* k_cache, const __half* v_cache, int B,
                         int n, int H, int Hkv, int S_max, int seq_len, const int* pos_dev,
                         float scale, int nsplit, float* pa, float* pm, float* pl, cudaStream_t s,
                         float theta_base) {
  constexpr int D = kAttnHeadDim;
  // The tensor-core pass unless OBN_ATTN_TC=0 selects the CUDA-core one.
  static const bool tc = [] {
    const char* v = std::getenv("OBN_ATTN_TC");
    return !(v && v[0] == '0');
  }();
  const size_t smem =
      tc ? static_cast<size_t>(kAttnChunk) * kKStride * 2 + static_cast<size_t>(kAttnChunk) * kVStride * 2 +
               static_cast<size_t>(G) * D * 4 + static_cast<size_t>(kAttnChunk) * G * 4
         : static_cast<size_t>(kAttnChunk) * kKStride * 2 + static_cast<size_t>(kAttnChunk) * D * 2 +
               static_cast<size_t>(G) * D * 4 + static_cast<size_t>(G) * kAttnChunk * 4;
  auto kern = tc ? k_attn_split_tc<G, ROPE> : k_attn_split<G, ROPE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, Hkv, B * n);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, q, k_cache, v_cache, n, H, Hkv, S_max, seq_len, pos_dev,
                            scale, nsplit, pa, pm, pl, theta_base);
}

// The persistent split pass when there are at least kPipeMinItemsPerSm items per
// SM (and q is 16-byte aligned for its bulk copy); OBN_ATTN_PIPE=0 keeps the
// one-item CTAs. Read once per process.
constexpr int kPipeMinItemsPerSm = 4;
bool attn_pipe_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("OBN_ATTN_PIPE");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <int G>
cudaError_t launch_split_pipe(const float* q, const __half* k_cache, const __half* v_cache, int B,
                              int n, int H, int Hkv, int S_max, int seq_len, const int* pos_dev,
                              float scale, int nsplit, float* pa, float* pm, float* pl,
                              cudaStream_t s) {
  constexpr int D = kAttnHeadDim;
  const size_t smem = static_cast<size_t>(kAttnChunk) * (kKStride + kVStride) * 2 +
                      (static_cast<size_t>(G) * D + static_cast<size_t>(kAttnChunk) * G) * 4;
  auto kern = k_attn_split_pipe<G>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAttnThreads, smem);
  if (e != cudaSuccess) return e;
  const int rows_total = B * n;
  const long long items = static_cast<long long>(rows_total) * Hkv * nsplit;
  const long long cap = static_cast<long long>(per_sm > 0 ? per_sm : 1) * num_sms_cached();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(items < cap ? items : cap));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, q, k_cache, v_cache, n, H, Hkv, S_max, seq_len, pos_dev,
                            scale, nsplit, rows_total, pa, pm, pl);
}

// Prefill chunks of >= kFaMinRows query rows per sequence take the 16-row tile
// pass; OBN_ATTN_FA=0 keeps them on split + combine. Read once per process.
bool attn_fa_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("OBN_ATTN_FA");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <int G, int KS>
cudaError_t launch_prefill_fa_ks(const float* q, const __half* k_cache, const __half* v_cache, int B,
                              int n, int H, int Hkv, int S_max, int seq_len,
                              const int* pos_dev, float scale, float* out, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(2) * KS * 2 * kFaKeys * kFaStride * 2;
  auto kern = k_attn_prefill_fa<G, KS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((n + kFaRows - 1) / kFaRows), Hkv, B);
  cfg.blockDim = dim3(32 * G * KS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, q, k_cache, v_cache, n, H, Hkv, S_max, seq_len, pos_dev,
                            scale, out);
}

// Two warps per head while the CTA's registers allow it (G <= 4).
template <int G>
cudaError_t launch_prefill_fa(const float* q, const __half* k_cache, const __half* v_cache, int B,
                              int n, int H, int Hkv, int S_max, int seq_len,
                              const int* pos_dev, float scale, float* out, cudaStream_t s) {
  return launch_prefill_fa_ks<G, (G <= 4 ? 2 : 1)>(q, k_cache, v_cache, B, n, H, Hkv, S_max,
                                                   seq_len, pos_dev, scale, out, s);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_attn(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Cluster size of the clustered decode pass for group size G on the current
// device: 16 when a 16-CTA cluster with the largest shared memory it uses can be
// resident, else 8 when an 8-CTA one can, else 0 (the split + combine passes).
// OBN_ATTN_CLUSTER=0 selects 0. Queried once per device.
template <int G>
int decode_cluster_size() {
  static const bool enabled = [] {
    const char* v = std::getenv("OBN_ATTN_CLUSTER");
    return !(v && v[0] == '0');
  }();
  static int cache[64] = {};  // 0 not queried, -1 none, else the size
  if (!enabled) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (cache[dev]) return cache[dev] > 0 ? cache[dev] : 0;
  auto kern = k_attn_decode_cl<G>;
  int best = -1;
  // the attribute ends at the largest size any launch uses (16 first, then 8)
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
      cudaSuccess) {
    for (int cs : {16, 8}) {
      const size_t smem = cl_smem_bytes(G, cs, kClMaxSlots);
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        continue;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cs, 1, 1);
      cfg.blockDim = dim3(kAttnThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = cs;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int count = 0;
      if (cudaOccupancyMaxActiveClusters(&count, kern, &cfg) == cudaSuccess && count > 0) {
        best = cs;
        break;
      }
    }
  }
  cudaGetLastError();  // a refused query only selects the split + combine passes
  cache[dev] = best;
  return best > 0 ? best : 0;
}

template <int G>
cudaError_t launch_decode_cl(const float* qkv, __half* k_cache, __half* v_cache, int B, int H,
                             int Hkv, int S_max, int pos, const int* pos_dev, float scale,
                             int nsplit, int CS, float* out, cudaStream_t s, float theta_base) {
  const int slots = (nsplit + CS - 1) / CS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CS, Hkv, B);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = cl_smem_bytes(G, CS, slots);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = CS;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, k_attn_decode_cl<G>, qkv, k_cache, v_cache, H, Hkv, S_max, pos,
                            pos_dev, scale, nsplit, slots, out, theta_base);
}

}  // namespace

cudaError_t launch_rope_kv_append(const float* qkv, int B, int n, int H, int Hkv, int d, int pos,
                                  float theta_base, float* q_out, __half* k_cache,
                                  __half* v_cache, int S_max, cudaStream_t s, const int* pos_dev) {
  // Many rows (prefill chunks): the per-row form. Fewer rows (decode batches) keep
  // one thread per pair, whose short chains finish sooner than a row's loop.
  if (d / 2 <= kRopeRowMaxHalf && B * n >= num_sms_cached())
    return launch_pdl_attn(k_rope_kv_append_row, dim3(static_cast<unsigned>(B * n)), dim3(256), s,
                           qkv, n, H, Hkv, d, pos, pos_dev, theta_base, q_out, k_cache, v_cache,
                           S_max);
  const size_t total = static_cast<size_t>(B) * n * (H + 2 * Hkv) * (d / 2);
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  return launch_pdl_attn(k_rope_kv_append, dim3(blocks), dim3(256), s, qkv, n, H, Hkv, d, pos,
                         pos_dev, theta_base, total, q_out, k_cache, v_cache, S_max);
}

size_t attention_workspace_bytes(int B, int n, int H, int d, int seq_len) {
  const size_t nsplit = (static_cast<size_t>(seq_len) + kAttnChunk - 1) / kAttnChunk;
  return static_cast<size_t>(B) * n * H * nsplit * (d + 2) * sizeof(float);
}

namespace {
cudaError_t attention_impl(const float* q, const __half* k_cache, const __half* v_cache, int B,
                           int n, int H, int Hkv, int d, int S_max, int seq_len, float scale,
                           float* out, void* workspace, cudaStream_t s, const int* pos_dev,
                           bool rope, float theta_base) {
  if (d != kAttnHeadDim || Hkv <= 0 || H % Hkv != 0 || H / Hkv > kAttnMaxGroup)
    return cudaErrorInvalidValue;
  if (rope && n != 1) return cudaErrorInvalidValue;
  // With the position on the device the split count covers the whole cache; the
  // chunks past the visible keys write nothing and the combine skips them.
  const int nsplit = ((pos_dev ? S_max : seq_len) + kAttnChunk - 1) / kAttnChunk;
  const size_t rows = static_cast<size_t>(B) * n * H * nsplit;
  float* pa = static_cast<float*>(workspace);
  float* pm = pa + rows * d;
  float* pl = pm + rows;
  const int G = H / Hkv;
  // One clustered launch when the chunks fit the cluster's slots and the clusters
  // fit about two CTAs per SM; more sequences run the split + combine passes,
  // whose smaller CTAs fill the SMs beside the neighbouring matmuls better.
  if (rope) {
#define OBN_CL(GG)                                                                              \
  {                                                                                             \
    const int cs = decode_cluster_size<GG>();                                                   \
    if (cs > 0 && nsplit <= cs * kClMaxSlots && B * Hkv * cs <= 2 * num_sms_cached())           \
      return launch_decode_cl<GG>(q, const_cast<__half*>(k_cache), const_cast<__half*>(v_cache), \
                                  B, H, Hkv, S_max, seq_len - 1, pos_dev, scale, nsplit, cs, out, \
                                  s, theta_base);                                               \
  }
    switch (G) {
      case 1: OBN_CL(1) break;
      case 2: OBN_CL(2) break;
      case 4: OBN_CL(4) break;
      case 8: OBN_CL(8) break;
      default: return cudaErrorInvalidValue;
    }
#undef OBN_CL
  }
  cudaError_t e;
  // Prefill chunks: the 16-row tile pass, no combine (its q loads and output stores are
  // 8-byte pairs; other alignments run split + combine).
  if (!rope && n >= kFaMinRows && attn_fa_enabled() &&
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) % 8) == 0) {
    switch (G) {
      case 1: return launch_prefill_fa<1>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev, scale, out, s);
      case 2: return launch_prefill_fa<2>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev, scale, out, s);
      case 4: return launch_prefill_fa<4>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev, scale, out, s);
      case 8: return launch_prefill_fa<8>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev, scale, out, s);
      default: return cudaErrorInvalidValue;
    }
  }
  const bool pipe = !rope && attn_pipe_enabled() &&
                    reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
                    static_cast<long long>(B) * n * Hkv * nsplit >=
                        static_cast<long long>(kPipeMinItemsPerSm) * num_sms_cached();
#define OBN_SPLIT(GG)                                                                           \
  (pipe   ? launch_split_pipe<GG>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev,  \
                                  scale, nsplit, pa, pm, pl, s)                                 \
   : rope ? launch_split<GG, true>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev,  \
                                 scale, nsplit, pa, pm, pl, s, theta_base)                     \
        : launch_split<GG, false>(q, k_cache, v_cache, B, n, H, Hkv, S_max, seq_len, pos_dev, \
                                  scale, nsplit, pa, pm, pl, s, theta_base))
  switch (G) {
    case 1: e = OBN_SPLIT(1); break;
    case 2: e = OBN_SPLIT(2); break;
    case 4: e = OBN_SPLIT(4); break;
    case 8: e = OBN_SPLIT(8); break;
    default: return cudaErrorInvalidValue;
  }
#undef OBN_SPLIT
  if (e != cudaSuccess) return e;
  return launch_pdl_attn(k_attn_combine, dim3(static_cast<unsigned>(B * n * H)),
                         dim3(kAttnThreads), s, static_cast<const float*>(pa),
                         static_cast<const float*>(pm), static_cast<const float*>(pl), nsplit, n,
                         S_max, pos_dev, out);
}
}  // namespace

cudaError_t launch_attention(const float* q, const __half* k_cache, const __half* v_cache, int B,
                             int n, int H, int Hkv, int d, int S_max, int seq_len, float scale,
                             float* out, void* workspace, cudaStream_t s, const int* pos_dev) {
  return attention_impl(q, k_cache, v_cache, B, n, H, Hkv, d, S_max, seq_len, scale, out,
                        workspace, s, pos_dev, false, 0.0f);
}

cudaError_t launch_attention_rope(const float* qkv, __half* k_cache, __half* v_cache, int B, int H,
                                  int Hkv, int d, int S_max, int pos, float theta_base,
                                  float scale, float* out, void* workspace, cudaStream_t s,
                                  const int* pos_dev) {
  return attention_impl(qkv, k_cache, v_cache, B, 1, H, Hkv, d, S_max, pos + 1, scale, out,
                        workspace, s, pos_dev, true, theta_base);
}

}  // namespace obn
