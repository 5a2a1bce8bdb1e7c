// attention.h — decode attention next to the BitLinear path (attention.cu):
// RoPE + fp16 KV-cache append, and split-KV ("flash-decode") GQA attention.
#pragma once

#include <cstddef>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace obn {

constexpr int kAttnHeadDim = 128;  // head_dim the kernels are built for
constexpr int kAttnChunk = 128;    // keys per split
constexpr int kAttnMaxGroup = 8;   // query heads per KV head

// qkv [B*n, (H + 2*Hkv) * d] f32 (the merged QKV projection output: q heads,
// then k heads, then v heads). Rotates q and k of token t of sequence b at
// position pos + t (rope.wgsl), writes q_out [B*n, H*d] f32, and stores the
// rotated k and the v of that token into the caches [B][S_max][Hkv][d] (binary16)
// at position pos + t. A non-null pos_dev replaces pos by the int it points to
// (read on the device, so a captured graph serves every position).
cudaError_t launch_rope_kv_append(const float* qkv, int B, int n, int H, int Hkv, int d, int pos,
                                  float theta_base, float* q_out, __half* k_cache,
                                  __half* v_cache, int S_max, cudaStream_t s,
                                  const int* pos_dev = nullptr);

// Scratch of launch_attention: per (query row, head, split) the partial
// softmax state (max, sum, d unnormalised outputs), f32.
size_t attention_workspace_bytes(int B, int n, int H, int d, int seq_len);

// Causal GQA attention for the n newest tokens of B sequences whose caches hold
// seq_len positions (the n new ones last): q [B*n, H*d] f32 -> out [B*n, H*d].
// A non-null pos_dev makes the visible length *pos_dev + n (read on the device);
// the workspace must then hold attention_workspace_bytes(B, n, H, d, S_max).
cudaError_t launch_attention(const float* q, const __half* k_cache, const __half* v_cache, int B,
                             int n, int H, int Hkv, int d, int S_max, int seq_len, float scale,
                             float* out, void* workspace, cudaStream_t s,
                             const int* pos_dev = nullptr);

// One decode token per sequence (n = 1) with the RoPE + KV append fused in:
// qkv [B, (H + 2*Hkv) * d] is the merged QKV projection output (unrotated); the
// new token sits at position pos (or *pos_dev), its rotated key and its value
// are stored into the caches, and out [B, H*d] is the attention of the rotated
// q over positions [0, pos]. Equal, bit for bit, to launch_rope_kv_append
// followed by launch_attention. Workspace as launch_attention with n = 1 and
// seq_len = pos + 1 (S_max when pos_dev is given).
cudaError_t launch_attention_rope(const float* qkv, __half* k_cache, __half* v_cache, int B, int H,
                                  int Hkv, int d, int S_max, int pos, float theta_base,
                                  float scale, float* out, void* workspace, cudaStream_t s,
                                  const int* pos_dev = nullptr);

}  // namespace obn
