/*
 * obn.h — C ABI of the B200-native ternary BitLinear path (libobn.so).
 *
 * Replaces the wgpu dispatches of 0xBitNet's BitLinear layer:
 *   BitLinear::new / BitLinear::forward
 *     packages/rust/crates/oxbitnet/src/nn/bitlinear.rs:31-97
 *     packages/core/src/nn/bitlinear.ts:47-169 (exported via packages/core/src/internals.ts:33)
 *   the I2_S upload + per-row scale extraction
 *     packages/rust/crates/oxbitnet/src/model/loader.rs:105-137
 *   and the four shaders they dispatch
 *     packages/core/src/shaders/{rmsnorm,quantize,ternary_gemv,ternary_gemm}.wgsl
 *
 * Conventions (those of the reference's C ABI, packages/rust/crates/oxbitnet-ffi):
 *   - every entry point returns OBN_OK (0) or a negative status; the message of
 *     the last failure on the calling thread is returned by obn_error_message()
 *     (thread-local, library-owned, valid until the next obn_* call on that
 *     thread; cf. oxbitnet-ffi/src/lib.rs:31-46, 528-541);
 *   - device pointers are caller-owned CUDA device memory; `stream` is a
 *     cudaStream_t passed as void* (NULL = the legacy default stream);
 *   - every compute entry point is stream-ordered and does not synchronise.
 *
 * Data formats:
 *   - activations x: float32 [n, in_dim], row-major;
 *   - quantized activations q: int8 [n, in_dim] (the reference stores the same
 *     values as i32, quantize.wgsl:74); per-token scales float32 [n];
 *     per-token code sums int32 [n] (sum_k q[t,k], used by the kernels to turn
 *     2-bit codes c in {0,1,2} into weights c-1 exactly);
 *   - weights: I2_S rows of in_dim/4 bytes (128-element blocks of 32 bytes,
 *     byte gp holding elements gp, 32+gp, 64+gp, 96+gp in bits 7:6..1:0, code
 *     c meaning weight c-1), in_dim % 128 == 0;
 *   - outputs y: float32 [n, out_dim], token-major (ternary_gemm.wgsl:133).
 */
#ifndef OBN_H
#define OBN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define OBN_API __attribute__((visibility("default")))
#else
#define OBN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define OBN_OK 0
#define OBN_ERR_INVALID_ARGUMENT -1  /* null pointer, bad size, misaligned buffer */
#define OBN_ERR_UNSUPPORTED -2       /* shape outside what the kernels handle */
#define OBN_ERR_CUDA -3              /* a CUDA runtime call failed */
#define OBN_ERR_OUT_OF_MEMORY -4
#define OBN_ERR_DEVICE_TIMEOUT -5    /* a bounded device-side wait gave up */
#define OBN_ERR_NO_DEVICE -6         /* no CUDA device, or not sm_100 */

typedef struct obn_bitlinear obn_bitlinear;

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
OBN_API int obn_version(void);

/* Last error on this thread, or NULL. Mirrors oxbitnet_error_message
 * (oxbitnet-ffi/oxbitnet.h:218-224). */
OBN_API const char* obn_error_message(void);

/* ---- layer lifecycle ------------------------------------------------------ */

/* Loads one GGUF I2_S tensor from host memory: `i2s_tensor` holds
 * out_dim*in_dim/4 packed bytes followed by 32 bytes whose first float32 is the
 * per-tensor scale (loader.rs:105-137; GGUF ne[0]=in_dim, ne[1]=out_dim).
 * The scale is replicated into a per-row [out_dim] table as the reference does
 * (loader.rs:129-137). `norm_weight` (host, nullable) is the optional [in_dim]
 * RMSNorm gamma applied before quantization (bitlinear.rs:61-71), `eps` its
 * epsilon (the reference hard-codes 1e-5, bitlinear.rs:112). The weights are
 * repacked into the device layout on `device`. */
OBN_API int obn_bitlinear_load_i2s(const uint8_t* i2s_tensor, size_t nbytes, int in_dim, int out_dim,
                           const float* norm_weight, float eps, int device,
                           obn_bitlinear** out_layer);

/* The gated FFN's gate and up projections merged into one layer
 * (FFN::forward_gated, ffn.rs:70-79: gate_proj and up_proj on the same input,
 * then activation.wgsl ReLU^2 on gate and elementwise.wgsl multiply by up).
 * gate_i2s / up_i2s are the two GGUF I2_S tensors ([out_dim, in_dim] each plus
 * their 32-byte scale trailers), sharing norm_weight and eps. The layer's
 * forward quantizes the input once, runs one matmul over the 2 * out_dim
 * interleaved weight rows (row 2i = gate row i, row 2i + 1 = up row i) and
 * writes y[t, i] = (r * r) * up[t, i] with r = max(0, gate[t, i]): [n, out_dim].
 * obn_ternary_matmul / obn_ternary_acc / obn_bitlinear_export_i2s on such a
 * layer work on the interleaved rows (obn_bitlinear_rows(layer) of them). */
OBN_API int obn_bitlinear_load_i2s_gated(const uint8_t* gate_i2s, size_t gate_bytes,
                                         const uint8_t* up_i2s, size_t up_bytes, int in_dim,
                                         int out_dim, const float* norm_weight, float eps,
                                         int device, obn_bitlinear** out_layer);

/* Several GGUF I2_S tensors that read the same input, stacked into one layer
 * (the merged q|k|v projection: Attention::forward, attention.rs:98-100, runs
 * three BitLinears on one normed input). Tensor t contributes out_dims[t] rows
 * scaled by its own per-tensor scale (loader.rs:129-137), so the output row
 * r of the layer equals row r - (rows before t) of tensor t's BitLinear.
 * out_dim of the layer = the sum of out_dims. */
OBN_API int obn_bitlinear_load_i2s_concat(int count, const uint8_t* const* tensors,
                                          const size_t* nbytes, const int* out_dims, int in_dim,
                                          const float* norm_weight, float eps, int device,
                                          obn_bitlinear** out_layer);

/* The activation of a gated layer's gate half: 0 = ReLU^2 (the default; bitnet-25
 * models), 1 = SiLU x / (1 + exp(-x)) (other architectures; activation.wgsl:28-33,
 * ffn.rs:64-80). */
OBN_API int obn_bitlinear_set_activation(obn_bitlinear* layer, int act);

/* activation.wgsl alone: y[i] = act(x[i]) for i < count, act as above (y may alias x).
 * FFN::forward_simple (ffn.rs:82-92) applies it to up_proj's output. */
OBN_API int obn_activation(const float* x, size_t count, int act, float* y, void* stream);

/* BitLinear::new(device, packed_weights, weight_scales, norm_weight, in_dim,
 * out_dim) (bitlinear.rs:31-49) over buffers already on the device in the
 * reference's layout: packed [out_dim, in_dim/16] u32, per-row scales
 * [out_dim] f32, norm [in_dim] f32 or NULL. The data is copied (repacked) into
 * library-owned memory on the current device, ordered on `stream`. */
OBN_API int obn_bitlinear_create(const void* packed_dev, const float* scales_dev, const float* norm_dev,
                         float eps, int in_dim, int out_dim, void* stream,
                         obn_bitlinear** out_layer);

/* Frees a layer; NULL is a no-op (oxbitnet-ffi/src/lib.rs:367-376). */
OBN_API void obn_bitlinear_free(obn_bitlinear* layer);

/* Shape queries. */
OBN_API int obn_bitlinear_in_dim(const obn_bitlinear* layer);
/* obn_bitlinear_load_i2s_gated over device buffers, as obn_bitlinear_create is
 * BitLinear::new over device buffers: gate / up packed I2_S rows [out_dim, in_dim/4]
 * and their row scales [out_dim]. Synchronises `stream` before returning. */
OBN_API int obn_bitlinear_create_gated(const void* gate_packed_dev, const float* gate_scales_dev,
                                       const void* up_packed_dev, const float* up_scales_dev,
                                       const float* norm_dev, float eps, int in_dim, int out_dim,
                                       void* stream, obn_bitlinear** out_layer);
OBN_API int obn_bitlinear_out_dim(const obn_bitlinear* layer);
/* Weight rows the matmul entry points compute: out_dim, or 2 * out_dim for a
 * gated layer. */
OBN_API int obn_bitlinear_rows(const obn_bitlinear* layer);

/* Device scratch that obn_bitlinear_forward needs for n tokens (bytes). */
OBN_API size_t obn_bitlinear_workspace_bytes(const obn_bitlinear* layer, int n);

/* BitLinear::forward(input, n) (bitlinear.rs:52-97; bitlinear.ts:117-169):
 * optional RMSNorm -> per-token absmax int8 quantize -> ternary GEMV (n == 1)
 * or GEMM (n > 1) -> y[n, out_dim]. `workspace` (device, 256-byte aligned) must
 * hold obn_bitlinear_workspace_bytes(layer, n) bytes and must not be used by
 * other work in flight. The epilogue rounds like the reference: n == 1 gives
 * (f32(acc) * s_w) * s_x (ternary_gemv.wgsl:95), n > 1 gives
 * f32(acc) * (s_w * s_x) (ternary_gemm.wgsl:132-133). */
OBN_API int obn_bitlinear_forward(const obn_bitlinear* layer, const float* x, int n, float* y,
                          void* workspace, size_t workspace_bytes, void* stream);

/* BitLinear::forward followed by the residual add the reference dispatches after
 * o_proj and down_proj (TransformerBlock::forward, transformer.rs:63,69;
 * elementwise.wgsl op 0): y[t, m] = y[t, m] + forward(x)[t, m], the sum rounded
 * once, in the matmul's epilogue (no separate add kernel). y must not alias x.
 * Not for gated layers. Same workspace as obn_bitlinear_forward. */
OBN_API int obn_bitlinear_forward_residual(const obn_bitlinear* layer, const float* x, int n,
                                           float* y, void* workspace, size_t workspace_bytes,
                                           void* stream);

/* No counterpart in the reference. obn_bitlinear_forward for callers that cannot
 * allocate device memory: hosts whose device memory is reserved up front by
 * another allocator, and latency-critical threads that must not call
 * cudaMalloc/cudaFree (they can block and synchronise the device). The scratch
 * obn_bitlinear_forward takes as `workspace` lives instead in one fixed device
 * array of 1 MiB + 32 KiB that every device loading the library holds until the
 * process exits; the call allocates nothing. Limits: n * in_dim <= 1048576 and
 * n <= 4096 (and obn_bitlinear_workspace_bytes(layer, n) <= 1 MiB + 32 KiB, which
 * those two imply for every layer whose matmul runs on the tensor cores or the
 * warp MMA); otherwise OBN_ERR_UNSUPPORTED with a message naming the sizes.
 * The first call on a device looks the array's device address up (once per
 * device, with that device current); make that first call before any stream
 * capture. The address is kept for the life of the process, so a device reset
 * (cudaDeviceReset) after that first call is not supported. All calls on a
 * device share the array and it keeps the previous
 * call's contents (nothing in it needs to start at zero: every byte read is
 * first written by the same call); calls that overlap on the GPU race on it. */
OBN_API int obn_bitlinear_forward_noalloc(const obn_bitlinear* layer, const float* x, int n,
                                          float* y, void* stream);

/* Tensor-parallel BitLinear::forward (bitlinear.rs:52-97) with the output
 * features split over `world` ranks (one GPU each) and the result gathered on
 * every rank, in one kernel per rank: `layer` holds the contiguous row block
 * [col0, col0 + out_dim) of an out_total-row weight; this call computes the
 * [n, out_dim] slice and its GEMM epilogue writes it straight into columns
 * [col0, col0 + out_dim) of the [n, out_total] f32 output that every rank holds:
 *   y_mc != NULL  a multicast (NVLS) device address bound to every rank's output
 *                 buffer: one store per element reaches all of them through the
 *                 NVSwitch;
 *   y_mc == NULL  y_ranks (host array of `world` device pointers) gives each
 *                 rank's output buffer as mapped on this device (this rank's own
 *                 buffer and peer mappings of the others): one store per rank.
 * Needs n >= 16 (the tensor-core GEMM; OBN_ERR_UNSUPPORTED otherwise) and
 * world <= 8. Stream-ordered: before reading its output a rank must order
 * every rank's call before the read (for instance a barrier on the stream).
 * Numerics are those of obn_bitlinear_forward for the same rows. */
OBN_API int obn_bitlinear_forward_tp(const obn_bitlinear* layer, const float* x, int n,
                                     float* y_mc, float* const* y_ranks, int world,
                                     int out_total, int col0, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* The f16 LM head behind the final RMSNorm: dispatch_final_norm + dispatch_lm_head_with
 * (model.rs:226-262, 393-430) running rmsnorm.wgsl then f32_matmul.wgsl:27-74 (tied
 * embedding or separate f16 head): logits[t, v] = sum_d y[t, d] * f32(embed[v, d]) for
 * t < n, v < vocab, with y = RMSNorm(x[t]) * norm_weight (norm_weight NULL: y = x[t]).
 * embed: [vocab, dim] IEEE binary16, row-major, 16-byte aligned; dim % 8 == 0 and
 * dim <= 14336. x: [n, dim] f32 (16-byte aligned); logits: [n, vocab] f32. Every logit is
 * the shader's: 256 lane partials over d-pairs, then its halving tree, in f32. The
 * reference calls it with the last token only (n = 1); n > 1 streams the table once per
 * 4 tokens. Stream-ordered, no workspace. */
OBN_API int obn_lm_head_f16(const void* embed, int vocab, int dim, const float* x,
                            const float* norm_weight, float eps, int n, float* logits,
                            void* stream);

/* obn_lm_head_f16 for batches of tokens on the tensor cores: the same logits with
 * the hidden rows split into binary16 hi + lo halves (y = hi + lo to 2^-22 |y|) and
 * f32 accumulation in the tensor core's order instead of the shader's 256-lane tree
 * (differences at the 1e-6 relative level; the reference itself only runs n = 1).
 * dim % 64 == 0. workspace (256-byte aligned) holds obn_lm_head_workspace_bytes(n, dim)
 * bytes. */
OBN_API size_t obn_lm_head_workspace_bytes(int n, int dim);
OBN_API int obn_lm_head_f16_batched(const void* embed, int vocab, int dim, const float* x,
                                    const float* norm_weight, float eps, int n, float* logits,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* ---- decode attention around the BitLinear path ----------------------------- */
/* RoPE + KV-cache append (attention.rs:98-104: apply_rope on q and k, then
 * append_to_cache; rope.wgsl). qkv: [B*n, (H + 2*Hkv) * head_dim] f32, the merged QKV
 * projection output of n new tokens of each of B sequences (q heads, then k heads,
 * then v heads). Token t of a sequence sits at position pos + t. Writes q_out
 * [B*n, H * head_dim] f32 (rotated) and stores the rotated k and the v of each new
 * token into the caches k_cache / v_cache [B][S_max][Hkv][head_dim] (IEEE binary16,
 * 16-byte aligned; the reference keeps f32). Needs head_dim == 128, pos + n <= S_max. */
OBN_API int obn_rope_kv_append(const float* qkv, int B, int n, int H, int Hkv, int head_dim,
                               int pos, float theta_base, float* q_out, void* k_cache,
                               void* v_cache, int S_max, void* stream);

/* Scratch bytes of obn_attention_decode for these sizes. */
OBN_API size_t obn_attention_workspace_bytes(int B, int n, int H, int head_dim, int seq_len);

/* Causal GQA attention of the n newest tokens of B sequences (attention.rs:106-121:
 * compute_scores, softmax, compute_attn_v; attention.wgsl, softmax.wgsl): the caches
 * hold seq_len positions per sequence, the n new ones last; query t attends to keys
 * [0, seq_len - n + t]. q [B*n, H * head_dim] f32 -> out [B*n, H * head_dim] f32,
 * scale = the score scale (the reference uses 1 / sqrt(head_dim)). Split-KV (128-key
 * chunks) with a combine pass; the workspace (256-byte aligned) holds
 * obn_attention_workspace_bytes(...) bytes. Needs head_dim == 128 and H / Hkv in
 * {1, 2, 4, 8}. */
OBN_API int obn_attention_decode(const float* q, const void* k_cache, const void* v_cache, int B,
                                 int n, int H, int Hkv, int head_dim, int S_max, int seq_len,
                                 float scale, float* out, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* obn_rope_kv_append / obn_attention_decode with the position in device memory:
 * `pos_dev` points to the int position of the first new token (the caches then
 * hold *pos_dev + n positions after the append), read by the kernels, so one
 * captured CUDA graph serves every decode step. A position with pos + n > S_max
 * writes nothing and sees at most S_max keys. The attention workspace must hold
 * obn_attention_workspace_bytes(B, n, H, head_dim, S_max) bytes. */
OBN_API int obn_rope_kv_append_at(const float* qkv, int B, int n, int H, int Hkv, int head_dim,
                                  const int* pos_dev, float theta_base, float* q_out,
                                  void* k_cache, void* v_cache, int S_max, void* stream);
OBN_API int obn_attention_decode_at(const float* q, const void* k_cache, const void* v_cache,
                                    int B, int n, int H, int Hkv, int head_dim, int S_max,
                                    const int* pos_dev, float scale, float* out, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* One decode token per sequence with RoPE + KV append fused into the attention:
 * qkv [B, (H + 2*Hkv) * head_dim] f32 is the merged QKV projection output (q, k, v
 * unrotated); the token sits at position pos (the _at form reads it from pos_dev),
 * its rotated key and its value are stored into the caches at that position and
 * out [B, H * head_dim] is its attention over positions [0, pos]. Bit-identical to
 * obn_rope_kv_append followed by obn_attention_decode (n = 1) and one launch fewer.
 * Workspace: obn_attention_workspace_bytes(B, 1, H, head_dim, pos + 1), or with
 * S_max in place of pos + 1 for the _at form (one and two sequences use none of it).
 * The cache rows below pos - 1 are read while the kernel before this call may still
 * run: the rows a decode sequence reads were appended by earlier calls (row pos - 1
 * is read after that kernel ends). A caller that moves forward on one cache by more
 * than one position must write the rows in between (obn_rope_kv_append or its own
 * copy) before this call. */
OBN_API int obn_attention_decode_rope(const float* qkv, void* k_cache, void* v_cache, int B, int H,
                                      int Hkv, int head_dim, int S_max, int pos, float theta_base,
                                      float scale, float* out, void* workspace,
                                      size_t workspace_bytes, void* stream);
OBN_API int obn_attention_decode_rope_at(const float* qkv, void* k_cache, void* v_cache, int B,
                                         int H, int Hkv, int head_dim, int S_max,
                                         const int* pos_dev, float theta_base, float scale,
                                         float* out, void* workspace, size_t workspace_bytes,
                                         void* stream);

/* ---- decoder glue ------------------------------------------------------------- */
/* Residual add (elementwise.wgsl op 0, TransformerBlock::forward's dispatch_add,
 * transformer.rs:63,69): y[i] = a[i] + b[i] for i < count (f32; y may alias a or b). */
OBN_API int obn_add(const float* a, const float* b, size_t count, float* y, void* stream);

/* Token embedding lookup (embedding.wgsl): y[t, :] = f32(table[ids[t], :]) for t < n;
 * ids outside [0, vocab) give zero rows. table [vocab, dim] binary16; ids int32 (device). */
OBN_API int obn_embed_f16(const void* table, int vocab, int dim, const int32_t* ids, int n,
                          float* y, void* stream);

/* ---- kernel-level entry points (one per reference shader) ------------------ */

/* Fused rmsnorm.wgsl + quantize.wgsl: per token, optional RMSNorm with gamma
 * `norm_weight` (NULL: none), then absmax int8 quantization. Writes q [n, d],
 * scales [n] and code sums qsum [n] (nullable). d % 4 == 0. */
OBN_API int obn_rmsnorm_quantize(const float* x, const float* norm_weight, float eps, int n, int d,
                         int8_t* q, float* scales, int32_t* qsum, void* stream);

/* rmsnorm.wgsl alone: y[n, d] = (x * rms) * w. */
OBN_API int obn_rmsnorm(const float* x, const float* w, float eps, int n, int d, float* y,
                void* stream);

/* ternary_gemv.wgsl / ternary_gemm.wgsl on already-quantized activations,
 * with the layer's weights: y[t, m] for t < n. `qsum` as written by
 * obn_rmsnorm_quantize. n == 1 rounds like the GEMV shader, n > 1 like the
 * GEMM shader. */
OBN_API int obn_ternary_matmul(const obn_bitlinear* layer, const int8_t* q, const float* scales,
                       const int32_t* qsum, int n, float* y, void* stream);

/* The exact int32 accumulators acc[t, m] = sum_k w[m,k] * q[t,k] (no scaling),
 * for bit-exact checks of the integer core. */
OBN_API int obn_ternary_acc(const obn_bitlinear* layer, const int8_t* q, const int32_t* qsum, int n,
                    int32_t* acc, void* stream);

/* Copies the layer's device weights back out in the reference's I2_S row
 * layout [out_dim, in_dim/4] bytes (device destination), for round-trip
 * checks of the repack. */
OBN_API int obn_bitlinear_export_i2s(const obn_bitlinear* layer, uint8_t* dst_dev, void* stream);

/* Reads (and clears) the device error word that bounded in-kernel waits set
 * when they give up; returns OBN_OK or OBN_ERR_DEVICE_TIMEOUT. Synchronises
 * the current device. */
OBN_API int obn_check_device_errors(void);

/* ---- measurement --------------------------------------------------------------
 * No counterpart in the reference. Multiply-accumulate rate of one integer MMA form,
 * as MACs per cycle per SM (one CTA per SM, back-to-back operations, slowest SM):
 * form 0 tcgen05.mma kind::i8 (M = 128, K = 32, A in tensor memory, N = n),
 * form 1 the same with A in shared memory, form 2 mma.sync m16n8k32 u8 x s8,
 * form 3 dp4a. `count` operations per issuing thread (1 .. 65536). The numbers
 * decide which kernel serves which token count (a flat tcgen05 cost per MMA up to
 * N = 256 favours the warp MMA at decode widths). Synchronises the device. */
OBN_API int obn_measure_mma_rate(int form, int n, int count, double* macs_per_cycle_per_sm);

#ifdef __cplusplus
}
#endif
#endif /* OBN_H */
