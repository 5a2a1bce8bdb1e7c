/* oxbitnet.h — the model-level C ABI of the B200 build (libobn.so).
 *
 * Drop-in for the reference's FFI header
 * (packages/rust/crates/oxbitnet-ffi/oxbitnet.h, implemented in
 * oxbitnet-ffi/src/lib.rs): the same types, enumerators, struct layouts and
 * functions, so a program (or a Java / Swift / C# binding) built against the
 * reference's header links against libobn.so unchanged. Behaviour follows the
 * reference's: NULL-returning load with a thread-local error message, 0 / -1
 * from generate and chat, a token callback that stops generation by returning
 * non-zero, a process-wide logger installed once.
 *
 * Differences, all documented where they apply: models run on one CUDA device
 * (sm_100a) through the kernels of obn.h; URL sources are served only from the
 * download cache (there is no network client); sampling draws from a seedable
 * generator (oxbitnet_set_seed). The functions after the "extensions" marker
 * are additions of this build: generation from token ids, raw logits, and a
 * tokenizer that works without a GPU.
 */
#ifndef OXBITNET_H
#define OXBITNET_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define OXBITNET_API __attribute__((visibility("default")))
#else
#define OXBITNET_API
#endif

/* Phase reported to the load progress callback (oxbitnet.h:14-18). */
typedef enum OxBitNetLoadPhase {
  Download = 0,
  Parse = 1,
  Upload = 2,
} OxBitNetLoadPhase;

/* Level passed to the logger callback (oxbitnet.h:23-29). */
typedef enum OxBitNetLogLevel {
  Trace = 0,
  Debug = 1,
  Info = 2,
  Warn = 3,
  Error = 4,
} OxBitNetLogLevel;

/* A loaded model (opaque). */
typedef struct OxBitNet OxBitNet;

/* Logger callback: level, message bytes (NUL-terminated) and their length. */
typedef void (*OxBitNetLogFn)(enum OxBitNetLogLevel level, const char *message, uintptr_t len,
                              void *userdata);

/* Generation options (oxbitnet.h:47-68). Defaults: 256, 1.0, 50, 1.1, 64. */
typedef struct OxBitNetGenerateOptions {
  uintptr_t max_tokens;   /* tokens to generate at most */
  float temperature;      /* logits are multiplied by 1 / temperature */
  uintptr_t top_k;        /* keep the k largest logits (0 = all) */
  float repeat_penalty;   /* llama.cpp-style penalty on recently generated tokens */
  uintptr_t repeat_last_n; /* window of generated tokens the penalty looks at (0 = all) */
} OxBitNetGenerateOptions;

/* Load progress (oxbitnet.h:73-78). */
typedef struct OxBitNetLoadProgress {
  enum OxBitNetLoadPhase phase;
  uint64_t loaded;
  uint64_t total;
  double fraction;
} OxBitNetLoadProgress;

typedef void (*OxBitNetProgressFn)(const struct OxBitNetLoadProgress *progress, void *userdata);

/* Load options (oxbitnet.h:88-101). */
typedef struct OxBitNetLoadOptions {
  OxBitNetProgressFn on_progress; /* nullable */
  void *progress_userdata;        /* nullable */
  const char *cache_dir;          /* nullable; default $XDG_CACHE_HOME or ~/.cache, + "/.0xbitnet" */
} OxBitNetLoadOptions;

/* Token callback: the token's text (UTF-8, valid during the call) and its
 * length. Return 0 to continue, non-zero to stop. */
typedef int32_t (*OxBitNetTokenFn)(const char *token, uintptr_t len, void *userdata);

/* One chat message (oxbitnet.h:111-120). */
typedef struct OxBitNetChatMessage {
  const char *role;    /* "system", "user", "assistant", ... */
  const char *content;
} OxBitNetChatMessage;

/* Installs the logger (lib.rs:226-237). The first call installs the callback;
 * every call sets the minimum level (0 trace .. 4 error; larger values mean 4). */
OXBITNET_API void oxbitnet_set_logger(OxBitNetLogFn callback, void *userdata, uint8_t min_level);

/* {256, 1.0, 50, 1.1, 64} (lib.rs:243-252). */
OXBITNET_API struct OxBitNetGenerateOptions oxbitnet_default_generate_options(void);

/* No progress callback, no cache directory (lib.rs:255-262). */
OXBITNET_API struct OxBitNetLoadOptions oxbitnet_default_load_options(void);

/* Loads a GGUF model (BitNet b1.58, I2_S ternary weights) from a local path
 * (one that starts with '/' or '.', or has no "://") or, for a URL, from the
 * download cache (<cache_dir>/<sha256 of the URL in hex>). NULL on error; the
 * message is in oxbitnet_error_message(). The model lives on the current CUDA
 * device. */
OXBITNET_API struct OxBitNet *oxbitnet_load(const char *source,
                                            const struct OxBitNetLoadOptions *options);

/* Frees a model and its device memory; NULL is a no-op. */
OXBITNET_API void oxbitnet_free(struct OxBitNet *model);

/* Encodes `prompt` (BOS first), clears the KV cache, prefills, then samples up
 * to max_tokens tokens, stopping at EOS, <|eot_id|> or <|im_end|>; each token's
 * text goes to `callback` (NULL: generate silently). options NULL = defaults.
 * 0 on success, -1 on error. */
OXBITNET_API int32_t oxbitnet_generate(struct OxBitNet *model, const char *prompt,
                                       const struct OxBitNetGenerateOptions *options,
                                       OxBitNetTokenFn callback, void *userdata);

/* As oxbitnet_generate over the chat template of `messages` (ChatML, LLaMA 3
 * headers, or the contents joined by newlines, whichever the vocabulary has). */
OXBITNET_API int32_t oxbitnet_chat(struct OxBitNet *model,
                                   const struct OxBitNetChatMessage *messages,
                                   uintptr_t num_messages,
                                   const struct OxBitNetGenerateOptions *options,
                                   OxBitNetTokenFn callback, void *userdata);

/* The last error on this thread, or NULL. Valid until the next call on this thread. */
OXBITNET_API const char *oxbitnet_error_message(void);

/* ---- extensions of this build ---------------------------------------------- */

/* Token callback with the id. */
typedef int32_t (*OxBitNetTokenIdFn)(uint32_t id, const char *token, uintptr_t len,
                                     void *userdata);

/* Model dimensions. */
typedef struct OxBitNetModelInfo {
  uint32_t vocab_size, hidden_size, intermediate_size, num_layers, num_heads, num_kv_heads,
      head_dim, max_seq_len, position;
  float rms_norm_eps, rope_theta;
  int32_t tied_embeddings, lm_head_f16, gated_ffn, activation; /* activation: 0 ReLU^2, 1 SiLU */
} OxBitNetModelInfo;

/* Generation from token ids (no BOS is added): as oxbitnet_generate after encoding. */
OXBITNET_API int32_t oxbitnet_generate_ids(struct OxBitNet *model, const uint32_t *ids,
                                           uintptr_t n, const struct OxBitNetGenerateOptions *options,
                                           OxBitNetTokenIdFn callback, void *userdata);

/* Reseeds the model's sampler. */
OXBITNET_API int32_t oxbitnet_set_seed(struct OxBitNet *model, uint64_t seed);

/* Runs n tokens at the current position (after clearing the KV cache if `reset`)
 * and copies the last token's logits [vocab] to host memory `logits` (nullable). */
OXBITNET_API int32_t oxbitnet_forward(struct OxBitNet *model, const uint32_t *ids, uintptr_t n,
                                      int32_t reset, float *logits, uintptr_t vocab);

OXBITNET_API int32_t oxbitnet_model_info(const struct OxBitNet *model,
                                         struct OxBitNetModelInfo *info);

/* Tokenizer of a GGUF file, without a GPU (opaque). */
typedef struct OxBitNetTokenizer OxBitNetTokenizer;

OXBITNET_API struct OxBitNetTokenizer *oxbitnet_tokenizer_load(const char *path);
OXBITNET_API void oxbitnet_tokenizer_free(struct OxBitNetTokenizer *tok);
/* Writes up to `cap` ids and the full count to *n_ids (0 / -1). */
OXBITNET_API int32_t oxbitnet_tokenize(const struct OxBitNetTokenizer *tok, const char *text,
                                       int32_t add_bos, uint32_t *ids, uintptr_t cap,
                                       uintptr_t *n_ids);
OXBITNET_API int32_t oxbitnet_chat_template(const struct OxBitNetTokenizer *tok,
                                            const struct OxBitNetChatMessage *messages,
                                            uintptr_t num_messages, uint32_t *ids, uintptr_t cap,
                                            uintptr_t *n_ids);
/* Decodes ids (BOS / EOS dropped) into buf (NUL-terminated when it fits); *len =
 * the full byte length. */
OXBITNET_API int32_t oxbitnet_detokenize(const struct OxBitNetTokenizer *tok, const uint32_t *ids,
                                         uintptr_t n, char *buf, uintptr_t cap, uintptr_t *len);
/* The text one generated token streams as. */
OXBITNET_API int32_t oxbitnet_token_text(const struct OxBitNetTokenizer *tok, uint32_t id,
                                         char *buf, uintptr_t cap, uintptr_t *len);

/* Samples the next token from the logits of the model's last forward with the
 * uniform draw `u`, as generation does (penalty, temperature and top-k on the
 * device, the draw on the host). The penalty modifies the device logits. */
OXBITNET_API int32_t oxbitnet_sample_next(struct OxBitNet *model, float temperature,
                                          uintptr_t top_k, float repeat_penalty,
                                          const uint32_t *recent, uintptr_t n_recent, float u,
                                          uint32_t *out);

/* One sampling step with the uniform draw `u` in [0, 1) given (logits are
 * modified); returns the id. */
OXBITNET_API uint32_t oxbitnet_sample(float *logits, uintptr_t vocab, float temperature,
                                      uintptr_t top_k, float repeat_penalty,
                                      const uint32_t *recent, uintptr_t n_recent, float u);

/* A JSON summary of a GGUF file's header, config and tensor table (library-owned,
 * valid until the next call on this thread), or NULL on error. */
OXBITNET_API const char *oxbitnet_gguf_describe(const char *path);

/* Where oxbitnet_load looks for a URL source: writes the path into buf. */
OXBITNET_API int32_t oxbitnet_cache_path(const char *source, const char *cache_dir, char *buf,
                                         uintptr_t cap);

#ifdef __cplusplus
}
#endif

#endif /* OXBITNET_H */
