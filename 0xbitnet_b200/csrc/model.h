// model.h — a BitNet b1.58 model from a GGUF file, run on libobn's kernels.
//
// The host-side runtime behind the oxbitnet_* C ABI (oxbitnet.cpp). It mirrors
// the reference's model stack (packages/rust/crates/oxbitnet/src/):
//   model/loader.rs:78-171, 214-313   GGUF -> config + device weights
//   nn/model.rs:44-262                embedding -> N blocks -> final norm -> LM head
//   nn/transformer.rs:51-72           x += attn(norm(x)); x += ffn(norm(x))
//   nn/attention.rs:85-124            q|k|v, RoPE, KV append, causal GQA, o_proj
//   nn/ffn.rs:58-92                   gated (ReLU^2 or SiLU) or plain FFN
//   lib.rs:125-185                    prefill, then one token per step with sampling
// B200 form: q|k|v are one BitLinear (per-row scales) and gate|up one gated
// layer; the block RMSNorms are fused into the BitLinear that consumes them;
// the residual adds happen in the o_proj / down_proj epilogues; the KV cache is
// binary16; the LM head runs on the last position only, as the reference's does.
// Prompts are prefilled in chunks of up to kChunk tokens (never a 1-token chunk
// unless the whole input is one token, so every prompt token takes the
// reference's n > 1 GEMM order).
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "bpe.h"
#include "sampler.h"

struct obn_bitlinear;

namespace obn {

namespace gguf {
struct File;
}

enum class Activation { kRelu2 = 0, kSilu = 1 };

// ModelConfig (model/config.rs:3-17), read as config_from_gguf_metadata does
// (loader.rs:246-313).
struct ModelConfig {
  std::string arch;
  int vocab = 0, hidden = 0, ffn = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0;
  int context_length = 0;
  float eps = 1e-5f, rope_theta = 10000.0f;
  bool tied = true;        // no output.weight tensor
  bool lm_head_f16 = false;
  bool gated = true;       // blk.*.ffn_gate.weight present
  Activation act = Activation::kRelu2;
};

// Reads the config from GGUF metadata; empty string on success.
std::string config_from_gguf(const gguf::File& f, ModelConfig* cfg);

// loader.rs:215-244: GGUF tensor names -> the HF names the reference uses.
std::string hf_name(const std::string& gguf_name);

using ProgressFn = std::function<void(int phase, uint64_t loaded, uint64_t total, double fraction)>;
using LogFn = std::function<void(int level, const std::string& message)>;  // 0 trace .. 4 error

class Model {
 public:
  static constexpr int kMaxSeq = 4096;  // BitNet::load builds with max_seq_len 4096 (lib.rs:82-88)
  static constexpr int kChunk = 512;    // prefill tokens per pass

  ~Model();
  // Builds the model from GGUF bytes [0, size) (which must stay valid during the
  // call) on the current CUDA device. Empty string on success.
  static std::string load(const uint8_t* data, size_t size, const ProgressFn& progress,
                          const LogFn& log, std::unique_ptr<Model>* out);

  // BitNetModel::forward (model.rs:200-262): runs `n` tokens at the current
  // position, appends them to the KV cache and leaves the logits of the last
  // one in logits() (host). Empty string on success.
  std::string forward(const uint32_t* ids, int n, bool copy_logits = true);
  // Next token from the logits of the last forward (sampling.rs:4-77 with the
  // uniform draw u): the penalty, temperature and top-k cut run on the device
  // and only the survivors come to the host, which draws in the reference's
  // order; top_k = 0 or >= vocab takes the whole-vocabulary host path.
  std::string sample(float temperature, size_t top_k, float repeat_penalty,
                     const uint32_t* recent, size_t n_recent, float u, uint32_t* out);
  // BitNetModel::reset_kv_cache (model.rs:305-316).
  void reset() { pos_ = 0; }
  int position() const { return pos_; }

  const float* logits() const { return logits_h_; }
  const ModelConfig& config() const { return cfg_; }
  const BpeTokenizer& tokenizer() const { return tok_; }
  bool has_tokenizer() const { return has_tok_; }
  Sampler& sampler() { return sampler_; }

 private:
  Model() = default;
  std::string build(const gguf::File& f, const uint8_t* data, size_t size,
                    const ProgressFn& progress, const LogFn& log);
  std::string run_chunk(const uint32_t* ids, int n, bool want_logits, bool copy_logits);
  std::string enqueue(int n, const int32_t* ids_dev, const int* pos_dev, bool want_logits);
  std::string enqueue_part(int n, const int32_t* ids_dev, const int* pos_dev, bool want_logits,
                           int first, int last);
  std::string logits_to_host();

  struct Layer {
    obn_bitlinear* qkv = nullptr;     // q|k|v, input_layernorm fused
    obn_bitlinear* o = nullptr;       // attn_sub_norm fused (if present)
    obn_bitlinear* ffn_in = nullptr;  // gate|up (gated) or up, post_attention_layernorm fused
    obn_bitlinear* down = nullptr;    // ffn_sub_norm fused (if present)
  };

  ModelConfig cfg_;
  BpeTokenizer tok_;
  bool has_tok_ = false;
  Sampler sampler_;
  int device_ = 0;
  int pos_ = 0;
  void* stream_ = nullptr;  // cudaStream_t
  std::vector<Layer> layers_;
  void* embed_ = nullptr;          // [vocab][hidden] binary16
  void* lm_f16_ = nullptr;         // untied binary16 head, or null
  obn_bitlinear* lm_ternary_ = nullptr;
  float* final_norm_ = nullptr;    // [hidden]
  std::vector<void*> k_cache_, v_cache_;  // per layer [kMaxSeq][kv_heads][head_dim] binary16
  float *x_ = nullptr, *qkv_ = nullptr, *q_ = nullptr, *attn_ = nullptr, *ffn_ = nullptr;
  float *lm_in_ = nullptr, *logits_d_ = nullptr;
  int32_t* ids_d_ = nullptr;
  void* ws_ = nullptr;
  size_t ws_bytes_ = 0;
  void* attn_ws_ = nullptr;
  size_t attn_ws_bytes_ = 0;
  float* logits_h_ = nullptr;  // pinned [vocab]
  int32_t* ids_h_ = nullptr;   // pinned [kChunk]
  static constexpr int kSelCap = 4096;  // top-k survivors the device path returns
  uint32_t* recent_d_ = nullptr;        // [kMaxSeq] penalty window
  uint32_t* recent_h_ = nullptr;        // pinned [kMaxSeq]
  void* sel_d_ = nullptr;               // count, then kSelCap ids, then kSelCap values
  void* sel_h_ = nullptr;               // pinned copy of sel_d_
  void* sel_scratch_d_ = nullptr;       // candidates of the two-stage top-k selection
  int32_t* step_d_ = nullptr;           // decode step input: token id, position
  int32_t* step_h_ = nullptr;           // pinned
  void* decode_exec_[3] = {};           // cudaGraphExec_t of one decode step, in three pieces
  bool use_graph_ = true;
  long long decode_steps_ = 0;
};

}  // namespace obn
