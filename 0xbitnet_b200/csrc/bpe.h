// bpe.h — the model-level tokenizer: byte-level BPE built from GGUF metadata.
//
// Restates what the reference's Tokenizer (packages/rust/crates/oxbitnet/src/
// tokenizer.rs:20-217) builds with the HF `tokenizers` crate (0.21.4, not
// vendored): a BPE model over `tokenizer.ggml.tokens` (token i has id i) and
// `tokenizer.ggml.merges` ("left right", rank = index), unk token "<unk>", the
// byte-level pre-tokenizer with add_prefix_space = false and use_regex = false
// (the whole text is one word: its UTF-8 bytes mapped to the GPT-2 byte
// alphabet, then merged), and the byte-level decoder.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace obn {
namespace gguf {
struct File;
}

class BpeTokenizer {
 public:
  // tokenizer.rs:22-92. Empty string on success, else the error text.
  std::string init_from_gguf(const gguf::File& f);
  // Direct construction (tests): tokens by id, merges as "left right".
  std::string init(const std::vector<std::string>& tokens, const std::vector<std::string>& merges,
                   uint32_t bos_id, uint32_t eos_id);

  // tokenizer.rs:108-119: BOS (optional) + the BPE ids of `text`.
  std::string encode(const std::string& text, bool add_bos, std::vector<uint32_t>* ids) const;
  // tokenizer.rs:122-133: drops BOS/EOS ids, then decodes (invalid UTF-8 -> U+FFFD).
  std::string decode(const std::vector<uint32_t>& ids) const;
  // tokenizer.rs:136-140: one id, as the streaming generator emits it (its
  // bytes with invalid UTF-8 repaired, so a split character shows as U+FFFD).
  std::string decode_one(uint32_t id) const;

  // HF Tokenizer::token_to_id: the id of an exact vocabulary string.
  bool token_to_id(const std::string& token, uint32_t* id) const;

  struct Message {
    std::string role, content;
  };
  // tokenizer.rs:160-217: ChatML when <|im_start|>/<|im_end|> exist, else LLaMA 3
  // headers when <|start_header_id|>/<|end_header_id|>/<|eot_id|> exist, else
  // the contents joined by "\n" and encoded with BOS.
  std::string apply_chat_template(const std::vector<Message>& msgs,
                                  std::vector<uint32_t>* ids) const;

  uint32_t bos_id() const { return bos_; }
  uint32_t eos_id() const { return eos_; }
  bool has_eot() const { return has_eot_; }
  uint32_t eot_id() const { return eot_; }
  bool has_im_end() const { return has_im_end_; }
  uint32_t im_end_id() const { return im_end_; }
  size_t vocab_size() const { return id_to_token_.size(); }

 private:
  struct PairHash {
    size_t operator()(uint64_t k) const { return std::hash<uint64_t>()(k * 0x9E3779B97F4A7C15ull); }
  };
  struct Merge {
    uint32_t rank, new_id;
  };
  std::string bpe(const std::string& piece, std::vector<uint32_t>* ids) const;
  // The bytes a token stands for (byte-level decoder, before UTF-8 repair).
  std::string token_bytes(uint32_t id) const;

  std::unordered_map<std::string, uint32_t> vocab_;
  std::vector<std::string> id_to_token_;
  std::unordered_map<uint64_t, Merge, PairHash> merges_;  // (left << 32 | right)
  std::string byte_to_char_[256];                          // UTF-8 of the byte's code point
  std::unordered_map<uint32_t, uint8_t> char_to_byte_;     // code point -> byte
  uint32_t bos_ = 1, eos_ = 2, eot_ = 0, im_end_ = 0;
  bool has_eot_ = false, has_im_end_ = false;
};

// String::from_utf8_lossy: each maximal invalid subsequence becomes U+FFFD.
std::string utf8_lossy(const std::string& bytes);

}  // namespace obn
