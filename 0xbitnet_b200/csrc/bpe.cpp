// bpe.cpp — byte-level BPE tokenizer (bpe.h).
#include "bpe.h"

#include <queue>

#include "gguf.h"

namespace obn {

namespace {

void append_utf8(std::string* s, uint32_t cp) {
  if (cp < 0x80) {
    s->push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    s->push_back(static_cast<char>(0xC0 | (cp >> 6)));
    s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    s->push_back(static_cast<char>(0xE0 | (cp >> 12)));
    s->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    s->push_back(static_cast<char>(0xF0 | (cp >> 18)));
    s->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    s->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

// Length of the well-formed UTF-8 sequence at p[0..n), or 0 with *maximal set
// to the length of its longest well-formed prefix (at least 1). Strings from
// std::string are well-formed where they came from valid UTF-8.
size_t utf8_seq(const unsigned char* p, size_t n, uint32_t* cp, size_t* maximal) {
  const unsigned c = p[0];
  *maximal = 1;
  if (c < 0x80) {
    *cp = c;
    return 1;
  }
  size_t len;
  unsigned lo = 0x80, hi = 0xBF;
  if (c >= 0xC2 && c <= 0xDF) {
    len = 2;
  } else if (c >= 0xE0 && c <= 0xEF) {
    len = 3;
    if (c == 0xE0) lo = 0xA0;
    if (c == 0xED) hi = 0x9F;
  } else if (c >= 0xF0 && c <= 0xF4) {
    len = 4;
    if (c == 0xF0) lo = 0x90;
    if (c == 0xF4) hi = 0x8F;
  } else {
    return 0;
  }
  uint32_t v = c & (len == 2 ? 0x1F : len == 3 ? 0x0F : 0x07);
  for (size_t k = 1; k < len; ++k) {
    if (k >= n) return 0;
    const unsigned b = p[k];
    const unsigned l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
    if (b < l || b > h) return 0;
    v = (v << 6) | (b & 0x3F);
    *maximal = k + 1;
  }
  *cp = v;
  return len;
}

}  // namespace

std::string utf8_lossy(const std::string& bytes) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(bytes.data());
  const size_t n = bytes.size();
  std::string out;
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    uint32_t cp;
    size_t maximal;
    const size_t len = utf8_seq(p + i, n - i, &cp, &maximal);
    if (len) {
      out.append(bytes, i, len);
      i += len;
    } else {
      out.append("\xEF\xBF\xBD");
      i += maximal;
    }
  }
  return out;
}

std::string BpeTokenizer::init(const std::vector<std::string>& tokens,
                               const std::vector<std::string>& merges, uint32_t bos_id,
                               uint32_t eos_id) {
  // GPT-2 byte alphabet: printable Latin-1 bytes stand for themselves, the
  // other 68 bytes take code points 256, 257, ... in byte order.
  int next = 0;
  for (int b = 0; b < 256; ++b) {
    const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
    const uint32_t cp = keep ? static_cast<uint32_t>(b) : 256u + static_cast<uint32_t>(next++);
    byte_to_char_[b].clear();
    append_utf8(&byte_to_char_[b], cp);
    char_to_byte_[cp] = static_cast<uint8_t>(b);
  }
  id_to_token_ = tokens;
  vocab_.clear();
  vocab_.reserve(tokens.size() * 2);
  for (size_t i = 0; i < tokens.size(); ++i)  // a repeated string keeps its last id
    vocab_[tokens[i]] = static_cast<uint32_t>(i);
  merges_.clear();
  merges_.reserve(merges.size() * 2);
  for (size_t r = 0; r < merges.size(); ++r) {
    const std::string& m = merges[r];
    const size_t sp = m.find(' ');  // tokenizer.rs:52-61: splitn(2, ' '), others dropped
    if (sp == std::string::npos) continue;
    const std::string a = m.substr(0, sp), b = m.substr(sp + 1);
    auto ia = vocab_.find(a), ib = vocab_.find(b), iab = vocab_.find(a + b);
    if (ia == vocab_.end() || ib == vocab_.end())
      return "Tokenizer error: Failed to build BPE: merge token `" +
             (ia == vocab_.end() ? a : b) + "` out of vocabulary";
    if (iab == vocab_.end())
      return "Tokenizer error: Failed to build BPE: merge token `" + a + b +
             "` out of vocabulary";
    const uint64_t key = (static_cast<uint64_t>(ia->second) << 32) | ib->second;
    merges_[key] = Merge{static_cast<uint32_t>(r), iab->second};  // a repeated pair keeps its last rank
  }
  bos_ = bos_id;
  eos_ = eos_id;
  has_eot_ = token_to_id("<|eot_id|>", &eot_);
  has_im_end_ = token_to_id("<|im_end|>", &im_end_);
  return std::string();
}

std::string BpeTokenizer::init_from_gguf(const gguf::File& f) {
  const gguf::Value* tv = f.get("tokenizer.ggml.tokens");
  std::vector<const std::string*> tok_ptrs;
  if (!tv || !tv->as_string_array(&tok_ptrs))
    return "Tokenizer error: Missing tokenizer.ggml.tokens";
  std::vector<std::string> tokens;
  tokens.reserve(tok_ptrs.size());
  for (const std::string* s : tok_ptrs) tokens.push_back(*s);
  std::vector<std::string> merges;
  std::vector<const std::string*> merge_ptrs;
  const gguf::Value* mv = f.get("tokenizer.ggml.merges");
  if (mv && mv->as_string_array(&merge_ptrs)) {
    merges.reserve(merge_ptrs.size());
    for (const std::string* s : merge_ptrs) merges.push_back(*s);
  }
  uint32_t bos = 1, eos = 2;  // tokenizer.rs:32-39 defaults
  if (const gguf::Value* v = f.get("tokenizer.ggml.bos_token_id")) {
    uint32_t x;
    if (v->as_u32(&x)) bos = x;
  }
  if (const gguf::Value* v = f.get("tokenizer.ggml.eos_token_id")) {
    uint32_t x;
    if (v->as_u32(&x)) eos = x;
  }
  return init(tokens, merges, bos, eos);
}

bool BpeTokenizer::token_to_id(const std::string& token, uint32_t* id) const {
  auto it = vocab_.find(token);
  if (it == vocab_.end()) return false;
  *id = it->second;
  return true;
}

// One pre-tokenized piece (already in the byte alphabet) through the BPE model:
// one symbol per character, then merges applied lowest rank first, leftmost
// first among equal ranks, until no adjacent pair has a merge.
std::string BpeTokenizer::bpe(const std::string& piece, std::vector<uint32_t>* ids) const {
  struct Sym {
    uint32_t id;
    int prev, next;
    bool alive;
  };
  std::vector<Sym> syms;
  syms.reserve(piece.size());
  const unsigned char* p = reinterpret_cast<const unsigned char*>(piece.data());
  bool have_unk = false;
  uint32_t unk_id = 0;
  size_t i = 0;
  while (i < piece.size()) {
    uint32_t cp;
    size_t maximal;
    size_t len = utf8_seq(p + i, piece.size() - i, &cp, &maximal);
    if (!len) len = maximal;
    auto it = vocab_.find(piece.substr(i, len));
    uint32_t id;
    if (it != vocab_.end()) {
      id = it->second;
    } else {  // an unknown character becomes "<unk>" (not fused)
      if (!have_unk) {
        auto u = vocab_.find("<unk>");
        if (u == vocab_.end())
          return "Tokenizer error: Encode failed: Unk token `<unk>` not found in the vocabulary";
        unk_id = u->second;
        have_unk = true;
      }
      id = unk_id;
    }
    const int k = static_cast<int>(syms.size());
    syms.push_back(Sym{id, k - 1, k + 1, true});
    i += len;
  }
  if (syms.empty()) return std::string();
  syms.back().next = -1;

  struct Cand {
    uint32_t rank;
    int pos;
    uint32_t new_id;
    bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
  };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> q;
  auto pair_of = [&](int a) -> const Merge* {
    const int b = syms[a].next;
    if (b < 0) return nullptr;
    auto it = merges_.find((static_cast<uint64_t>(syms[a].id) << 32) | syms[b].id);
    return it == merges_.end() ? nullptr : &it->second;
  };
  for (int a = 0; a + 1 < static_cast<int>(syms.size()); ++a)
    if (const Merge* m = pair_of(a)) q.push(Cand{m->rank, a, m->new_id});
  while (!q.empty()) {
    const Cand c = q.top();
    q.pop();
    Sym& s = syms[c.pos];
    if (!s.alive || s.next < 0) continue;
    const Merge* m = pair_of(c.pos);
    if (!m || m->new_id != c.new_id) continue;  // the pair changed since it was queued
    const int b = s.next;
    s.id = c.new_id;
    syms[b].alive = false;
    s.next = syms[b].next;
    if (s.next >= 0) syms[s.next].prev = c.pos;
    if (s.prev >= 0)
      if (const Merge* pm = pair_of(s.prev)) q.push(Cand{pm->rank, s.prev, pm->new_id});
    if (const Merge* nm = pair_of(c.pos)) q.push(Cand{nm->rank, c.pos, nm->new_id});
  }
  for (int a = 0; a >= 0; a = syms[a].next) ids->push_back(syms[a].id);
  return std::string();
}

std::string BpeTokenizer::encode(const std::string& text, bool add_bos,
                                 std::vector<uint32_t>* ids) const {
  ids->clear();
  if (add_bos) ids->push_back(bos_);
  std::string piece;
  piece.reserve(text.size() * 2);
  for (unsigned char c : text) piece += byte_to_char_[c];
  return bpe(piece, ids);
}

std::string BpeTokenizer::token_bytes(uint32_t id) const {
  if (id >= id_to_token_.size()) return std::string();  // unknown ids are skipped
  const std::string& tok = id_to_token_[id];
  // Byte-level decoder: every character maps back to its byte; a token with a
  // character outside the alphabet contributes its own UTF-8 bytes instead.
  std::string bytes;
  const unsigned char* p = reinterpret_cast<const unsigned char*>(tok.data());
  size_t i = 0;
  bool all = true;
  while (i < tok.size()) {
    uint32_t cp;
    size_t maximal;
    const size_t len = utf8_seq(p + i, tok.size() - i, &cp, &maximal);
    if (!len) {
      all = false;
      break;
    }
    auto it = char_to_byte_.find(cp);
    if (it == char_to_byte_.end()) {
      all = false;
      break;
    }
    bytes.push_back(static_cast<char>(it->second));
    i += len;
  }
  return all ? bytes : tok;
}

std::string BpeTokenizer::decode_one(uint32_t id) const { return utf8_lossy(token_bytes(id)); }

std::string BpeTokenizer::decode(const std::vector<uint32_t>& ids) const {
  std::string bytes;
  for (uint32_t id : ids) {
    if (id == bos_ || id == eos_) continue;
    bytes += token_bytes(id);
  }
  return utf8_lossy(bytes);
}

std::string BpeTokenizer::apply_chat_template(const std::vector<Message>& msgs,
                                              std::vector<uint32_t>* ids) const {
  ids->clear();
  std::vector<uint32_t> part;
  auto add = [&](const std::string& text) -> std::string {
    std::string e = encode(text, false, &part);
    if (e.empty()) ids->insert(ids->end(), part.begin(), part.end());
    return e;
  };
  uint32_t im_start, im_end;
  if (token_to_id("<|im_start|>", &im_start) && token_to_id("<|im_end|>", &im_end)) {
    ids->push_back(bos_);  // ChatML, tokenizer.rs:200-217
    for (const Message& m : msgs) {
      ids->push_back(im_start);
      if (std::string e = add(m.role + "\n" + m.content); !e.empty()) return e;
      ids->push_back(im_end);
      if (std::string e = add("\n"); !e.empty()) return e;
    }
    ids->push_back(im_start);
    return add("assistant\n");
  }
  uint32_t sh, eh, eot;
  if (!token_to_id("<|start_header_id|>", &sh) || !token_to_id("<|end_header_id|>", &eh) ||
      !token_to_id("<|eot_id|>", &eot)) {
    std::string text;  // tokenizer.rs:171-175
    for (size_t k = 0; k < msgs.size(); ++k) {
      if (k) text += "\n";
      text += msgs[k].content;
    }
    std::vector<uint32_t> out;
    std::string e = encode(text, true, &out);
    *ids = out;
    return e;
  }
  ids->push_back(bos_);  // LLaMA 3, tokenizer.rs:177-196
  for (const Message& m : msgs) {
    ids->push_back(sh);
    if (std::string e = add(m.role); !e.empty()) return e;
    ids->push_back(eh);
    if (std::string e = add("\n\n" + m.content); !e.empty()) return e;
    ids->push_back(eot);
  }
  ids->push_back(sh);
  if (std::string e = add("assistant"); !e.empty()) return e;
  ids->push_back(eh);
  return add("\n\n");
}

}  // namespace obn
