// oxbitnet.cpp — the model-level C ABI (include/oxbitnet.h).
//
// Mirrors packages/rust/crates/oxbitnet-ffi/src/lib.rs: thread-local error
// (lib.rs:31-46), once-installed logger with a settable minimum level
// (lib.rs:120-237), default options (lib.rs:243-262), load / free (lib.rs:
// 278-376), generate / chat with a stop-by-return-value token callback
// (lib.rs:392-527, 548-573), and the generation loop of BitNet::generate_from_ids
// (oxbitnet/src/lib.rs:125-185) and model loading (model/loader.rs:45-76, 355-419).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/oxbitnet.h"
#include "bpe.h"
#include "gguf.h"
#include "model.h"
#include "sampler.h"

struct OxBitNet {
  std::unique_ptr<obn::Model> model;
};

struct OxBitNetTokenizer {
  obn::BpeTokenizer tok;
};

namespace {

// ---- thread-local error (lib.rs:31-46) --------------------------------------
thread_local std::string t_error;
thread_local bool t_has_error = false;
thread_local std::string t_describe;

void set_error(const std::string& m) {
  t_error = m;
  t_has_error = true;
}
void clear_error() { t_has_error = false; }

// ---- logger (lib.rs:120-237) ---------------------------------------------------
std::atomic<OxBitNetLogFn> g_log_fn{nullptr};
std::atomic<void*> g_log_ud{nullptr};
std::atomic<int> g_log_min{2};  // Info
std::once_flag g_log_once;

void log_msg(int level, const std::string& m) {
  OxBitNetLogFn fn = g_log_fn.load();
  if (!fn || level < g_log_min.load()) return;
  fn(static_cast<OxBitNetLogLevel>(level), m.c_str(), m.size(), g_log_ud.load());
}

// ---- UTF-8 validation of C strings (lib.rs:289-300) -----------------------------
bool valid_utf8(const char* s) {
  const std::string str(s);
  return obn::utf8_lossy(str) == str;  // repair changes exactly the ill-formed strings
}

// ---- SHA-256 (FIPS 180-4), for the download-cache file name (loader.rs:371-373) --
std::string sha256_hex(const std::string& msg) {
  static const uint32_t k[64] = {
      0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4,
      0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe,
      0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f,
      0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7,
      0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc,
      0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b,
      0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116,
      0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
      0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
      0xc67178f2};
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  std::vector<uint8_t> m(msg.begin(), msg.end());
  const uint64_t bits = static_cast<uint64_t>(m.size()) * 8;
  m.push_back(0x80);
  while (m.size() % 64 != 56) m.push_back(0);
  for (int i = 7; i >= 0; --i) m.push_back(static_cast<uint8_t>(bits >> (8 * i)));
  auto rotr = [](uint32_t x, int n) { return (x >> n) | (x << (32 - n)); };
  for (size_t off = 0; off < m.size(); off += 64) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(m[off + 4 * i]) << 24) | (uint32_t(m[off + 4 * i + 1]) << 16) |
             (uint32_t(m[off + 4 * i + 2]) << 8) | uint32_t(m[off + 4 * i + 3]);
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + k[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + mj;
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  char out[65];
  for (int i = 0; i < 8; ++i) std::snprintf(out + 8 * i, 9, "%08x", h[i]);
  return std::string(out, 64);
}

bool is_local(const std::string& src) {  // loader.rs:360-361
  return src.rfind("/", 0) == 0 || src.rfind(".", 0) == 0 || src.find("://") == std::string::npos;
}

std::string default_cache_dir() {  // dirs::cache_dir() joined with ".0xbitnet"
  const char* xdg = std::getenv("XDG_CACHE_HOME");
  if (xdg && *xdg == '/') return std::string(xdg) + "/.0xbitnet";
  const char* home = std::getenv("HOME");
  if (home && *home) return std::string(home) + "/.cache/.0xbitnet";
  return std::string();
}

std::string cache_path_for(const std::string& src, const char* cache_dir) {
  const std::string dir = (cache_dir && *cache_dir) ? std::string(cache_dir) : default_cache_dir();
  if (dir.empty()) return std::string();
  return dir + "/" + sha256_hex(src);
}

// A read-only mapping of a whole file.
struct Mapped {
  const uint8_t* data = nullptr;
  size_t size = 0;
  ~Mapped() {
    if (data && size) munmap(const_cast<uint8_t*>(data), size);
  }
  std::string open(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return "IO error: " + path + ": " + std::strerror(errno);
    struct stat st;
    if (fstat(fd, &st) != 0) {
      const std::string e = "IO error: " + path + ": " + std::strerror(errno);
      ::close(fd);
      return e;
    }
    size = static_cast<size_t>(st.st_size);
    if (size == 0) {
      ::close(fd);
      data = reinterpret_cast<const uint8_t*>("");
      return std::string();
    }
    void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) {
      size = 0;
      return "IO error: mmap of " + path + ": " + std::strerror(errno);
    }
    data = static_cast<const uint8_t*>(p);
    return std::string();
  }
};

OxBitNetGenerateOptions read_options(const OxBitNetGenerateOptions* o) {
  if (o) return *o;
  // lib.rs:579-585: NULL means the crate defaults with repeat_penalty 1.1
  return OxBitNetGenerateOptions{256, 1.0f, 50, 1.1f, 64};
}

// oxbitnet/src/lib.rs:125-185 over token ids; `emit` gets each token and
// returns true to stop. 0 / -1.
template <typename Emit>
int32_t run_generation(OxBitNet* h, const std::vector<uint32_t>& ids,
                       const OxBitNetGenerateOptions& o, Emit emit) {
  obn::Model& m = *h->model;
  m.reset();
  log_msg(1, "generate: " + std::to_string(ids.size()) + " input tokens");
  if (ids.empty()) return 0;
  if (ids.size() > static_cast<size_t>(obn::Model::kMaxSeq)) {
    set_error("prompt of " + std::to_string(ids.size()) + " tokens exceeds the " +
              std::to_string(obn::Model::kMaxSeq) + "-position KV cache");
    return -1;
  }
  std::string e = m.forward(ids.data(), static_cast<int>(ids.size()), /*copy_logits=*/false);
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  const obn::BpeTokenizer& tok = m.tokenizer();
  std::vector<uint32_t> recent;
  for (size_t step = 0; step < o.max_tokens; ++step) {
    const size_t start =
        o.repeat_last_n > 0 && recent.size() > o.repeat_last_n ? recent.size() - o.repeat_last_n : 0;
    uint32_t next = 0;
    e = m.sample(o.temperature, o.top_k, o.repeat_penalty, recent.data() + start,
                 recent.size() - start, m.sampler().uniform(), &next);
    if (!e.empty()) {
      set_error(e);
      return -1;
    }
    if (next == tok.eos_id() || (tok.has_eot() && next == tok.eot_id()) ||
        (tok.has_im_end() && next == tok.im_end_id()))
      break;
    recent.push_back(next);
    if (emit(next, tok.decode_one(next))) break;
    if (step + 1 == o.max_tokens) break;  // the reference's last forward is never read
    if (m.position() >= obn::Model::kMaxSeq) {
      log_msg(3, "generation stopped: the KV cache is full");
      break;
    }
    e = m.forward(&next, 1, /*copy_logits=*/false);
    if (!e.empty()) {
      set_error(e);
      return -1;
    }
  }
  return 0;
}

// lib.rs:548-573: a token whose text holds a NUL byte is skipped (CString::new fails).
bool call_text(OxBitNetTokenFn cb, void* ud, const std::string& text) {
  if (!cb || text.find('\0') != std::string::npos) return false;
  return cb(text.c_str(), text.size(), ud) != 0;
}

int32_t copy_ids(const std::vector<uint32_t>& ids, uint32_t* out, uintptr_t cap, uintptr_t* n) {
  if (n) *n = ids.size();
  if (out)
    for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  return 0;
}

int32_t copy_text(const std::string& s, char* buf, uintptr_t cap, uintptr_t* len) {
  if (len) *len = s.size();
  if (buf && cap) {
    const size_t k = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), k);
    buf[k] = '\0';
  }
  return 0;
}

bool read_messages(const OxBitNetChatMessage* msgs, uintptr_t n,
                   std::vector<obn::BpeTokenizer::Message>* out) {
  if (!msgs && n > 0) {
    set_error("messages must not be NULL when num_messages > 0");
    return false;
  }
  out->clear();
  for (uintptr_t i = 0; i < n; ++i) {
    const OxBitNetChatMessage& m = msgs[i];
    if (!m.role) {
      set_error("messages[" + std::to_string(i) + "].role must not be NULL");
      return false;
    }
    if (!valid_utf8(m.role)) {
      set_error("invalid UTF-8 in messages[" + std::to_string(i) + "].role");
      return false;
    }
    if (!m.content) {
      set_error("messages[" + std::to_string(i) + "].content must not be NULL");
      return false;
    }
    if (!valid_utf8(m.content)) {
      set_error("invalid UTF-8 in messages[" + std::to_string(i) + "].content");
      return false;
    }
    out->push_back({m.role, m.content});
  }
  return true;
}

}  // namespace

extern "C" {

void oxbitnet_set_logger(OxBitNetLogFn callback, void* userdata, uint8_t min_level) {
  g_log_min.store(min_level > 4 ? 4 : min_level);
  std::call_once(g_log_once, [&] {
    g_log_ud.store(userdata);
    g_log_fn.store(callback);
  });
}

OxBitNetGenerateOptions oxbitnet_default_generate_options(void) {
  return OxBitNetGenerateOptions{256, 1.0f, 50, 1.1f, 64};
}

OxBitNetLoadOptions oxbitnet_default_load_options(void) {
  return OxBitNetLoadOptions{nullptr, nullptr, nullptr};
}

OxBitNet* oxbitnet_load(const char* source, const OxBitNetLoadOptions* options) {
  clear_error();
  if (!source) {
    set_error("source must not be NULL");
    return nullptr;
  }
  if (!valid_utf8(source)) {
    set_error("invalid UTF-8 in source");
    return nullptr;
  }
  OxBitNetProgressFn cb = options ? options->on_progress : nullptr;
  void* ud = options ? options->progress_userdata : nullptr;
  const char* cache_dir = options ? options->cache_dir : nullptr;
  auto progress = [&](int phase, uint64_t loaded, uint64_t total, double fraction) {
    if (!cb) return;
    OxBitNetLoadProgress p{static_cast<OxBitNetLoadPhase>(phase), loaded, total, fraction};
    cb(&p, ud);
  };
  progress(0, 0, 0, 0.0);  // loader.rs:53-58
  std::string path = source;
  if (!is_local(path)) {  // loader.rs:366-384: the cache serves URLs; nothing is downloaded
    const std::string cached = cache_path_for(path, cache_dir);
    if (cached.empty() || access(cached.c_str(), R_OK) != 0) {
      set_error("HTTP error: downloading " + path +
                " needs a network client, which this build does not have; place the file at " +
                (cached.empty() ? std::string("<cache dir>/<sha256 of the URL>") : cached) +
                " or pass a local path");
      return nullptr;
    }
    log_msg(2, "Loading from cache: " + cached);
    path = cached;
  }
  Mapped file;
  std::string e = file.open(path);
  if (!e.empty()) {
    set_error(e);
    return nullptr;
  }
  progress(0, file.size, file.size, 1.0);
  progress(1, 0, 1, 0.0);  // loader.rs:62-67
  std::unique_ptr<obn::Model> model;
  e = obn::Model::load(file.data, file.size, progress, log_msg, &model);
  if (!e.empty()) {
    set_error(e);
    return nullptr;
  }
  auto* h = new OxBitNet;
  h->model = std::move(model);
  return h;
}

void oxbitnet_free(OxBitNet* model) { delete model; }

int32_t oxbitnet_generate(OxBitNet* model, const char* prompt,
                          const OxBitNetGenerateOptions* options, OxBitNetTokenFn callback,
                          void* userdata) {
  clear_error();
  if (!model) {
    set_error("model must not be NULL");
    return -1;
  }
  if (!prompt) {
    set_error("prompt must not be NULL");
    return -1;
  }
  if (!valid_utf8(prompt)) {
    set_error("invalid UTF-8 in prompt");
    return -1;
  }
  if (!model->model) {
    set_error("model has been disposed");
    return -1;
  }
  std::vector<uint32_t> ids;
  std::string e = model->model->tokenizer().encode(prompt, true, &ids);
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  return run_generation(model, ids, read_options(options),
                        [&](uint32_t, const std::string& t) { return call_text(callback, userdata, t); });
}

int32_t oxbitnet_chat(OxBitNet* model, const OxBitNetChatMessage* messages, uintptr_t num_messages,
                      const OxBitNetGenerateOptions* options, OxBitNetTokenFn callback,
                      void* userdata) {
  clear_error();
  if (!model) {
    set_error("model must not be NULL");
    return -1;
  }
  std::vector<obn::BpeTokenizer::Message> msgs;
  if (!read_messages(messages, num_messages, &msgs)) return -1;
  if (!model->model) {
    set_error("model has been disposed");
    return -1;
  }
  std::vector<uint32_t> ids;
  std::string e = model->model->tokenizer().apply_chat_template(msgs, &ids);
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  return run_generation(model, ids, read_options(options),
                        [&](uint32_t, const std::string& t) { return call_text(callback, userdata, t); });
}

const char* oxbitnet_error_message(void) { return t_has_error ? t_error.c_str() : nullptr; }

// ---- extensions ------------------------------------------------------------------

int32_t oxbitnet_generate_ids(OxBitNet* model, const uint32_t* ids, uintptr_t n,
                              const OxBitNetGenerateOptions* options, OxBitNetTokenIdFn callback,
                              void* userdata) {
  clear_error();
  if (!model || !model->model) {
    set_error("model must not be NULL");
    return -1;
  }
  if (!ids && n > 0) {
    set_error("ids must not be NULL when n > 0");
    return -1;
  }
  std::vector<uint32_t> v(ids, ids + n);
  return run_generation(model, v, read_options(options), [&](uint32_t id, const std::string& t) {
    return callback ? callback(id, t.c_str(), t.size(), userdata) != 0 : false;
  });
}

int32_t oxbitnet_set_seed(OxBitNet* model, uint64_t seed) {
  clear_error();
  if (!model || !model->model) {
    set_error("model must not be NULL");
    return -1;
  }
  model->model->sampler().reseed(seed);
  return 0;
}

int32_t oxbitnet_forward(OxBitNet* model, const uint32_t* ids, uintptr_t n, int32_t reset,
                         float* logits, uintptr_t vocab) {
  clear_error();
  if (!model || !model->model) {
    set_error("model must not be NULL");
    return -1;
  }
  if (!ids || n == 0) {
    set_error("forward needs at least one token id");
    return -1;
  }
  obn::Model& m = *model->model;
  if (logits && vocab < static_cast<uintptr_t>(m.config().vocab)) {
    set_error("the logits buffer holds fewer than vocab_size floats");
    return -1;
  }
  if (reset) m.reset();
  std::string e = m.forward(ids, static_cast<int>(n));
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  if (logits) std::memcpy(logits, m.logits(), sizeof(float) * m.config().vocab);
  return 0;
}

int32_t oxbitnet_model_info(const OxBitNet* model, OxBitNetModelInfo* info) {
  clear_error();
  if (!model || !model->model || !info) {
    set_error("model and info must not be NULL");
    return -1;
  }
  const obn::ModelConfig& c = model->model->config();
  info->vocab_size = c.vocab;
  info->hidden_size = c.hidden;
  info->intermediate_size = c.ffn;
  info->num_layers = c.layers;
  info->num_heads = c.heads;
  info->num_kv_heads = c.kv_heads;
  info->head_dim = c.head_dim;
  info->max_seq_len = obn::Model::kMaxSeq;
  info->position = model->model->position();
  info->rms_norm_eps = c.eps;
  info->rope_theta = c.rope_theta;
  info->tied_embeddings = c.tied;
  info->lm_head_f16 = c.lm_head_f16;
  info->gated_ffn = c.gated;
  info->activation = static_cast<int32_t>(c.act);
  return 0;
}

OxBitNetTokenizer* oxbitnet_tokenizer_load(const char* path) {
  clear_error();
  if (!path) {
    set_error("path must not be NULL");
    return nullptr;
  }
  Mapped file;
  std::string e = file.open(path);
  obn::gguf::File f;
  if (e.empty()) e = obn::gguf::parse(file.data, file.size, &f);
  auto* t = new OxBitNetTokenizer;
  if (e.empty()) e = t->tok.init_from_gguf(f);
  if (!e.empty()) {
    delete t;
    set_error(e);
    return nullptr;
  }
  return t;
}

void oxbitnet_tokenizer_free(OxBitNetTokenizer* tok) { delete tok; }

int32_t oxbitnet_tokenize(const OxBitNetTokenizer* tok, const char* text, int32_t add_bos,
                          uint32_t* ids, uintptr_t cap, uintptr_t* n_ids) {
  clear_error();
  if (!tok || !text) {
    set_error("tokenizer and text must not be NULL");
    return -1;
  }
  std::vector<uint32_t> v;
  std::string e = tok->tok.encode(text, add_bos != 0, &v);
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  return copy_ids(v, ids, cap, n_ids);
}

int32_t oxbitnet_chat_template(const OxBitNetTokenizer* tok, const OxBitNetChatMessage* messages,
                               uintptr_t num_messages, uint32_t* ids, uintptr_t cap,
                               uintptr_t* n_ids) {
  clear_error();
  if (!tok) {
    set_error("tokenizer must not be NULL");
    return -1;
  }
  std::vector<obn::BpeTokenizer::Message> msgs;
  if (!read_messages(messages, num_messages, &msgs)) return -1;
  std::vector<uint32_t> v;
  std::string e = tok->tok.apply_chat_template(msgs, &v);
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  return copy_ids(v, ids, cap, n_ids);
}

int32_t oxbitnet_detokenize(const OxBitNetTokenizer* tok, const uint32_t* ids, uintptr_t n,
                            char* buf, uintptr_t cap, uintptr_t* len) {
  clear_error();
  if (!tok || (!ids && n)) {
    set_error("tokenizer and ids must not be NULL");
    return -1;
  }
  return copy_text(tok->tok.decode(std::vector<uint32_t>(ids, ids + n)), buf, cap, len);
}

int32_t oxbitnet_token_text(const OxBitNetTokenizer* tok, uint32_t id, char* buf, uintptr_t cap,
                            uintptr_t* len) {
  clear_error();
  if (!tok) {
    set_error("tokenizer must not be NULL");
    return -1;
  }
  return copy_text(tok->tok.decode_one(id), buf, cap, len);
}

int32_t oxbitnet_sample_next(OxBitNet* model, float temperature, uintptr_t top_k,
                             float repeat_penalty, const uint32_t* recent, uintptr_t n_recent,
                             float u, uint32_t* out) {
  clear_error();
  if (!model || !model->model || !out || (!recent && n_recent)) {
    set_error("model and out must not be NULL");
    return -1;
  }
  std::string e = model->model->sample(temperature, top_k, repeat_penalty, recent, n_recent, u, out);
  if (!e.empty()) {
    set_error(e);
    return -1;
  }
  return 0;
}

uint32_t oxbitnet_sample(float* logits, uintptr_t vocab, float temperature, uintptr_t top_k,
                         float repeat_penalty, const uint32_t* recent, uintptr_t n_recent,
                         float u) {
  if (!logits) return 0;
  return obn::sample_logits(logits, vocab, temperature, top_k, repeat_penalty, recent,
                            recent ? n_recent : 0, u);
}

const char* oxbitnet_gguf_describe(const char* path) {
  clear_error();
  if (!path) {
    set_error("path must not be NULL");
    return nullptr;
  }
  Mapped file;
  std::string e = file.open(path);
  obn::gguf::File f;
  if (e.empty()) e = obn::gguf::parse(file.data, file.size, &f);
  obn::ModelConfig c;
  if (e.empty()) e = obn::config_from_gguf(f, &c);
  if (!e.empty()) {
    set_error(e);
    return nullptr;
  }
  auto q = [](const std::string& s) {  // JSON string (names and keys are plain UTF-8)
    std::string o = "\"";
    for (unsigned char ch : s) {
      if (ch == '"' || ch == '\\') {
        o += '\\';
        o += static_cast<char>(ch);
      } else if (ch < 0x20) {
        char b[8];
        std::snprintf(b, sizeof(b), "\\u%04x", ch);
        o += b;
      } else {
        o += static_cast<char>(ch);
      }
    }
    return o + "\"";
  };
  char b[512];
  std::snprintf(b, sizeof(b),
                "{\"version\": %u, \"tensor_count\": %llu, \"data_offset\": %zu, \"config\": "
                "{\"arch\": %s, \"vocab_size\": %d, \"hidden_size\": %d, \"intermediate_size\": %d, "
                "\"num_layers\": %d, \"num_heads\": %d, \"num_kv_heads\": %d, \"head_dim\": %d, "
                "\"context_length\": %d, \"rms_norm_eps\": %.9g, \"rope_theta\": %.9g, "
                "\"tied\": %s, \"gated\": %s, \"activation\": %d}",
                f.version, static_cast<unsigned long long>(f.tensor_count), f.data_offset,
                q(c.arch).c_str(), c.vocab, c.hidden, c.ffn, c.layers, c.heads, c.kv_heads,
                c.head_dim, c.context_length, static_cast<double>(c.eps),
                static_cast<double>(c.rope_theta), c.tied ? "true" : "false",
                c.gated ? "true" : "false", static_cast<int>(c.act));
  std::string out = b;
  out += ", \"metadata_keys\": [";
  for (size_t i = 0; i < f.key_order.size(); ++i) out += (i ? ", " : "") + q(f.key_order[i]);
  out += "], \"tensors\": [";
  for (size_t i = 0; i < f.tensors.size(); ++i) {
    const obn::gguf::TensorInfo& t = f.tensors[i];
    size_t bytes = 0;
    const bool known = obn::gguf::tensor_bytes(t, &bytes).empty();
    out += i ? ", " : "";
    out += "{\"name\": " + q(t.name) + ", \"hf_name\": " + q(obn::hf_name(t.name)) +
           ", \"type\": " + std::to_string(t.type) + ", \"shape\": [";
    for (size_t k = 0; k < t.shape.size(); ++k)
      out += (k ? ", " : "") + std::to_string(t.shape[k]);
    out += "], \"offset\": " + std::to_string(t.offset) +
           ", \"bytes\": " + (known ? std::to_string(bytes) : std::string("null")) + "}";
  }
  out += "]}";
  t_describe = out;
  return t_describe.c_str();
}

int32_t oxbitnet_cache_path(const char* source, const char* cache_dir, char* buf, uintptr_t cap) {
  clear_error();
  if (!source) {
    set_error("source must not be NULL");
    return -1;
  }
  const std::string p = cache_path_for(source, cache_dir);
  if (p.empty()) {
    set_error("no cache directory (HOME and XDG_CACHE_HOME are unset)");
    return -1;
  }
  return copy_text(p, buf, cap, nullptr);
}

}  // extern "C"
