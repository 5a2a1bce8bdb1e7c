// model.cpp — GGUF -> device model, and the forward pass over libobn (model.h).
#include "model.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <utility>

#include "../../include/obn.h"
#include "gguf.h"
#include "sampling.h"

namespace obn {

namespace {

std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char* f, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof(buf), f, ap);
  va_end(ap);
  return buf;
}

std::string obn_fail(const char* what) {
  const char* m = obn_error_message();
  return std::string(what) + ": " + (m ? m : "unknown error");
}

std::string cuda_fail(cudaError_t e, const char* what) {
  return fmt("GPU error: %s: %s", what, cudaGetErrorString(e));
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: value = man * 2^-24
      float v = std::ldexp(static_cast<float>(man), -24);
      std::memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

}  // namespace

std::string hf_name(const std::string& name) {
  if (name == "token_embd.weight") return "model.embed_tokens.weight";
  if (name == "output_norm.weight") return "model.norm.weight";
  if (name == "output.weight") return "lm_head.weight";
  if (name.compare(0, 4, "blk.") == 0) {
    const size_t dot = name.find('.', 4);
    if (dot != std::string::npos) {
      const std::string layer = name.substr(4, dot - 4), comp = name.substr(dot + 1);
      static const char* const kMap[][2] = {
          {"attn_q.weight", "self_attn.q_proj.weight"},
          {"attn_k.weight", "self_attn.k_proj.weight"},
          {"attn_v.weight", "self_attn.v_proj.weight"},
          {"attn_output.weight", "self_attn.o_proj.weight"},
          {"attn_norm.weight", "input_layernorm.weight"},
          {"ffn_norm.weight", "post_attention_layernorm.weight"},
          {"attn_sub_norm.weight", "self_attn.sub_norm.weight"},
          {"ffn_sub_norm.weight", "mlp.sub_norm.weight"},
          {"ffn_up.weight", "mlp.up_proj.weight"},
          {"ffn_down.weight", "mlp.down_proj.weight"},
          {"ffn_gate.weight", "mlp.gate_proj.weight"},
      };
      for (const auto& m : kMap)
        if (comp == m[0]) return "model.layers." + layer + "." + m[1];
      return "model.layers." + layer + "." + comp;
    }
  }
  return name;
}

std::string config_from_gguf(const gguf::File& f, ModelConfig* cfg) {
  ModelConfig c;
  const gguf::Value* av = f.get("general.architecture");
  c.arch = (av && av->as_str()) ? *av->as_str() : "bitnet";
  auto get = [&](const char* suffix) -> const gguf::Value* {
    for (const std::string& pre : {c.arch, std::string("llama"), std::string("bitnet"),
                                   std::string("bitnet-25")})
      if (const gguf::Value* v = f.get(pre + "." + suffix)) return v;
    return nullptr;
  };
  auto get_u32 = [&](const char* suffix, uint32_t def) {
    uint32_t v;
    const gguf::Value* p = get(suffix);
    return (p && p->as_u32(&v)) ? v : def;
  };
  auto get_f32 = [&](const char* suffix, float def) {
    float v;
    const gguf::Value* p = get(suffix);
    return (p && p->as_f32(&v)) ? v : def;
  };
  c.hidden = static_cast<int>(get_u32("embedding_length", 2560));
  c.layers = static_cast<int>(get_u32("block_count", 30));
  c.heads = static_cast<int>(get_u32("attention.head_count", 20));
  c.kv_heads = static_cast<int>(get_u32("attention.head_count_kv", static_cast<uint32_t>(c.heads)));
  uint32_t vocab = 0;
  const gguf::Value* vs = get("vocab_size");
  if (!(vs && vs->as_u32(&vocab))) {
    std::vector<const std::string*> toks;
    const gguf::Value* tv = f.get("tokenizer.ggml.tokens");
    vocab = (tv && tv->as_string_array(&toks)) ? static_cast<uint32_t>(toks.size()) : 128256u;
  }
  c.vocab = static_cast<int>(vocab);
  c.ffn = static_cast<int>(get_u32("feed_forward_length", 6912));
  const bool b25 = c.arch == "bitnet-25";
  c.context_length = static_cast<int>(get_u32("context_length", 4096));
  c.eps = get_f32("attention.layer_norm_rms_epsilon", 1e-5f);
  c.rope_theta = get_f32("rope.freq_base", b25 ? 500000.0f : 10000.0f);
  c.act = b25 ? Activation::kRelu2 : Activation::kSilu;  // loader.rs:301-305
  c.tied = f.tensor("output.weight") == nullptr;           // loader.rs:85-86
  c.gated = f.tensor("blk.0.ffn_gate.weight") != nullptr;
  if (c.heads <= 0 || c.kv_heads <= 0 || c.hidden <= 0 || c.layers <= 0 || c.ffn <= 0 ||
      c.vocab <= 0)
    return "model config has a zero dimension";
  c.head_dim = c.hidden / c.heads;
  *cfg = c;
  return std::string();
}

Model::~Model() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
  for (Layer& L : layers_) {
    obn_bitlinear_free(L.qkv);
    obn_bitlinear_free(L.o);
    obn_bitlinear_free(L.ffn_in);
    obn_bitlinear_free(L.down);
  }
  obn_bitlinear_free(lm_ternary_);
  for (void* p : k_cache_) cudaFree(p);
  for (void* p : v_cache_) cudaFree(p);
  for (void* p : {embed_, lm_f16_, static_cast<void*>(final_norm_), static_cast<void*>(x_),
                  static_cast<void*>(qkv_), static_cast<void*>(q_), static_cast<void*>(attn_),
                  static_cast<void*>(ffn_), static_cast<void*>(lm_in_),
                  static_cast<void*>(logits_d_), static_cast<void*>(ids_d_), ws_, attn_ws_})
    cudaFree(p);
  for (void* ge : decode_exec_)
    if (ge) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(ge));
  cudaFree(recent_d_);
  cudaFree(sel_d_);
  cudaFree(sel_scratch_d_);
  cudaFree(step_d_);
  cudaFreeHost(step_h_);
  cudaFreeHost(logits_h_);
  cudaFreeHost(ids_h_);
  cudaFreeHost(recent_h_);
  cudaFreeHost(sel_h_);
  if (stream_) cudaStreamDestroy(static_cast<cudaStream_t>(stream_));
  cudaSetDevice(prev);
}

std::string Model::load(const uint8_t* data, size_t size, const ProgressFn& progress,
                        const LogFn& log, std::unique_ptr<Model>* out) {
  gguf::File f;
  std::string e = gguf::parse(data, size, &f);
  if (!e.empty()) return e;
  std::unique_ptr<Model> m(new Model);
  e = m->build(f, data, size, progress, log);
  if (!e.empty()) return e;
  *out = std::move(m);
  return std::string();
}

std::string Model::build(const gguf::File& f, const uint8_t* data, size_t size,
                         const ProgressFn& progress, const LogFn& log) {
  std::string e = config_from_gguf(f, &cfg_);
  if (!e.empty()) return e;
  const ModelConfig& c = cfg_;
  log(1, fmt("config: arch=%s, heads=%d, kv_heads=%d, head_dim=%d, hidden=%d, intermediate=%d, "
             "layers=%d, tied=%s",
             c.arch.c_str(), c.heads, c.kv_heads, c.head_dim, c.hidden, c.ffn, c.layers,
             c.tied ? "true" : "false"));
  const int G = c.heads / c.kv_heads;
  if (c.head_dim != 128 || c.head_dim * c.heads != c.hidden)
    return fmt("unsupported model: head_dim %d (hidden %d / %d heads); the attention kernels "
               "are built for head_dim 128",
               c.head_dim, c.hidden, c.heads);
  if (c.heads % c.kv_heads != 0 || (G != 1 && G != 2 && G != 4 && G != 8))
    return fmt("unsupported model: %d heads over %d KV heads (groups of 1, 2, 4 or 8)", c.heads,
               c.kv_heads);
  e = tok_.init_from_gguf(f);  // lib.rs:90-96: the tokenizer comes from the same metadata
  if (!e.empty()) return e;
  has_tok_ = true;

  cudaError_t ce = cudaGetDevice(&device_);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
  cudaStream_t s;
  ce = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamCreate");
  stream_ = s;

  const uint64_t total = f.tensors.size();
  uint64_t done = 0;
  auto tick = [&](uint64_t k) {
    done += k;
    if (done > total) done = total;
    progress(2, done, total, total ? static_cast<double>(done) / static_cast<double>(total) : 1.0);
  };
  auto find = [&](const std::string& name, bool required, const gguf::TensorInfo** ti,
                  const uint8_t** p, size_t* bytes) -> std::string {
    *ti = f.tensor(name);
    if (!*ti) return required ? "Missing weight tensor: \"" + hf_name(name) + "\"" : std::string();
    std::string err = gguf::tensor_bytes(**ti, bytes);
    if (!err.empty()) return err;
    const size_t off = f.data_offset + (*ti)->offset;
    if ((*ti)->offset > size || off > size || *bytes > size - off)
      return "GGUF parse error: data of tensor '" + name + "' runs past the end of the file";
    *p = data + off;
    log(1, fmt("tensor: %s -> %s (type=%u, %zu bytes)", name.c_str(), hf_name(name).c_str(),
               (*ti)->type, *bytes));
    return std::string();
  };
  // A norm weight [n] in F32 (F16 is widened, loader.rs:146-148); empty if absent and optional.
  auto vec_f32 = [&](const std::string& name, bool required, int n,
                     std::vector<float>* out) -> std::string {
    const gguf::TensorInfo* ti;
    const uint8_t* p = nullptr;
    size_t bytes = 0;
    out->clear();
    std::string err = find(name, required, &ti, &p, &bytes);
    if (!err.empty() || !ti) return err;
    if (ti->elements() != static_cast<uint64_t>(n))
      return fmt("tensor %s has %llu elements, expected %d", name.c_str(),
                 static_cast<unsigned long long>(ti->elements()), n);
    out->resize(n);
    if (ti->type == gguf::kTypeF32) {
      std::memcpy(out->data(), p, sizeof(float) * n);
    } else if (ti->type == gguf::kTypeF16) {
      for (int i = 0; i < n; ++i) {
        uint16_t h;
        std::memcpy(&h, p + 2 * i, 2);
        (*out)[i] = f16_to_f32(h);
      }
    } else {
      return fmt("unsupported model: tensor %s has GGML type %u (F32 or F16 expected)",
                 name.c_str(), ti->type);
    }
    return std::string();
  };
  struct Ternary {
    const uint8_t* p = nullptr;
    size_t bytes = 0;
  };
  auto ternary = [&](const std::string& name, int in, int out_rows, Ternary* t) -> std::string {
    const gguf::TensorInfo* ti;
    std::string err = find(name, true, &ti, &t->p, &t->bytes);
    if (!err.empty()) return err;
    if (ti->type != gguf::kTypeI2_S)
      return fmt("unsupported model: tensor %s has GGML type %u (I2_S expected)", name.c_str(),
                 ti->type);
    if (ti->shape.size() < 2 || ti->shape[0] != static_cast<uint64_t>(in) ||
        ti->shape[1] != static_cast<uint64_t>(out_rows))
      return fmt("tensor %s is not [%d, %d] (ne0 = in, ne1 = out)", name.c_str(), in, out_rows);
    return std::string();
  };

  const int D = c.hidden, F = c.ffn, H = c.heads, Hkv = c.kv_heads, d = c.head_dim;
  layers_.resize(c.layers);
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "blk." + std::to_string(i) + ".";
    Layer& L = layers_[i];
    std::vector<float> attn_norm, ffn_norm, attn_sub, ffn_sub;
    Ternary tq, tk, tv, to, tg, tu, td;
    if (!(e = vec_f32(p + "attn_norm.weight", true, D, &attn_norm)).empty()) return e;
    if (!(e = vec_f32(p + "ffn_norm.weight", true, D, &ffn_norm)).empty()) return e;
    if (!(e = vec_f32(p + "attn_sub_norm.weight", false, H * d, &attn_sub)).empty()) return e;
    if (!(e = vec_f32(p + "ffn_sub_norm.weight", false, F, &ffn_sub)).empty()) return e;
    if (!(e = ternary(p + "attn_q.weight", D, H * d, &tq)).empty()) return e;
    if (!(e = ternary(p + "attn_k.weight", D, Hkv * d, &tk)).empty()) return e;
    if (!(e = ternary(p + "attn_v.weight", D, Hkv * d, &tv)).empty()) return e;
    if (!(e = ternary(p + "attn_output.weight", H * d, D, &to)).empty()) return e;
    if (!(e = ternary(p + "ffn_up.weight", D, F, &tu)).empty()) return e;
    if (!(e = ternary(p + "ffn_down.weight", F, D, &td)).empty()) return e;
    if (c.gated && !(e = ternary(p + "ffn_gate.weight", D, F, &tg)).empty()) return e;

    // q|k|v on the block's input RMSNorm (transformer.rs:59-61, config eps)
    const uint8_t* qkv_t[3] = {tq.p, tk.p, tv.p};
    const size_t qkv_b[3] = {tq.bytes, tk.bytes, tv.bytes};
    const int qkv_m[3] = {H * d, Hkv * d, Hkv * d};
    if (obn_bitlinear_load_i2s_concat(3, qkv_t, qkv_b, qkv_m, D, attn_norm.data(), c.eps, device_,
                                      &L.qkv) != OBN_OK)
      return obn_fail(("loading " + p + "attn_q|k|v").c_str());
    // o_proj with the attention sub-norm as its own RMSNorm (model.rs:105-112; eps 1e-5)
    if (obn_bitlinear_load_i2s(to.p, to.bytes, H * d, D, attn_sub.empty() ? nullptr : attn_sub.data(),
                               1e-5f, device_, &L.o) != OBN_OK)
      return obn_fail(("loading " + p + "attn_output").c_str());
    if (c.gated) {  // gate|up on post_attention_layernorm (config eps), ffn.rs:64-80
      if (obn_bitlinear_load_i2s_gated(tg.p, tg.bytes, tu.p, tu.bytes, D, F, ffn_norm.data(),
                                       c.eps, device_, &L.ffn_in) != OBN_OK)
        return obn_fail(("loading " + p + "ffn_gate|up").c_str());
      if (obn_bitlinear_set_activation(L.ffn_in, static_cast<int>(c.act)) != OBN_OK)
        return obn_fail("setting the FFN activation");
    } else {
      if (obn_bitlinear_load_i2s(tu.p, tu.bytes, D, F, ffn_norm.data(), c.eps, device_,
                                 &L.ffn_in) != OBN_OK)
        return obn_fail(("loading " + p + "ffn_up").c_str());
    }
    if (obn_bitlinear_load_i2s(td.p, td.bytes, F, D, ffn_sub.empty() ? nullptr : ffn_sub.data(),
                               1e-5f, device_, &L.down) != OBN_OK)
      return obn_fail(("loading " + p + "ffn_down").c_str());
    tick(9 + (c.gated ? 1 : 0) + (attn_sub.empty() ? 0 : 1) + (ffn_sub.empty() ? 0 : 1));
  }

  // Embedding (binary16 [vocab][hidden]), final norm, LM head (model.rs:190-198).
  {
    const gguf::TensorInfo* ti;
    const uint8_t* p = nullptr;
    size_t bytes = 0;
    if (!(e = find("token_embd.weight", true, &ti, &p, &bytes)).empty()) return e;
    if (ti->type != gguf::kTypeF16)
      return fmt("unsupported model: token_embd.weight has GGML type %u (F16 expected)", ti->type);
    if (ti->shape.size() < 2 || ti->shape[0] != static_cast<uint64_t>(D) ||
        ti->shape[1] != static_cast<uint64_t>(c.vocab))
      return fmt("token_embd.weight is not [%d, %d]", D, c.vocab);
    const size_t tb = static_cast<size_t>(c.vocab) * D * 2;
    if ((ce = cudaMalloc(&embed_, tb)) != cudaSuccess) return cuda_fail(ce, "embedding allocation");
    if ((ce = cudaMemcpy(embed_, p, tb, cudaMemcpyHostToDevice)) != cudaSuccess)
      return cuda_fail(ce, "embedding upload");
    tick(1);
  }
  std::vector<float> fnorm;
  if (!(e = vec_f32("output_norm.weight", true, D, &fnorm)).empty()) return e;
  if ((ce = cudaMalloc(&final_norm_, sizeof(float) * D)) != cudaSuccess)
    return cuda_fail(ce, "final norm allocation");
  if ((ce = cudaMemcpy(final_norm_, fnorm.data(), sizeof(float) * D, cudaMemcpyHostToDevice)) !=
      cudaSuccess)
    return cuda_fail(ce, "final norm upload");
  tick(1);
  if (!c.tied) {
    const gguf::TensorInfo* ti;
    const uint8_t* p = nullptr;
    size_t bytes = 0;
    if (!(e = find("output.weight", true, &ti, &p, &bytes)).empty()) return e;
    if (ti->shape.size() < 2 || ti->shape[0] != static_cast<uint64_t>(D) ||
        ti->shape[1] != static_cast<uint64_t>(c.vocab))
      return fmt("output.weight is not [%d, %d]", D, c.vocab);
    if (ti->type == gguf::kTypeF16) {  // loader.rs:150-152: an untied f16 head
      cfg_.lm_head_f16 = true;
      const size_t tb = static_cast<size_t>(c.vocab) * D * 2;
      if ((ce = cudaMalloc(&lm_f16_, tb)) != cudaSuccess) return cuda_fail(ce, "LM head allocation");
      if ((ce = cudaMemcpy(lm_f16_, p, tb, cudaMemcpyHostToDevice)) != cudaSuccess)
        return cuda_fail(ce, "LM head upload");
    } else if (ti->type == gguf::kTypeI2_S) {  // model.rs:181-189: a ternary BitLinear head
      if (obn_bitlinear_load_i2s(p, bytes, D, c.vocab, fnorm.data(), 1e-5f, device_,
                                 &lm_ternary_) != OBN_OK)
        return obn_fail("loading output.weight");
    } else {
      return fmt("unsupported model: output.weight has GGML type %u (F16 or I2_S expected)",
                 ti->type);
    }
    tick(1);
  }

  // KV caches and activations for kChunk tokens.
  const size_t cache_bytes = static_cast<size_t>(kMaxSeq) * Hkv * d * 2;
  k_cache_.assign(c.layers, nullptr);
  v_cache_.assign(c.layers, nullptr);
  for (int i = 0; i < c.layers; ++i) {
    if ((ce = cudaMalloc(&k_cache_[i], cache_bytes)) != cudaSuccess ||
        (ce = cudaMalloc(&v_cache_[i], cache_bytes)) != cudaSuccess)
      return cuda_fail(ce, "KV cache allocation");
  }
  const size_t n = kChunk;
  struct Buf {
    float** p;
    size_t floats;
  } bufs[] = {{&x_, n * D}, {&qkv_, n * (H + 2 * Hkv) * d}, {&q_, n * H * d},
              {&attn_, n * H * d}, {&ffn_, n * F}, {&lm_in_, static_cast<size_t>(D)},
              {&logits_d_, static_cast<size_t>(c.vocab)}};
  for (Buf& b : bufs)
    if ((ce = cudaMalloc(reinterpret_cast<void**>(b.p), sizeof(float) * b.floats)) != cudaSuccess)
      return cuda_fail(ce, "activation allocation");
  if ((ce = cudaMalloc(&ids_d_, sizeof(int32_t) * n)) != cudaSuccess)
    return cuda_fail(ce, "id buffer allocation");
  size_t ws = 0;
  for (const Layer& L : layers_)
    for (const obn_bitlinear* b : {L.qkv, L.o, L.ffn_in, L.down}) {
      ws = std::max(ws, obn_bitlinear_workspace_bytes(b, kChunk));
      ws = std::max(ws, obn_bitlinear_workspace_bytes(b, 1));
    }
  if (lm_ternary_) ws = std::max(ws, obn_bitlinear_workspace_bytes(lm_ternary_, 1));
  ws_bytes_ = std::max<size_t>(ws, 256);
  if ((ce = cudaMalloc(&ws_, ws_bytes_)) != cudaSuccess) return cuda_fail(ce, "workspace allocation");
  attn_ws_bytes_ = std::max<size_t>(obn_attention_workspace_bytes(1, kChunk, H, d, kMaxSeq), 256);
  if ((ce = cudaMalloc(&attn_ws_, attn_ws_bytes_)) != cudaSuccess)
    return cuda_fail(ce, "attention workspace allocation");
  const size_t sel_bytes = 16 + static_cast<size_t>(kSelCap) * 8;
  if ((ce = cudaMallocHost(&logits_h_, sizeof(float) * c.vocab)) != cudaSuccess ||
      (ce = cudaMallocHost(&ids_h_, sizeof(int32_t) * kChunk)) != cudaSuccess ||
      (ce = cudaMallocHost(&recent_h_, sizeof(uint32_t) * kMaxSeq)) != cudaSuccess ||
      (ce = cudaMallocHost(&sel_h_, sel_bytes)) != cudaSuccess)
    return cuda_fail(ce, "pinned host buffers");
  if ((ce = cudaMalloc(&recent_d_, sizeof(uint32_t) * kMaxSeq)) != cudaSuccess ||
      (ce = cudaMalloc(&sel_d_, sel_bytes)) != cudaSuccess ||
      (ce = cudaMalloc(&sel_scratch_d_, select_topk_scratch_bytes(c.vocab))) != cudaSuccess ||
      (ce = cudaMalloc(&step_d_, 2 * sizeof(int32_t))) != cudaSuccess ||
      (ce = cudaMallocHost(&step_h_, 2 * sizeof(int32_t))) != cudaSuccess)
    return cuda_fail(ce, "sampling buffers");
  const char* g = std::getenv("OXBITNET_CUDA_GRAPH");  // "0" runs every step eagerly
  use_graph_ = !(g && g[0] == '0');
  if ((ce = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(ce, "model upload");
  progress(2, total, total, 1.0);
  log(2, fmt("%llu tensors loaded", static_cast<unsigned long long>(total)));
  return std::string();
}

std::string Model::forward(const uint32_t* ids, int n, bool copy_logits) {
  if (n <= 0) return "forward needs at least one token";
  if (pos_ + n > kMaxSeq)
    return fmt("context full: %d positions + %d new tokens exceed the %d-position KV cache", pos_,
               n, kMaxSeq);
  int done = 0;
  while (done < n) {
    int len = std::min(kChunk, n - done);
    // Keep every chunk of a multi-token input at >= 2 tokens, so each prompt token
    // takes the n > 1 (GEMM) epilogue order as in one reference forward.
    if (n > 1 && n - done - len == 1) --len;
    std::string e = run_chunk(ids + done, len, done + len == n, copy_logits);
    if (!e.empty()) return e;
    done += len;
  }
  return std::string();
}

// Enqueues the forward of n tokens whose ids are at ids_dev. pos_dev == nullptr:
// the first token sits at pos_ (host value); else at *pos_dev (read by the
// kernels, for the captured decode step). With want_logits the last token's
// logits land in logits_d_.
std::string Model::enqueue(int n, const int32_t* ids_dev, const int* pos_dev, bool want_logits) {
  return enqueue_part(n, ids_dev, pos_dev, want_logits, 0, static_cast<int>(layers_.size()));
}

// The forward's launches for layers [first, last): the embedding when first is 0,
// the final norm and the LM head (want_logits) when last is the layer count.
std::string Model::enqueue_part(int n, const int32_t* ids_dev, const int* pos_dev,
                                bool want_logits, int first, int last) {
  const ModelConfig& c = cfg_;
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  const int D = c.hidden, H = c.heads, Hkv = c.kv_heads, d = c.head_dim;
  const float scale = 1.0f / std::sqrt(static_cast<float>(d));  // attention.rs:206
  const int seq = pos_ + n;
  if (first == 0 &&
      obn_embed_f16(embed_, c.vocab, D, ids_dev, n, x_, s) != OBN_OK)
    return obn_fail("embedding");
  for (size_t i = static_cast<size_t>(first); i < static_cast<size_t>(last); ++i) {
    const Layer& L = layers_[i];
    if (obn_bitlinear_forward(L.qkv, x_, n, qkv_, ws_, ws_bytes_, s) != OBN_OK)
      return obn_fail("q|k|v projection");
    if (n == 1) {  // decode: RoPE + KV append fused into the attention pass
      const int rc =
          pos_dev ? obn_attention_decode_rope_at(qkv_, k_cache_[i], v_cache_[i], 1, H, Hkv, d,
                                                 kMaxSeq, pos_dev, c.rope_theta, scale, attn_,
                                                 attn_ws_, attn_ws_bytes_, s)
                  : obn_attention_decode_rope(qkv_, k_cache_[i], v_cache_[i], 1, H, Hkv, d,
                                              kMaxSeq, pos_, c.rope_theta, scale, attn_,
                                              attn_ws_, attn_ws_bytes_, s);
      if (rc != OBN_OK) return obn_fail("RoPE + attention");
    } else if (pos_dev) {
      if (obn_rope_kv_append_at(qkv_, 1, n, H, Hkv, d, pos_dev, c.rope_theta, q_, k_cache_[i],
                                v_cache_[i], kMaxSeq, s) != OBN_OK)
        return obn_fail("RoPE + KV append");
      if (obn_attention_decode_at(q_, k_cache_[i], v_cache_[i], 1, n, H, Hkv, d, kMaxSeq, pos_dev,
                                  scale, attn_, attn_ws_, attn_ws_bytes_, s) != OBN_OK)
        return obn_fail("attention");
    } else {
      if (obn_rope_kv_append(qkv_, 1, n, H, Hkv, d, pos_, c.rope_theta, q_, k_cache_[i],
                             v_cache_[i], kMaxSeq, s) != OBN_OK)
        return obn_fail("RoPE + KV append");
      if (obn_attention_decode(q_, k_cache_[i], v_cache_[i], 1, n, H, Hkv, d, kMaxSeq, seq,
                               scale, attn_, attn_ws_, attn_ws_bytes_, s) != OBN_OK)
        return obn_fail("attention");
    }
    if (obn_bitlinear_forward_residual(L.o, attn_, n, x_, ws_, ws_bytes_, s) != OBN_OK)
      return obn_fail("o_proj + residual");
    if (obn_bitlinear_forward(L.ffn_in, x_, n, ffn_, ws_, ws_bytes_, s) != OBN_OK)
      return obn_fail("FFN input projection");
    if (!c.gated &&
        obn_activation(ffn_, static_cast<size_t>(n) * c.ffn, static_cast<int>(c.act), ffn_, s) !=
            OBN_OK)
      return obn_fail("FFN activation");
    if (obn_bitlinear_forward_residual(L.down, ffn_, n, x_, ws_, ws_bytes_, s) != OBN_OK)
      return obn_fail("down_proj + residual");
  }
  if (!want_logits || last < static_cast<int>(layers_.size())) return std::string();
  // model.rs:235-262: final RMSNorm and the LM head on the last position only.
  const float* x_last = x_ + static_cast<size_t>(n - 1) * D;
  if (lm_ternary_) {
    if (obn_rmsnorm(x_last, final_norm_, c.eps, 1, D, lm_in_, s) != OBN_OK)
      return obn_fail("final norm");
    if (obn_bitlinear_forward(lm_ternary_, lm_in_, 1, logits_d_, ws_, ws_bytes_, s) != OBN_OK)
      return obn_fail("LM head");
  } else {
    const void* table = lm_f16_ ? lm_f16_ : embed_;
    if (obn_lm_head_f16(table, c.vocab, D, x_last, final_norm_, c.eps, 1, logits_d_, s) != OBN_OK)
      return obn_fail("LM head");
  }
  return std::string();
}

std::string Model::run_chunk(const uint32_t* ids, int n, bool want_logits, bool copy_logits) {
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device_) cudaSetDevice(device_);
  struct Restore {
    int dev, cur;
    ~Restore() {
      if (dev != cur) cudaSetDevice(dev);
    }
  } restore{prev, device_};
  cudaError_t ce = cudaStreamSynchronize(s);  // the pinned input buffers are free again
  if (ce != cudaSuccess) return cuda_fail(ce, "stream");
  std::string e;
  if (n == 1 && want_logits && use_graph_) {
    // One decode step: the token and its position go to the device, then the
    // whole step (every layer and the LM head) is one graph launch. The graph
    // is captured at the second step (the first one, eager, has set up every
    // kernel's attributes) and serves every later position.
    step_h_[0] = static_cast<int32_t>(ids[0]);
    step_h_[1] = pos_;
    ce = cudaMemcpyAsync(step_d_, step_h_, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) return cuda_fail(ce, "step upload");
    if (!decode_exec_[0] && decode_steps_ >= 1) {
      // Three graphs of growing size: launching a graph costs the host ~0.9 us
      // per kernel, so the next piece is launched while the previous one runs
      // and only the small first piece's launch is exposed after sampling. A
      // capture that fails (nothing was enqueued: the stream was capturing)
      // leaves the model on eager steps.
      const int L = static_cast<int>(layers_.size());
      const int cut[4] = {0, std::min(1, L), std::min(6, L), L};
      bool ok = true;
      for (int g = 0; g < 3 && ok; ++g) {
        cudaGraph_t gr = nullptr;
        cudaGraphExec_t ge = nullptr;
        ok = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
        if (ok) {
          ok = enqueue_part(1, step_d_, step_d_ + 1, true, cut[g], cut[g + 1]).empty();
          ok = cudaStreamEndCapture(s, &gr) == cudaSuccess && ok;
          ok = ok && cudaGraphInstantiate(&ge, gr, 0) == cudaSuccess;
          if (gr) cudaGraphDestroy(gr);
        }
        decode_exec_[g] = ok ? ge : nullptr;
      }
      if (!ok) {
        for (int g = 0; g < 3; ++g) {
          if (decode_exec_[g]) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(decode_exec_[g]));
          decode_exec_[g] = nullptr;
        }
        use_graph_ = false;
        cudaGetLastError();
      }
    }
    if (decode_exec_[0]) {
      for (int g = 0; g < 3; ++g) {
        ce = cudaGraphLaunch(static_cast<cudaGraphExec_t>(decode_exec_[g]), s);
        if (ce != cudaSuccess) return cuda_fail(ce, "graph launch");
      }
    } else {
      e = enqueue(1, step_d_, step_d_ + 1, true);
      if (!e.empty()) return e;
    }
    ++decode_steps_;
  } else {
    for (int t = 0; t < n; ++t) ids_h_[t] = static_cast<int32_t>(ids[t]);
    ce = cudaMemcpyAsync(ids_d_, ids_h_, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) return cuda_fail(ce, "token upload");
    e = enqueue(n, ids_d_, nullptr, want_logits);
    if (!e.empty()) return e;
  }
  pos_ += n;  // model.rs:231-232: the cache now holds the chunk
  if (!want_logits || !copy_logits) return std::string();
  return logits_to_host();
}

std::string Model::logits_to_host() {
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  cudaError_t ce = cudaMemcpyAsync(logits_h_, logits_d_, sizeof(float) * cfg_.vocab,
                                   cudaMemcpyDeviceToHost, s);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) return cuda_fail(ce, "logits read-back");
  if (obn_check_device_errors() != OBN_OK) return obn_fail("device-side check");
  return std::string();
}

std::string Model::sample(float temperature, size_t top_k, float repeat_penalty,
                          const uint32_t* recent, size_t n_recent, float u, uint32_t* out) {
  const size_t V = static_cast<size_t>(cfg_.vocab);
  const bool greedy = !(temperature > 0.0f);
  const size_t k = greedy ? 1 : top_k;
  if (k == 0 || k >= V || k > kSelCap / 2 || n_recent > static_cast<size_t>(kMaxSeq)) {
    std::string e = logits_to_host();  // the whole vocabulary on the host
    if (!e.empty()) return e;
    *out = sample_logits(logits_h_, V, temperature, top_k, repeat_penalty, recent, n_recent, u);
    return std::string();
  }
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device_) cudaSetDevice(device_);
  struct Restore {
    int dev, cur;
    ~Restore() {
      if (dev != cur) cudaSetDevice(dev);
    }
  } restore{prev, device_};
  cudaStream_t s = static_cast<cudaStream_t>(stream_);
  cudaError_t ce = cudaSuccess;
  const bool penalise = repeat_penalty != 1.0f && n_recent > 0;
  if (penalise) {
    std::memcpy(recent_h_, recent, sizeof(uint32_t) * n_recent);
    ce = cudaMemcpyAsync(recent_d_, recent_h_, sizeof(uint32_t) * n_recent,
                         cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) return cuda_fail(ce, "penalty window upload");
  }
  int* count_d = static_cast<int*>(sel_d_);
  uint2* pairs_d = reinterpret_cast<uint2*>(static_cast<uint8_t*>(sel_d_) + 16);
  ce = launch_select_topk(logits_d_, cfg_.vocab, recent_d_, penalise ? static_cast<int>(n_recent) : 0,
                          penalise ? repeat_penalty : 1.0f, temperature, static_cast<int>(k),
                          pairs_d, kSelCap, count_d, sel_scratch_d_, s);
  if (ce != cudaSuccess) return cuda_fail(ce, "top-k launch");
  // The count and the first 4k + 256 pairs (ties past that need a second copy).
  const size_t first = std::min<size_t>(kSelCap, 4 * k + 256);
  ce = cudaMemcpyAsync(sel_h_, sel_d_, 16 + first * 8, cudaMemcpyDeviceToHost, s);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) return cuda_fail(ce, "top-k read-back");
  const int count = *static_cast<const int*>(sel_h_);
  if (count > static_cast<int>(first) && count <= kSelCap) {
    ce = cudaMemcpy(static_cast<uint8_t*>(sel_h_) + 16 + first * 8,
                    static_cast<uint8_t*>(sel_d_) + 16 + first * 8, (count - first) * 8,
                    cudaMemcpyDeviceToHost);
    if (ce != cudaSuccess) return cuda_fail(ce, "top-k read-back");
  }
  if (count <= 0 || count > kSelCap) {  // more ties than the buffer holds: host path
    std::string e = logits_to_host();   // the penalty is already applied
    if (!e.empty()) return e;
    *out = sample_logits(logits_h_, V, temperature, top_k, 1.0f, nullptr, 0, u);
    return std::string();
  }
  const uint32_t* pr = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(sel_h_) + 16);
  std::vector<std::pair<uint32_t, float>> surv(count);
  for (int i = 0; i < count; ++i) {
    float v;
    std::memcpy(&v, pr + 2 * i + 1, 4);
    surv[i] = {pr[2 * i], v};
  }
  std::sort(surv.begin(), surv.end());
  if (greedy) {  // the first index among the maxima
    *out = surv.front().first;
    return std::string();
  }
  // sampling.rs:62-76 over the survivors in index order; the masked logits
  // contribute exp(-inf) = 0 to every sum, which leaves it unchanged.
  float max_val = -std::numeric_limits<float>::infinity();
  for (const auto& p : surv) max_val = std::fmax(max_val, p.second);
  std::vector<float> e(count);
  float sum = 0.0f;
  for (int i = 0; i < count; ++i) {
    e[i] = std::exp(surv[i].second - max_val);
    sum += e[i];
  }
  const float r = u * sum;
  if (!(r > 0.0f)) {  // r = 0: the running sum reaches it at index 0; NaN: never
    *out = r == 0.0f ? 0u : static_cast<uint32_t>(V - 1);
    return std::string();
  }
  float cumsum = 0.0f;
  for (int i = 0; i < count; ++i) {
    cumsum += e[i];
    if (cumsum >= r) {
      *out = surv[i].first;
      return std::string();
    }
  }
  *out = static_cast<uint32_t>(V - 1);
  return std::string();
}

}  // namespace obn
