// gguf.cpp — GGUF container parser (gguf.h).
#include "gguf.h"

#include <cmath>
#include <cstdio>
#include <cstring>

namespace obn {
namespace gguf {

bool Value::as_u32(uint32_t* out) const {
  switch (type) {
    case kU32: case kU8: case kU16: *out = static_cast<uint32_t>(u); return true;
    case kI32: *out = static_cast<uint32_t>(static_cast<int32_t>(i)); return true;
    default: return false;
  }
}

bool Value::as_f32(float* out) const {
  if (type == kF32 || type == kF64) {
    *out = static_cast<float>(f);
    return true;
  }
  return false;
}

bool Value::as_string_array(std::vector<const std::string*>* out) const {
  if (type != kArray) return false;
  out->clear();
  out->reserve(arr.size());
  for (const Value& v : arr) {
    if (v.type != kString) return false;
    out->push_back(&v.s);
  }
  return true;
}

uint64_t TensorInfo::elements() const {
  uint64_t n = 1;
  for (uint64_t d : shape) n *= d;
  return n;
}

const Value* File::get(const std::string& key) const {
  auto it = metadata.find(key);
  return it == metadata.end() ? nullptr : &it->second;
}

const TensorInfo* File::tensor(const std::string& name) const {
  for (const TensorInfo& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

namespace {

// Bounds-checked little-endian reader; the first failure is kept in `err`.
struct Reader {
  const uint8_t* data;
  size_t size;
  size_t off = 0;
  std::string err;

  bool ensure(size_t n) {
    if (!err.empty()) return false;
    if (n > size || off > size - n) {
      char buf[160];
      std::snprintf(buf, sizeof(buf),
                    "GGUF parse error: Unexpected EOF at offset %zu (need %zu bytes, have %zu)", off,
                    n, size);
      err = buf;
      return false;
    }
    return true;
  }
  template <typename T>
  T get() {
    T v{};
    if (!ensure(sizeof(T))) return v;
    std::memcpy(&v, data + off, sizeof(T));  // hosts are little-endian
    off += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!err.empty() || !ensure(static_cast<size_t>(n))) return std::string();
    std::string s(reinterpret_cast<const char*>(data + off), static_cast<size_t>(n));
    off += static_cast<size_t>(n);
    if (!valid_utf8(s)) {
      char buf[120];
      std::snprintf(buf, sizeof(buf), "GGUF parse error: Invalid UTF-8 in string at offset %zu",
                    off - static_cast<size_t>(n));
      err = buf;
    }
    return s;
  }
  static bool valid_utf8(const std::string& s) {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
    size_t i = 0, n = s.size();
    while (i < n) {
      const unsigned c = p[i];
      size_t len;
      uint32_t cp;
      if (c < 0x80) { ++i; continue; }
      if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
      else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
      else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
      else return false;
      if (i + len > n) return false;
      for (size_t k = 1; k < len; ++k) {
        if ((p[i + k] & 0xC0) != 0x80) return false;
        cp = (cp << 6) | (p[i + k] & 0x3F);
      }
      if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
          cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
        return false;
      i += len;
    }
    return true;
  }
};

bool read_value(Reader& r, uint32_t type, Value* v, int depth) {
  v->type = type;
  switch (type) {
    case kU8: v->u = r.get<uint8_t>(); break;
    case kI8: v->i = r.get<int8_t>(); break;
    case kU16: v->u = r.get<uint16_t>(); break;
    case kI16: v->i = r.get<int16_t>(); break;
    case kU32: v->u = r.get<uint32_t>(); break;
    case kI32: v->i = r.get<int32_t>(); break;
    case kF32: v->f = r.get<float>(); break;
    case kBool: v->u = r.get<uint8_t>() != 0; break;
    case kString: v->s = r.str(); break;
    case kU64: v->u = r.get<uint64_t>(); break;
    case kI64: v->i = r.get<int64_t>(); break;
    case kF64: v->f = r.get<double>(); break;
    case kArray: {
      if (depth > 8) {
        r.err = "GGUF parse error: arrays nested too deeply";
        return false;
      }
      v->elem_type = r.get<uint32_t>();
      const uint64_t len = r.get<uint64_t>();
      if (!r.err.empty()) return false;
      // Every element takes at least one byte: a longer array cannot fit.
      if (len > r.size - r.off) {
        r.ensure(static_cast<size_t>(len > SIZE_MAX ? SIZE_MAX : len));
        return false;
      }
      v->arr.resize(static_cast<size_t>(len));
      for (uint64_t k = 0; k < len; ++k)
        if (!read_value(r, v->elem_type, &v->arr[static_cast<size_t>(k)], depth + 1)) return false;
      break;
    }
    default: {
      char buf[80];
      std::snprintf(buf, sizeof(buf), "Unknown GGUF metadata type: %u", type);
      r.err = buf;
      return false;
    }
  }
  return r.err.empty();
}

}  // namespace

std::string parse(const uint8_t* data, size_t size, File* out) {
  Reader r{data, size, 0, std::string()};
  File f;
  const uint32_t magic = r.get<uint32_t>();
  if (!r.err.empty()) return r.err;
  if (magic != kMagic) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "Invalid GGUF magic: 0x%08x (expected 0x46554747)", magic);
    return buf;
  }
  f.version = r.get<uint32_t>();
  if (!r.err.empty()) return r.err;
  if (f.version < 2 || f.version > 3) {
    char buf[64];
    std::snprintf(buf, sizeof(buf), "Unsupported GGUF version: %u", f.version);
    return buf;
  }
  f.tensor_count = r.get<uint64_t>();
  const uint64_t kv_count = r.get<uint64_t>();
  if (!r.err.empty()) return r.err;
  for (uint64_t k = 0; k < kv_count; ++k) {
    std::string key = r.str();
    const uint32_t type = r.get<uint32_t>();
    if (!r.err.empty()) return r.err;
    Value v;
    if (!read_value(r, type, &v, 0)) return r.err;
    if (f.metadata.find(key) == f.metadata.end()) f.key_order.push_back(key);
    f.metadata[key] = std::move(v);  // a repeated key keeps the last value, as a map insert does
  }
  if (f.tensor_count > r.size - r.off) {  // each info takes more than one byte
    r.ensure(static_cast<size_t>(f.tensor_count > SIZE_MAX ? SIZE_MAX : f.tensor_count));
    return r.err;
  }
  f.tensors.resize(static_cast<size_t>(f.tensor_count));
  for (TensorInfo& t : f.tensors) {
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (!r.err.empty()) return r.err;
    if (nd > 8) return "GGUF parse error: tensor '" + t.name + "' has too many dimensions";
    t.shape.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) t.shape[d] = r.get<uint64_t>();
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    if (!r.err.empty()) return r.err;
  }
  uint32_t alignment = 32;  // gguf.rs:180-185
  if (const Value* a = f.get("general.alignment")) {
    uint32_t v;
    if (a->as_u32(&v)) alignment = v;
  }
  if (alignment == 0) return "GGUF parse error: general.alignment is 0";
  f.data_offset = (r.off + alignment - 1) / alignment * alignment;
  *out = std::move(f);
  return std::string();
}

std::string tensor_bytes(const TensorInfo& t, size_t* out) {
  const uint64_t n = t.elements();
  double per;
  switch (t.type) {
    case kTypeI2_S: *out = static_cast<size_t>((n + 3) / 4 + 32); return std::string();
    case kTypeF32: case kTypeI32: per = 4.0; break;
    case kTypeF16: case kTypeI16: case kTypeBF16: per = 2.0; break;
    case kTypeI8: per = 1.0; break;
    case kTypeI64: case kTypeF64: per = 8.0; break;
    case kTypeTQ1_0: per = 54.0 / 256.0; break;
    case kTypeTQ2_0: per = 66.0 / 256.0; break;
    default: {
      char buf[64];
      std::snprintf(buf, sizeof(buf), "Unsupported GGML type: %u", t.type);
      return buf;
    }
  }
  *out = static_cast<size_t>(std::ceil(static_cast<double>(n) * per));
  return std::string();
}

}  // namespace gguf
}  // namespace obn
