// gguf.h — GGUF v2/v3 container parser (host side of the model loader).
//
// Follows the reference's streaming parser (packages/rust/crates/oxbitnet/src/
// model/gguf.rs:140-323): little-endian header (magic "GGUF", version 2 or 3,
// tensor count, metadata count), typed metadata key/value pairs (arrays nest),
// tensor infos (name, dims, ggml type, offset), tensor data starting at the
// next multiple of general.alignment (default 32) after the infos. Error texts
// follow the reference's (error.rs:13-32).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace obn {
namespace gguf {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little-endian

// Metadata value types (gguf.rs:8-20).
enum ValueType : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6,
  kBool = 7, kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

// GGML tensor types the reference knows (gguf.rs:22-36).
enum GgmlType : uint32_t {
  kTypeF32 = 0, kTypeF16 = 1, kTypeI8 = 16, kTypeI16 = 17, kTypeI32 = 18,
  kTypeI64 = 27, kTypeF64 = 28, kTypeBF16 = 30, kTypeTQ1_0 = 34, kTypeTQ2_0 = 35,
  kTypeI2_S = 36,  // ternary, 2 bits per weight, + a 32-byte scale trailer
};

struct Value {
  uint32_t type = kU8;
  uint64_t u = 0;   // unsigned integers and bool
  int64_t i = 0;    // signed integers
  double f = 0.0;   // F32 / F64
  std::string s;    // kString
  uint32_t elem_type = kU8;
  std::vector<Value> arr;  // kArray

  // GgufValue::as_u32 (gguf.rs:85-93): U32, I32 (reinterpreted), U8, U16.
  bool as_u32(uint32_t* out) const;
  // GgufValue::as_f32 (gguf.rs:95-101): F32, F64 (narrowed).
  bool as_f32(float* out) const;
  const std::string* as_str() const { return type == kString ? &s : nullptr; }
  // GgufValue::as_string_array (gguf.rs:103-114): every element a string.
  bool as_string_array(std::vector<const std::string*>* out) const;
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> shape;  // ne[0] (innermost) first
  uint32_t type = 0;
  uint64_t offset = 0;          // from the start of the tensor data
  uint64_t elements() const;
};

struct File {
  uint32_t version = 0;
  uint64_t tensor_count = 0;
  std::unordered_map<std::string, Value> metadata;
  std::vector<std::string> key_order;  // metadata keys in file order
  std::vector<TensorInfo> tensors;
  size_t data_offset = 0;  // absolute offset of the tensor data section

  const Value* get(const std::string& key) const;
  const TensorInfo* tensor(const std::string& name) const;
};

// Parses the header, metadata and tensor infos of the GGUF bytes [0, size).
// Returns an empty string on success, else the error text.
std::string parse(const uint8_t* data, size_t size, File* out);

// Bytes of a tensor's data: ceil(n / 4) + 32 for I2_S (loader.rs:104-111),
// else ceil(n * type size) (gguf.rs:38-54). Empty error string on success.
std::string tensor_bytes(const TensorInfo& t, size_t* out);

}  // namespace gguf
}  // namespace obn
