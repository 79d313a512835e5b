// GGUF v3 container: a reader over caller-owned bytes and a writer.
// Follows the public GGUF v3 specification (magic "GGUF", version 3,
// little-endian, u64 counts, typed metadata, tensor infos, aligned data).
// The reference crate's GGUF parser lives in the un-vendored jero-core
// crate; this is an independent implementation of the same file format.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace jal {

enum GgufValueType : uint32_t {
  GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4,
  GGUF_I32 = 5, GGUF_F32 = 6, GGUF_BOOL = 7, GGUF_STRING = 8,
  GGUF_ARRAY = 9, GGUF_U64 = 10, GGUF_I64 = 11, GGUF_F64 = 12
};

struct GgufValue {
  uint32_t type = GGUF_U32;
  uint64_t u = 0;        // unsigned / bool
  int64_t i = 0;         // signed
  double f = 0.0;        // float
  std::string s;         // string
  uint32_t arr_type = 0; // array element type
  std::vector<GgufValue> arr;

  bool as_usize(uint64_t *out) const;
  bool as_f32(float *out) const;
  bool is_string() const { return type == GGUF_STRING; }
};

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  uint64_t ne[4] = {1, 1, 1, 1};
  uint32_t type = 0;
  uint64_t offset = 0;       // relative to the data section
  const uint8_t *data = nullptr;
  size_t nbytes = 0;         // bytes available for this tensor
  uint64_t num_elements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

class GgufFile {
 public:
  // Parses `bytes` (not copied; must outlive the object). Throws JalError.
  GgufFile(const uint8_t *bytes, size_t len);
  const std::string &architecture() const { return arch_; }
  const GgufValue *value(const std::string &key) const;
  const GgufTensor *tensor(const std::string &name) const;
  bool contains(const std::string &name) const { return tensor(name) != nullptr; }
  size_t tensor_count() const { return tensors_.size(); }
  const std::vector<GgufTensor> &tensors() const { return tensors_; }

 private:
  std::string arch_;
  std::map<std::string, GgufValue> kv_;
  std::vector<GgufTensor> tensors_;
  std::map<std::string, size_t> index_;
};

// Bytes per row of `cols` elements for a GGML type (0 if unsupported or
// misaligned). Mirrors quant_row_bytes (repack_cache.rs:1065-1073) plus the
// ternary types used by the streaming GEMV.
size_t ggml_row_bytes(uint32_t type, uint64_t cols);
bool ggml_block_geometry(uint32_t type, size_t *elems, size_t *bytes);

class GgufWriter {
 public:
  void add_u32(const std::string &k, uint32_t v);
  void add_f32(const std::string &k, float v);
  void add_string(const std::string &k, const std::string &v);
  void add_tensor(const std::string &name, uint32_t type,
                  std::vector<uint64_t> dims);
  size_t total_size() const;
  // Offset of tensor i's payload inside the file (after finalize layout).
  size_t tensor_file_offset(size_t i) const;
  size_t tensor_bytes(size_t i) const;
  // Writes header + metadata + tensor infos; payloads are written by the
  // caller at tensor_file_offset(i). Returns bytes written (header part).
  void write_header(uint8_t *buf, size_t len) const;
  size_t n_tensors() const { return infos_.size(); }
  const std::string &tensor_name(size_t i) const { return infos_[i].name; }
  uint32_t tensor_type(size_t i) const { return infos_[i].type; }
  const std::vector<uint64_t> &tensor_dims(size_t i) const { return infos_[i].dims; }

 private:
  struct Kv { std::string key; uint32_t type; uint32_t u; float f; std::string s; };
  struct Info { std::string name; uint32_t type; std::vector<uint64_t> dims; size_t bytes; };
  std::vector<Kv> kvs_;
  std::vector<Info> infos_;
  size_t header_size() const;
  static constexpr size_t kAlign = 32;
};

}  // namespace jal
