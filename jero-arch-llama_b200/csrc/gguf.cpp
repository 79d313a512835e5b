// GGUF v3 reader / writer (public GGUF v3 file-format specification).
#include "gguf.hpp"

#include <cstring>

#include "common.hpp"

namespace jal {

bool GgufValue::as_usize(uint64_t *out) const {
  switch (type) {
    case GGUF_U8: case GGUF_U16: case GGUF_U32: case GGUF_U64: case GGUF_BOOL:
      *out = u; return true;
    case GGUF_I8: case GGUF_I16: case GGUF_I32: case GGUF_I64:
      if (i < 0) return false;
      *out = (uint64_t)i; return true;
    default: return false;
  }
}

bool GgufValue::as_f32(float *out) const {
  switch (type) {
    case GGUF_F32: case GGUF_F64: *out = (float)f; return true;
    case GGUF_U8: case GGUF_U16: case GGUF_U32: case GGUF_U64: *out = (float)u; return true;
    case GGUF_I8: case GGUF_I16: case GGUF_I32: case GGUF_I64: *out = (float)i; return true;
    default: return false;
  }
}

bool ggml_block_geometry(uint32_t type, size_t *elems, size_t *bytes) {
  size_t e = 0, b = 0;
  switch (type) {
    case JAL_F32: e = 1; b = 4; break;
    case JAL_F16: case JAL_BF16: e = 1; b = 2; break;
    case JAL_Q4_0: e = 32; b = 18; break;
    case JAL_Q5_0: e = 32; b = 22; break;
    case JAL_Q8_0: e = 32; b = 34; break;
    case JAL_Q4_K: e = 256; b = 144; break;
    case JAL_Q5_K: e = 256; b = 176; break;
    case JAL_Q6_K: e = 256; b = 210; break;
    case JAL_TQ1_0: e = 256; b = 54; break;
    case JAL_TQ2_0: e = 256; b = 66; break;
    case 3: e = 32; b = 20; break;    // Q4_1 (sizes only; not admitted)
    case 7: e = 32; b = 24; break;    // Q5_1
    case 9: e = 32; b = 36; break;    // Q8_1
    case 10: e = 256; b = 84; break;  // Q2_K
    case 11: e = 256; b = 110; break; // Q3_K
    default: return false;
  }
  if (elems) *elems = e;
  if (bytes) *bytes = b;
  return true;
}

size_t ggml_row_bytes(uint32_t type, uint64_t cols) {
  size_t e, b;
  if (!ggml_block_geometry(type, &e, &b) || cols == 0 || cols % e) return 0;
  return (size_t)(cols / e) * b;
}

namespace {
struct Reader {
  const uint8_t *p;
  size_t len, pos = 0;
  void need(size_t n) {
    if (pos + n > len || pos + n < pos) fail(JAL_ERR_TENSOR_BOUNDS, "GGUF truncated at byte %zu", pos);
  }
  template <class T> T get() { need(sizeof(T)); T v; memcpy(&v, p + pos, sizeof(T)); pos += sizeof(T); return v; }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (n > (1ull << 30)) fail(JAL_ERR_TENSOR_BOUNDS, "GGUF string too long");
    need((size_t)n);
    std::string s((const char *)p + pos, (size_t)n);
    pos += (size_t)n;
    return s;
  }
  GgufValue value(uint32_t type, int depth = 0) {
    GgufValue v;
    v.type = type;
    switch (type) {
      case GGUF_U8: v.u = get<uint8_t>(); break;
      case GGUF_I8: v.i = get<int8_t>(); break;
      case GGUF_U16: v.u = get<uint16_t>(); break;
      case GGUF_I16: v.i = get<int16_t>(); break;
      case GGUF_U32: v.u = get<uint32_t>(); break;
      case GGUF_I32: v.i = get<int32_t>(); break;
      case GGUF_F32: v.f = get<float>(); break;
      case GGUF_BOOL: v.u = get<uint8_t>() ? 1 : 0; break;
      case GGUF_STRING: v.s = str(); break;
      case GGUF_U64: v.u = get<uint64_t>(); break;
      case GGUF_I64: v.i = get<int64_t>(); break;
      case GGUF_F64: v.f = get<double>(); break;
      case GGUF_ARRAY: {
        if (depth > 2) fail(JAL_ERR_TENSOR_BOUNDS, "GGUF nested array too deep");
        v.arr_type = get<uint32_t>();
        uint64_t n = get<uint64_t>();
        if (n > len) fail(JAL_ERR_TENSOR_BOUNDS, "GGUF array too long");
        v.arr.reserve((size_t)n);
        for (uint64_t k = 0; k < n; k++) v.arr.push_back(value(v.arr_type, depth + 1));
        break;
      }
      default: fail(JAL_ERR_TENSOR_BOUNDS, "GGUF unknown value type %u", type);
    }
    return v;
  }
};
}  // namespace

GgufFile::GgufFile(const uint8_t *bytes, size_t len) {
  if (!bytes) fail(JAL_ERR_INVALID_ARGUMENT, "null GGUF buffer");
  Reader r{bytes, len};
  uint32_t magic = r.get<uint32_t>();
  if (magic != 0x46554747u) fail(JAL_ERR_TENSOR_BOUNDS, "not a GGUF file (bad magic)");
  uint32_t version = r.get<uint32_t>();
  if (version != 3 && version != 2) fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported GGUF version %u", version);
  uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
  if (n_tensors > (1u << 24) || n_kv > (1u << 24)) fail(JAL_ERR_TENSOR_BOUNDS, "GGUF counts implausible");
  for (uint64_t k = 0; k < n_kv; k++) {
    std::string key = r.str();
    uint32_t type = r.get<uint32_t>();
    kv_[key] = r.value(type);
  }
  tensors_.reserve((size_t)n_tensors);
  for (uint64_t t = 0; t < n_tensors; t++) {
    GgufTensor ti;
    ti.name = r.str();
    ti.n_dims = r.get<uint32_t>();
    if (ti.n_dims == 0 || ti.n_dims > 4) fail(JAL_ERR_TENSOR_BOUNDS, "tensor '%s' has %u dims", ti.name.c_str(), ti.n_dims);
    for (uint32_t d = 0; d < ti.n_dims; d++) ti.ne[d] = r.get<uint64_t>();
    ti.type = r.get<uint32_t>();
    ti.offset = r.get<uint64_t>();
    tensors_.push_back(ti);
  }
  uint64_t align = 32;
  auto it = kv_.find("general.alignment");
  if (it != kv_.end()) {
    uint64_t a;
    if (it->second.as_usize(&a) && a > 0 && (a & (a - 1)) == 0) align = a;
  }
  size_t data_start = (r.pos + align - 1) / align * align;
  for (size_t t = 0; t < tensors_.size(); t++) {
    GgufTensor &ti = tensors_[t];
    size_t start = data_start + ti.offset;
    if (start > len) fail(JAL_ERR_TENSOR_BOUNDS, "tensor '%s' offset beyond file", ti.name.c_str());
    ti.data = bytes + start;
    // Bytes up to the next tensor's start (or the file end) are available.
    size_t end = len;
    for (const GgufTensor &o : tensors_)
      if (o.offset > ti.offset && data_start + o.offset < end) end = data_start + o.offset;
    ti.nbytes = end - start;
    index_[ti.name] = t;
  }
  auto a = kv_.find("general.architecture");
  if (a != kv_.end() && a->second.is_string()) arch_ = a->second.s;
}

const GgufValue *GgufFile::value(const std::string &key) const {
  auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}

const GgufTensor *GgufFile::tensor(const std::string &name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

// ---- writer ---------------------------------------------------------------

void GgufWriter::add_u32(const std::string &k, uint32_t v) { kvs_.push_back({k, GGUF_U32, v, 0.f, {}}); }
void GgufWriter::add_f32(const std::string &k, float v) { kvs_.push_back({k, GGUF_F32, 0, v, {}}); }
void GgufWriter::add_string(const std::string &k, const std::string &v) { kvs_.push_back({k, GGUF_STRING, 0, 0.f, v}); }

void GgufWriter::add_tensor(const std::string &name, uint32_t type, std::vector<uint64_t> dims) {
  uint64_t rest = 1;
  for (size_t i = 1; i < dims.size(); i++) rest *= dims[i];
  size_t rb = ggml_row_bytes(type, dims[0]);
  if (!rb) fail(JAL_ERR_TENSOR_BOUNDS, "tensor '%s': cols %llu incompatible with type %u", name.c_str(),
                (unsigned long long)dims[0], type);
  infos_.push_back({name, type, std::move(dims), (size_t)(rb * rest)});
}

size_t GgufWriter::header_size() const {
  size_t n = 4 + 4 + 8 + 8;
  for (const Kv &k : kvs_) {
    n += 8 + k.key.size() + 4;
    n += k.type == GGUF_STRING ? 8 + k.s.size() : 4;
  }
  for (const Info &t : infos_) n += 8 + t.name.size() + 4 + 8 * t.dims.size() + 4 + 8;
  return (n + kAlign - 1) / kAlign * kAlign;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t GgufWriter::tensor_file_offset(size_t i) const {
  size_t off = header_size();
  for (size_t k = 0; k < i; k++) off = align_up(off + infos_[k].bytes, kAlign);
  return off;
}

size_t GgufWriter::tensor_bytes(size_t i) const { return infos_[i].bytes; }

size_t GgufWriter::total_size() const {
  if (infos_.empty()) return header_size();
  return tensor_file_offset(infos_.size() - 1) + infos_.back().bytes;
}

void GgufWriter::write_header(uint8_t *buf, size_t len) const {
  size_t pos = 0;
  auto put = [&](const void *src, size_t n) {
    if (pos + n > len) fail(JAL_ERR_TENSOR_BOUNDS, "GGUF writer buffer too small");
    memcpy(buf + pos, src, n);
    pos += n;
  };
  auto put_str = [&](const std::string &s) { uint64_t n = s.size(); put(&n, 8); put(s.data(), s.size()); };
  uint32_t magic = 0x46554747u, version = 3;
  uint64_t nt = infos_.size(), nk = kvs_.size();
  put(&magic, 4); put(&version, 4); put(&nt, 8); put(&nk, 8);
  for (const Kv &k : kvs_) {
    put_str(k.key);
    put(&k.type, 4);
    if (k.type == GGUF_STRING) put_str(k.s);
    else if (k.type == GGUF_F32) put(&k.f, 4);
    else put(&k.u, 4);
  }
  size_t data_start = header_size(), rel = 0;
  for (size_t i = 0; i < infos_.size(); i++) {
    const Info &t = infos_[i];
    put_str(t.name);
    uint32_t nd = (uint32_t)t.dims.size();
    put(&nd, 4);
    for (uint64_t d : t.dims) put(&d, 8);
    put(&t.type, 4);
    uint64_t off = tensor_file_offset(i) - data_start;
    put(&off, 8);
    rel = off;
  }
  (void)rel;
  while (pos < data_start) { uint8_t z = 0; put(&z, 1); }
}

}  // namespace jal
