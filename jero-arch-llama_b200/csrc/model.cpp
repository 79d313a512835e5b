// Recipe hydration, ModelRepackCache build, execution context and the
// decode / prefill step sequences.  File:line citations refer to the
// reference crate.
#include <atomic>
#include "model.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.hpp"

namespace jal {

// ---------------------------------------------------------------------------
// Recipe
// ---------------------------------------------------------------------------

Recipe Recipe::for_arch(const std::string &arch) {  // recipe.rs:163-222
  Recipe r;
  if (arch == "qwen2") {
    r.architecture = "qwen2";
    r.num_layers = 28; r.hidden_dim = 1536; r.ffn_dim = 8960; r.n_heads_q = 12; r.n_heads_kv = 2;
    r.head_dim = 128; r.vocab_size = 151936; r.rms_eps = 1e-6f; r.rope_theta = 1000000.f;
    r.rope_type = JAL_ROPE_NEOX;
  } else {
    r.architecture = arch == "llama4" ? "llama4" : "llama";
  }
  return r;
}

bool Recipe::should_skip_rope(size_t layer) const {  // recipe.rs:466-472
  return has_irope_mask && layer < irope_mask.size() && irope_mask[layer];
}

bool Recipe::supports_quant(int q) const {  // recipe.rs:1819-1832
  switch (q) {
    case JAL_F32: case JAL_F16: case JAL_BF16: case JAL_Q4_K: case JAL_Q5_K: case JAL_Q5_0:
    case JAL_Q8_0: case JAL_Q4_0: case JAL_Q6_K: return true;
    default: return false;
  }
}

namespace {

bool meta_usize(const GgufFile &g, const std::string &k, uint64_t *out) {
  const GgufValue *v = g.value(k);
  return v && v->as_usize(out);
}
bool meta_f32(const GgufFile &g, const std::string &k, float *out) {
  const GgufValue *v = g.value(k);
  return v && v->as_f32(out);
}

// infer_descriptor_rows (recipe.rs:3065-3077)
bool infer_rows(const GgufTensor *t, uint64_t expected_cols, uint64_t *rows) {
  if (!t || t->n_dims != 2) return false;
  if (t->ne[0] == expected_cols) { *rows = t->ne[1]; return true; }
  if (t->ne[1] == expected_cols) { *rows = t->ne[0]; return true; }
  return false;
}

// resolve_2d_dims (repack_cache.rs:1094-1158)
void resolve_2d(const GgufTensor *t, uint64_t expected_cols, uint64_t *rows, uint64_t *cols) {
  if (t->n_dims != 2) fail(JAL_ERR_TENSOR_BOUNDS, "%s: expected 2D tensor", t->name.c_str());
  uint64_t d0 = t->ne[0], d1 = t->ne[1];
  if (d0 == expected_cols) { *rows = d1; *cols = d0; }
  else if (d1 == expected_cols) { *rows = d0; *cols = d1; }
  else fail(JAL_ERR_TENSOR_BOUNDS, "2D tensor %s shape [%llu, %llu] does not match expected cols %llu", t->name.c_str(),
            (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)expected_cols);
  size_t rb = ggml_row_bytes(t->type, *cols);
  if (!rb) fail(JAL_ERR_TENSOR_BOUNDS, "cols %llu incompatible with quant %u on tensor '%s'", (unsigned long long)*cols,
                t->type, t->name.c_str());
  if (t->nbytes < *rows * rb) fail(JAL_ERR_TENSOR_BOUNDS, "tensor '%s' buffer smaller than required", t->name.c_str());
}

std::string key(size_t l, const char *suffix) { return "blk." + std::to_string(l) + "." + suffix; }

// probe_live_layer_count (decode_gemv.rs:148-166)
uint64_t probe_layers(const GgufFile &g) {
  uint64_t probed = 0;
  for (size_t l = 0; l < 512; l++) {
    bool has = g.contains(key(l, "attn_norm.weight")) || g.contains(key(l, "attn_q.weight")) ||
               g.contains(key(l, "ffn_gate.weight")) || g.contains(key(l, "attn_output.weight"));
    if (has) probed = l + 1;
    else if (probed > 0) break;
  }
  return probed;
}

std::vector<float> read_f32_array(const GgufFile &g, const std::string &k, bool *present) {
  *present = false;
  const GgufValue *v = g.value(k);
  if (!v) return {};
  if (v->type != GGUF_ARRAY) fail(JAL_ERR_CAPABILITY_MISMATCH, "expected array for GGUF metadata key '%s'", k.c_str());
  std::vector<float> out;
  for (const GgufValue &e : v->arr) {
    float f;
    if (!(e.type == GGUF_F32 || e.type == GGUF_F64 || e.type == GGUF_I32 || e.type == GGUF_U32) || !e.as_f32(&f))
      fail(JAL_ERR_CAPABILITY_MISMATCH, "expected numeric array for GGUF metadata key '%s'", k.c_str());
    out.push_back(f);
  }
  for (float f : out)
    if (!std::isfinite(f) || f <= 0.f) fail(JAL_ERR_CAPABILITY_MISMATCH, "GGUF key '%s' has invalid RoPE factors", k.c_str());
  if (out.empty()) fail(JAL_ERR_CAPABILITY_MISMATCH, "GGUF key '%s' is empty", k.c_str());
  *present = true;
  return out;
}

// parse_rope_scaling_from_gguf (recipe.rs:3259-3356) and helpers (:3115-3257)
RopeScaling parse_rope_scaling(const GgufFile &g, const std::string &arch) {
  RopeScaling sc;
  const GgufValue *tv = g.value(arch + ".rope.scaling.type");
  std::string type;
  bool has_type = false;
  if (tv) {
    if (!tv->is_string()) fail(JAL_ERR_CAPABILITY_MISMATCH, "expected string for %s.rope.scaling.type", arch.c_str());
    type = tv->s;
    has_type = true;
  }
  auto pos_f32 = [&](const std::string &k, float *out) -> bool {
    const GgufValue *v = g.value(k);
    if (!v) return false;
    float f;
    if (!v->as_f32(&f)) fail(JAL_ERR_CAPABILITY_MISMATCH, "expected numeric GGUF metadata value for '%s'", k.c_str());
    if (!std::isfinite(f) || f <= 0.f) fail(JAL_ERR_CAPABILITY_MISMATCH, "expected finite positive f32 for '%s'", k.c_str());
    *out = f;
    return true;
  };
  float factor = 0.f, lo = 0.f, hi = 0.f;
  bool has_factor = pos_f32(arch + ".rope.scaling.factor", &factor);
  bool has_lo = pos_f32(arch + ".rope.scaling.low_freq_factor", &lo);
  bool has_hi = pos_f32(arch + ".rope.scaling.high_freq_factor", &hi);
  uint64_t orig = 0;
  bool has_orig = false;
  for (const char *suf : {"rope.scaling.original_context_length", "rope.scaling.orig_ctx_len",
                          "rope.scaling.original_max_position_embeddings"}) {
    const GgufValue *v = g.value(arch + "." + suf);
    if (v) {
      if (!v->as_usize(&orig)) fail(JAL_ERR_CAPABILITY_MISMATCH, "expected integer for '%s.%s'", arch.c_str(), suf);
      if (orig == 0) fail(JAL_ERR_CAPABILITY_MISMATCH, "expected non-zero context length for '%s.%s'", arch.c_str(), suf);
      has_orig = true;
      break;
    }
  }
  bool has_short, has_long, has_factors;
  std::vector<float> sf = read_f32_array(g, arch + ".rope.scaling.short_factor", &has_short);
  std::vector<float> lf = read_f32_array(g, arch + ".rope.scaling.long_factor", &has_long);
  std::vector<float> ff = read_f32_array(g, arch + ".rope.scaling.factors", &has_factors);
  auto longrope = [&]() {
    RopeScaling r;
    r.kind = JAL_ROPE_SCALING_LONGROPE;
    r.original_max_position_embeddings = has_orig ? orig : 8192;
    if (has_short && has_long) {
      if (sf.size() != lf.size()) fail(JAL_ERR_CAPABILITY_MISMATCH, "LongRoPE short/long factor lengths differ");
      r.short_factor = sf; r.long_factor = lf;
    } else if (!has_short && has_long) {
      r.short_factor.assign(lf.size(), 1.0f); r.long_factor = lf;
    } else if (has_short && !has_long && !has_factors) {
      r.short_factor = sf; r.long_factor = sf;
    } else if (has_factors) {
      r.short_factor = ff; r.long_factor = ff;
    } else fail(JAL_ERR_CAPABILITY_MISMATCH, "missing LongRoPE scaling factor tables in GGUF metadata");
    return r;
  };
  auto llama3 = [&]() {
    if (!has_factor) fail(JAL_ERR_CAPABILITY_MISMATCH, "missing '%s.rope.scaling.factor' for llama3 RoPE scaling", arch.c_str());
    RopeScaling r;
    r.kind = JAL_ROPE_SCALING_LLAMA3;
    r.factor = factor;
    r.low_freq_factor = has_lo ? lo : 1.0f;
    r.high_freq_factor = has_hi ? hi : 4.0f;
    if (r.high_freq_factor <= r.low_freq_factor) fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid llama3 RoPE frequency bounds");
    r.original_max_position_embeddings = has_orig ? orig : 8192;
    return r;
  };
  if (has_type) {
    if (type == "none" || type.empty()) return sc;
    if (type == "linear") {
      if (!has_factor) fail(JAL_ERR_CAPABILITY_MISMATCH, "missing '%s.rope.scaling.factor' for linear RoPE scaling", arch.c_str());
      sc.kind = JAL_ROPE_SCALING_LINEAR;
      sc.factor = factor;
      return sc;
    }
    if (type == "llama3") return llama3();
    if (type == "longrope" || type == "yarn" || type == "su") return longrope();
    fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported RoPE scaling type '%s'", type.c_str());
  }
  if (has_short || has_long || has_factors) return longrope();
  if (has_factor) {
    if (has_lo || has_hi || has_orig) return llama3();
    sc.kind = JAL_ROPE_SCALING_LINEAR;
    sc.factor = factor;
  }
  return sc;
}

}  // namespace

// LlamaRecipe::from_metadata + from_gguf (recipe.rs:226-422)
Recipe Recipe::from_gguf(const GgufFile &g) {
  const std::string &arch = g.architecture();
  if (arch != "llama" && arch != "llama4" && arch != "qwen2")
    fail(JAL_ERR_CAPABILITY_MISMATCH, "LlamaRecipe supports 'llama', 'llama4', and 'qwen2', got '%s'", arch.c_str());
  Recipe r = for_arch(arch);
  uint64_t v = 0;
  float f = 0.f;
  uint64_t hidden = r.hidden_dim;
  if (meta_usize(g, arch + ".embedding_length", &v) && v > 0) hidden = v;
  else if (const GgufTensor *n = g.tensor("blk.0.attn_norm.weight") ? g.tensor("blk.0.attn_norm.weight") : g.tensor("output_norm.weight"))
    hidden = std::max<uint64_t>(n->num_elements(), 16);
  r.hidden_dim = hidden;
  uint64_t probed = 0;
  for (const GgufTensor &t : g.tensors()) {
    if (t.name.rfind("blk.", 0) == 0) {
      size_t dot = t.name.find('.', 4);
      if (dot != std::string::npos) {
        char *end = nullptr;
        unsigned long long idx = strtoull(t.name.c_str() + 4, &end, 10);
        if (end == t.name.c_str() + dot) probed = std::max<uint64_t>(probed, idx + 1);
      }
    }
  }
  if (meta_usize(g, arch + ".block_count", &v) && v > 0) r.num_layers = v;
  else if (probed > 0) r.num_layers = probed;
  uint64_t hc = 0, hkv = 0;
  bool has_hc = meta_usize(g, arch + ".attention.head_count", &hc) && hc > 0;
  bool has_hkv = meta_usize(g, arch + ".attention.head_count_kv", &hkv) && hkv > 0;
  if (has_hc) r.n_heads_q = hc;
  if (has_hkv) r.n_heads_kv = hkv;
  uint64_t kd = 0, q_rows = 0;
  const GgufTensor *qd = g.tensor("blk.0.attn_q.weight");
  if (meta_usize(g, arch + ".attention.key_length", &kd) && kd >= 2) {
    r.head_dim = kd;
    if (!has_hc && infer_rows(qd, hidden, &q_rows) && q_rows % kd == 0) r.n_heads_q = q_rows / kd;
  } else if (infer_rows(qd, hidden, &q_rows)) {
    if (has_hc && q_rows % r.n_heads_q == 0) r.head_dim = q_rows / r.n_heads_q;
    else if (r.head_dim > 0 && q_rows % r.head_dim == 0) r.n_heads_q = q_rows / r.head_dim;
  } else if (r.n_heads_q > 0 && hidden % r.n_heads_q == 0) {
    r.head_dim = hidden / r.n_heads_q;
  }
  uint64_t k_rows = 0;
  if (!has_hkv && infer_rows(g.tensor("blk.0.attn_k.weight"), hidden, &k_rows) && r.head_dim > 0 &&
      k_rows % r.head_dim == 0)
    r.n_heads_kv = k_rows / r.head_dim;
  uint64_t ffn_rows = 0;
  if (meta_usize(g, arch + ".feed_forward_length", &v) && v > 0) r.ffn_dim = v;
  else if (infer_rows(g.tensor("blk.0.ffn_gate.weight"), hidden, &ffn_rows) ||
           infer_rows(g.tensor("blk.0.ffn_up.weight"), hidden, &ffn_rows) ||
           infer_rows(g.tensor("blk.0.ffn_down.weight"), hidden, &ffn_rows))
    r.ffn_dim = ffn_rows;
  uint64_t vocab_rows = 0;
  const GgufTensor *vt = g.tensor("output.weight") ? g.tensor("output.weight") : g.tensor("token_embd.weight");
  if (infer_rows(vt, hidden, &vocab_rows)) r.vocab_size = vocab_rows;
  if (meta_f32(g, arch + ".attention.layer_norm_rms_epsilon", &f) && std::isfinite(f) && f > 0.f) r.rms_eps = f;
  if (meta_f32(g, arch + ".rope.freq_base", &f) && std::isfinite(f) && f > 0.f) r.rope_theta = f;
  if (meta_usize(g, arch + ".rope.dimension_count", &v)) r.rotary_dim = (int64_t)v;
  // from_gguf overrides (recipe.rs:349-404)
  if (meta_usize(g, arch + ".vocab_size", &v) && v > 0) r.vocab_size = v;
  else if (!g.tensor("output.weight") && !g.tensor("token_embd.weight")) {
    const GgufValue *tok = g.value("tokenizer.ggml.tokens");
    if (tok && tok->type == GGUF_ARRAY && !tok->arr.empty()) r.vocab_size = tok->arr.size();
  }
  r.scaling = parse_rope_scaling(g, arch);
  if (meta_usize(g, arch + ".attention.no_rope_layer_step", &v) && v > 0 && r.num_layers > 0) {
    r.has_irope_mask = true;
    r.irope_mask.resize(r.num_layers);
    for (uint64_t l = 0; l < r.num_layers; l++) r.irope_mask[l] = ((l + 1) % v) == 0;
  }
  return r;
}

static uint64_t resolve_rotary(const Recipe &r, uint64_t head_d_even) {  // recipe.rs:1165-1178
  if (r.rotary_dim < 0) return head_d_even;
  uint64_t rd = (uint64_t)r.rotary_dim;
  if (rd < 2 || rd % 2 || rd > head_d_even)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid rotary_dim %llu for head_dim %llu", (unsigned long long)rd,
         (unsigned long long)head_d_even);
  return rd;
}

static uint64_t gcd64(uint64_t a, uint64_t b) { while (b) { uint64_t t = a % b; a = b; b = t; } return a; }

// resolve_heads_from_totals (recipe.rs:1321-1373)
static void resolve_heads(const Recipe &r, uint64_t q_rows, uint64_t k_rows, Geometry &g) {
  uint64_t hd = std::max<uint64_t>(r.head_dim, 2);
  if (hd % 2) hd -= 1;
  uint64_t cq = std::max<uint64_t>(r.n_heads_q, 1), ckv = std::max<uint64_t>(r.n_heads_kv, 1);
  if (cq * hd == q_rows && ckv * hd == k_rows && cq % ckv == 0) {
    g.n_heads_q = cq; g.n_heads_kv = ckv; g.head_dim = hd;
    return;
  }
  uint64_t gg = gcd64(q_rows, k_rows);
  uint64_t cands[] = {hd, 128, 64, 96, 80, 48, 32, 16, 8, 4, (gg >= 2 && gg % 2 == 0) ? gg : 2, 2};
  for (uint64_t c : cands) {
    if (c >= 2 && c % 2 == 0 && q_rows >= c && k_rows >= c && q_rows % c == 0 && k_rows % c == 0) {
      uint64_t nq = q_rows / c, nkv = k_rows / c;
      if (nkv > 0 && nq % nkv == 0) { g.n_heads_q = nq; g.n_heads_kv = nkv; g.head_dim = c; return; }
    }
  }
  fail(JAL_ERR_CAPABILITY_MISMATCH, "unable to resolve valid even head_dim for q_rows=%llu, k_rows=%llu",
       (unsigned long long)q_rows, (unsigned long long)k_rows);
}

// resolve_geometry with resident tensors (recipe.rs:1180-1260)
Geometry resolve_geometry(const Recipe &r, const GgufFile &g) {
  Geometry ge;
  const GgufTensor *t;
  if ((t = g.tensor("blk.0.attn_norm.weight"))) ge.hidden_dim = t->num_elements();
  else if ((t = g.tensor("output_norm.weight"))) ge.hidden_dim = t->num_elements();
  else if ((t = g.tensor("token_embd.weight")) && t->n_dims == 2)
    ge.hidden_dim = (t->ne[0] == r.hidden_dim || t->ne[1] == r.hidden_dim) ? r.hidden_dim : t->ne[0];
  else fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'blk.0.attn_norm.weight'");
  ge.num_layers = probe_layers(g);
  if (!ge.num_layers) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'blk.0.attn_norm.weight'");
  const GgufTensor *q = g.tensor("blk.0.attn_q.weight"), *k = g.tensor("blk.0.attn_k.weight");
  if (!q) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'blk.0.attn_q.weight'");
  if (!k) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'blk.0.attn_k.weight'");
  uint64_t q_rows, k_rows, c;
  resolve_2d(q, ge.hidden_dim, &q_rows, &c);
  resolve_2d(k, ge.hidden_dim, &k_rows, &c);
  resolve_heads(r, q_rows, k_rows, ge);
  ge.rotary_dim = resolve_rotary(r, ge.head_dim);
  if ((t = g.tensor("blk.0.ffn_gate.weight")) || (t = g.tensor("blk.0.ffn_up.weight"))) resolve_2d(t, ge.hidden_dim, &ge.ffn_dim, &c);
  else if ((t = g.tensor("blk.0.ffn_down.weight"))) {
    if (t->n_dims != 2) fail(JAL_ERR_TENSOR_BOUNDS, "expected 2D tensor for blk.0.ffn_down.weight");
    if (t->ne[0] == ge.hidden_dim) ge.ffn_dim = t->ne[1];
    else if (t->ne[1] == ge.hidden_dim) ge.ffn_dim = t->ne[0];
    else fail(JAL_ERR_TENSOR_BOUNDS, "ffn_down shape does not match hidden_dim");
  } else fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'blk.0.ffn_gate.weight'");
  ge.total_q = ge.n_heads_q * ge.head_dim;
  ge.total_kv = ge.n_heads_kv * ge.head_dim;
  return ge;
}

// ArchRecipe::validate_model (recipe.rs:1834-1931)
void Recipe::validate_model(const GgufFile &g) const {
  const std::string &arch = g.architecture();
  if (arch != "llama" && arch != "llama4" && arch != "qwen2")
    fail(JAL_ERR_CAPABILITY_MISMATCH, "LlamaRecipe supports 'llama', 'llama4', and 'qwen2', got '%s'", arch.c_str());
  if (n_heads_kv == 0 || n_heads_q < n_heads_kv || n_heads_q % n_heads_kv)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid GQA head counts: n_heads_q=%llu n_heads_kv=%llu",
         (unsigned long long)n_heads_q, (unsigned long long)n_heads_kv);
  for (const GgufTensor &t : g.tensors())
    if (!supports_quant((int)t.type))
      fail(JAL_ERR_CAPABILITY_MISMATCH, "tensor '%s' uses unsupported quant %u", t.name.c_str(), t.type);
  if (g.tensor_count() == 0) {
    uint64_t hd = std::max<uint64_t>(head_dim, 2);
    if (hd % 2) hd -= 1;
    resolve_rotary(*this, hd);
    return;
  }
  Geometry ge = resolve_geometry(*this, g);
  auto need = [&](const std::string &n) {
    if (!g.tensor(n)) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor '%s'", n.c_str());
  };
  need("token_embd.weight");
  need("output_norm.weight");
  for (uint64_t l = 0; l < ge.num_layers; l++)
    for (const char *s : {"attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                          "ffn_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"})
      need(key(l, s));
}

// ---------------------------------------------------------------------------
// Device buffers and repack
// ---------------------------------------------------------------------------

DevBuffer::DevBuffer(size_t n) : bytes(n) {
  if (n) JAL_CUDA(cudaMalloc(&ptr, n));
}
DevBuffer::~DevBuffer() {
  if (ptr) cudaFree(ptr);
}

static DevBufferPtr alloc(size_t n) { return std::make_shared<DevBuffer>(n); }

// Quants of the device GEMV / GEMM path; Q5_0 runs in the Q8_0 layout.
static bool device_quant(int q) { return q == JAL_Q4_0 || q == JAL_Q5_0 || q == JAL_Q8_0; }
static int device_layout(int q) { return q == JAL_Q5_0 ? JAL_Q8_0 : q; }

CachedMatrix repack_matrix(const uint8_t *raw_dev, int quant, uint64_t rows, uint64_t cols, cudaStream_t s) {
  std::vector<CachedMatrix> parts;
  DevMat stacked;
  std::vector<DevBufferPtr> storage;
  repack_stacked({raw_dev}, {rows}, quant, cols, s, parts, stacked, storage);
  parts[0].storage = storage;
  return parts[0];
}

void repack_stacked(const std::vector<const uint8_t *> &raws, const std::vector<uint64_t> &rows, int quant,
                    uint64_t cols, cudaStream_t s, std::vector<CachedMatrix> &parts, DevMat &stacked,
                    std::vector<DevBufferPtr> &storage) {
  uint64_t total = 0;
  for (uint64_t r : rows) total += r;
  parts.clear();
  if (device_quant(quant)) {
    if (cols % 32) fail(JAL_ERR_TENSOR_BOUNDS, "cols %llu not a multiple of 32", (unsigned long long)cols);
    // Row-interleaved: each row is its quants then its padded f16 scales.
    const int64_t nib = quant == JAL_Q4_0 ? (int64_t)cols / 2 : (int64_t)cols;
    const int64_t row_bytes = nib + 2 * d_stride_for((int64_t)cols);
    const int64_t qs_stride = row_bytes, d_stride = row_bytes / 2;
    DevBufferPtr buf = alloc((size_t)total * row_bytes);
    JAL_CUDA(cudaMemsetAsync(buf->ptr, 0, buf->bytes, s));
    storage.push_back(buf);
    stacked = DevMat{};
    stacked.quant = device_layout(quant); stacked.rows = (int64_t)total; stacked.cols = (int64_t)cols;
    stacked.qs = buf->as<uint8_t>(); stacked.d = (const uint16_t *)(buf->as<uint8_t>() + nib);
    stacked.qs_stride = qs_stride; stacked.d_stride = d_stride;
    uint64_t r0 = 0;
    for (size_t i = 0; i < raws.size(); i++) {
      launch_repack(raws[i], quant, (int64_t)rows[i], (int64_t)cols, buf->as<uint8_t>() + r0 * qs_stride,
                    (uint16_t *)(buf->as<uint8_t>() + nib) + r0 * d_stride, qs_stride, d_stride, s);
      JAL_CUDA(cudaGetLastError());
      CachedMatrix m;
      m.quant = quant; m.rows = rows[i]; m.cols = cols;
      m.dm = stacked;
      m.dm.rows = (int64_t)rows[i];
      m.dm.qs = stacked.qs + r0 * qs_stride;
      m.dm.d = stacked.d + r0 * d_stride;
      m.aligned_bytes = (size_t)rows[i] * row_bytes;
      parts.push_back(m);
      r0 += rows[i];
    }
    return;
  }
  if (kquant(quant)) {
    if (cols % 256) fail(JAL_ERR_TENSOR_BOUNDS, "cols %llu not a multiple of 256", (unsigned long long)cols);
    const int64_t ng = (int64_t)cols / kquant_group(quant), row_q = (int64_t)cols;
    const bool mins = quant != JAL_Q6_K;
    DevBufferPtr bq = alloc((size_t)total * row_q), bs = alloc((size_t)total * ng * 4);
    DevBufferPtr bm = mins ? alloc((size_t)total * ng * 4) : nullptr;
    storage.push_back(bq);
    storage.push_back(bs);
    if (bm) storage.push_back(bm);
    stacked = DevMat{};
    stacked.quant = quant; stacked.rows = (int64_t)total; stacked.cols = (int64_t)cols;
    stacked.qs = bq->as<uint8_t>(); stacked.qs_stride = row_q;
    stacked.ks = bs->as<float>(); stacked.km = bm ? bm->as<float>() : nullptr; stacked.k_stride = ng;
    uint64_t r0 = 0;
    for (size_t i = 0; i < raws.size(); i++) {
      launch_repack_kquant(raws[i], quant, (int64_t)rows[i], (int64_t)cols, (int8_t *)(bq->as<uint8_t>() + r0 * row_q),
                           row_q, bs->as<float>() + r0 * ng, bm ? bm->as<float>() + r0 * ng : nullptr, ng, s);
      JAL_CUDA(cudaGetLastError());
      CachedMatrix m;
      m.quant = quant; m.rows = rows[i]; m.cols = cols;
      m.dm = stacked;
      m.dm.rows = (int64_t)rows[i];
      m.dm.qs = stacked.qs + r0 * row_q;
      m.dm.ks = stacked.ks + r0 * ng;
      m.dm.km = stacked.km ? stacked.km + r0 * ng : nullptr;
      m.aligned_bytes = (size_t)rows[i] * (row_q + ng * 4 * (mins ? 2 : 1));
      parts.push_back(m);
      r0 += rows[i];
    }
    return;
  }
  if (dense_quant(quant)) {
    // Dense rows keep their GGUF element type (repack_dense's sanitising
    // happens on load in the dense kernels).
    const size_t es = quant == JAL_F32 ? 4 : 2;
    DevBufferPtr buf = alloc((size_t)total * cols * es);
    storage.push_back(buf);
    stacked = DevMat{};
    stacked.quant = quant; stacked.rows = (int64_t)total; stacked.cols = (int64_t)cols;
    stacked.dense = buf->ptr;
    uint64_t r0 = 0;
    for (size_t i = 0; i < raws.size(); i++) {
      char *dst = (char *)buf->ptr + r0 * cols * es;
      JAL_CUDA(cudaMemcpyAsync(dst, raws[i], (size_t)rows[i] * cols * es, cudaMemcpyDeviceToDevice, s));
      CachedMatrix m;
      m.quant = quant; m.rows = rows[i]; m.cols = cols;
      m.dm = stacked;
      m.dm.rows = (int64_t)rows[i];
      m.dm.dense = dst;
      m.aligned_bytes = (size_t)rows[i] * cols * es;
      parts.push_back(m);
      r0 += rows[i];
    }
    return;
  }
  fail(JAL_ERR_CAPABILITY_MISMATCH, "quant %d is admitted by the recipe but not implemented on the device path", quant);
}

size_t ModelCache::total_aligned_bytes() const {  // repack_cache.rs:2348-2380
  size_t t = output_norm ? output_norm->bytes : 0;
  for (const Layer &l : layers) {
    t += l.norms ? l.norms->bytes : 0;
    t += l.biases ? l.biases->bytes : 0;
    for (const CachedMatrix *m : {&l.wq, &l.wk, &l.wv, &l.wo, &l.wgate, &l.wup, &l.wdown}) t += m->aligned_bytes;
  }
  return t + lm_head.aligned_bytes;
}

// decode_row_payload_to_f32 for 1D vectors (repack_cache.rs:1244-1301) on the host.
static float h_f16(uint16_t bits) {
  uint32_t sign = (bits >> 15) & 1u, exp = (bits >> 10) & 0x1Fu, mant = bits & 0x3FFu, out;
  if (exp == 0) {
    if (mant == 0) out = sign << 31;
    else {
      uint32_t m = mant, e = 113;
      while (!(m & 0x400u)) { m <<= 1; e--; }
      out = (sign << 31) | (e << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (exp == 31) return sign ? -0.0625f : 0.0625f;
  else out = (sign << 31) | ((exp + 112u) << 23) | (mant << 13);
  float f;
  memcpy(&f, &out, 4);
  return f;
}

static std::vector<float> decode_1d(const GgufTensor *t, uint64_t len, bool sanitize) {
  if (t->num_elements() != len)
    fail(JAL_ERR_TENSOR_BOUNDS, "%s: expected 1D len %llu, got %llu", t->name.c_str(), (unsigned long long)len,
         (unsigned long long)t->num_elements());
  size_t rb = ggml_row_bytes(t->type, len);
  if (!rb) fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported quant %u for %s", t->type, t->name.c_str());
  if (t->nbytes < rb) fail(JAL_ERR_TENSOR_BOUNDS, "%s truncated", t->name.c_str());
  std::vector<float> out(len);
  const uint8_t *p = t->data;
  for (uint64_t i = 0; i < len; i++) {
    float v;
    if (t->type == JAL_F32) {
      memcpy(&v, p + i * 4, 4);
      if (!std::isfinite(v)) v = 0.f;
      else if (sanitize && std::fabs(v) > 1.0e6f) v = std::signbit(v) ? -0.0625f : 0.0625f;
    } else if (t->type == JAL_F16) {
      v = h_f16((uint16_t)(p[i * 2] | (p[i * 2 + 1] << 8)));
    } else if (t->type == JAL_BF16) {
      uint16_t b = (uint16_t)(p[i * 2] | (p[i * 2 + 1] << 8));
      if (((b >> 7) & 0xFF) == 0xFF) v = (b & 0x8000) ? -0.0625f : 0.0625f;
      else { uint32_t u = (uint32_t)b << 16; memcpy(&v, &u, 4); }
    } else if (t->type == JAL_Q8_0 || t->type == JAL_Q4_0) {
      size_t bb = t->type == JAL_Q8_0 ? 34 : 18;
      const uint8_t *blk = p + (i / 32) * bb;
      float d = h_f16((uint16_t)(blk[0] | (blk[1] << 8)));
      int e = (int)(i % 32), q;
      if (t->type == JAL_Q8_0) q = (int8_t)blk[2 + e];
      else q = (int)(e < 16 ? (blk[2 + e] & 15) : (blk[2 + e - 16] >> 4)) - 8;
      v = d == 0.f ? 0.f : d * (float)q;
    } else fail(JAL_ERR_CAPABILITY_MISMATCH, "1D tensor %s quant %u not supported on the device path", t->name.c_str(), t->type);
    out[i] = v;
  }
  return out;
}

namespace {
struct Uploader {
  cudaStream_t s;
  DevBufferPtr staging;
  const uint8_t *put(const GgufTensor *t, size_t bytes) {
    if (!staging || staging->bytes < bytes) {
      JAL_CUDA(cudaStreamSynchronize(s));
      staging = alloc(bytes);
    }
    JAL_CUDA(cudaMemcpyAsync(staging->ptr, t->data, bytes, cudaMemcpyHostToDevice, s));
    return staging->as<uint8_t>();
  }
};
}  // namespace

std::unique_ptr<ModelCache> build_model_cache(const Recipe &r, const GgufFile &g, int device, const TpComm *tp) {
  if (g.tensor_count() == 0) fail(JAL_ERR_CAPABILITY_MISMATCH, "build_repack_cache requires resident model tensors");
  JAL_CUDA(cudaSetDevice(device));
  auto c = std::make_unique<ModelCache>();
  c->architecture = r.architecture;
  c->device = device;
  Geometry ge = resolve_geometry(r, g);
  c->geom = ge;
  const GgufTensor *lm = g.tensor("output.weight") ? g.tensor("output.weight") : g.tensor("token_embd.weight");
  if (!lm) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'output.weight'");
  uint64_t vrows, vcols;
  resolve_2d(lm, ge.hidden_dim, &vrows, &vcols);
  c->vocab_size = vrows;
  // This rank's shard (tp.hpp); rank 0 of 1 without tensor parallelism.
  c->tp = tp;
  c->plan = tp_plan(ge.n_heads_q, ge.n_heads_kv, ge.ffn_dim, vrows, tp ? tp->rank : 0, tp ? tp->world : 1);
  const TpPlan &pl = c->plan;
  c->lgeom = ge;
  c->lgeom.n_heads_q = pl.q_n;
  c->lgeom.n_heads_kv = pl.kv_n;
  c->lgeom.total_q = pl.q_n * ge.head_dim;
  c->lgeom.total_kv = pl.kv_n * ge.head_dim;
  c->lgeom.ffn_dim = pl.f_n;
  cudaStream_t s;
  JAL_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  struct StreamGuard { cudaStream_t s; ~StreamGuard() { cudaStreamSynchronize(s); cudaStreamDestroy(s); } } sg{s};
  const uint64_t H = ge.hidden_dim, F = ge.ffn_dim, Q = ge.total_q, KV = ge.total_kv;
  const uint64_t HD = ge.head_dim;
  // Shard extents: Q/K/V rows by heads, FFN rows (gate / up) and down input
  // columns by FFN index, O input columns by query-head width.
  const uint64_t Ql = pl.q_n * HD, q0 = pl.q_lo * HD, KVl = pl.kv_n * HD, kv0 = pl.kv_lo * HD;
  const uint64_t Fl = pl.f_n, f0 = pl.f_lo;

  // Raw upload of several tensors (row ranges, optionally a column range
  // of whole blocks: one pitched copy) into one staging block, then repack.
  struct Piece {
    const GgufTensor *t;
    uint64_t row0, rows, full_cols, col0, cols;
  };
  auto stage_many = [&](const std::vector<Piece> &ps, DevBufferPtr &blk) {
    size_t total = 0;
    std::vector<size_t> offs;
    for (const Piece &p : ps) {
      offs.push_back(total);
      total += (ggml_row_bytes(p.t->type, p.cols) * p.rows + 255) / 256 * 256;
    }
    blk = alloc(total);
    std::vector<const uint8_t *> out;
    for (size_t i = 0; i < ps.size(); i++) {
      const Piece &p = ps[i];
      const size_t full = ggml_row_bytes(p.t->type, p.full_cols), part = ggml_row_bytes(p.t->type, p.cols);
      const size_t skip = ggml_row_bytes(p.t->type, p.col0);
      if ((p.col0 && !skip) || !part)
        fail(JAL_ERR_CAPABILITY_MISMATCH, "column shard of %s is not block aligned", p.t->name.c_str());
      const uint8_t *src = (const uint8_t *)p.t->data + p.row0 * full + skip;
      if (part == full)
        JAL_CUDA(cudaMemcpyAsync(blk->as<uint8_t>() + offs[i], src, part * p.rows, cudaMemcpyHostToDevice, s));
      else
        JAL_CUDA(cudaMemcpy2DAsync(blk->as<uint8_t>() + offs[i], part, src, full, part, p.rows, cudaMemcpyHostToDevice,
                                   s));
      out.push_back(blk->as<uint8_t>() + offs[i]);
    }
    return out;
  };
  auto tensor2d = [&](size_t l, const char *suf, uint64_t exp_cols, uint64_t exp_rows) {
    std::string n = key(l, suf);
    const GgufTensor *t = g.tensor(n);
    if (!t) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor '%s'", n.c_str());
    uint64_t rows, cols;
    resolve_2d(t, exp_cols, &rows, &cols);
    if (rows != exp_rows)
      fail(JAL_ERR_TENSOR_BOUNDS, "expected %llu rows for %s, got %llu", (unsigned long long)exp_rows, n.c_str(),
           (unsigned long long)rows);
    return t;
  };

  c->layers.resize(ge.num_layers);
  for (uint64_t l = 0; l < ge.num_layers; l++) {
    Layer &L = c->layers[l];
    const GgufTensor *an = g.tensor(key(l, "attn_norm.weight")), *fn = g.tensor(key(l, "ffn_norm.weight"));
    if (!an) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor '%s'", key(l, "attn_norm.weight").c_str());
    if (!fn) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor '%s'", key(l, "ffn_norm.weight").c_str());
    std::vector<float> norms = decode_1d(an, H, true), fnv = decode_1d(fn, H, true);
    norms.insert(norms.end(), fnv.begin(), fnv.end());
    L.norms = alloc(norms.size() * 4);
    JAL_CUDA(cudaMemcpyAsync(L.norms->ptr, norms.data(), norms.size() * 4, cudaMemcpyHostToDevice, s));
    L.attn_norm = L.norms->as<float>();
    L.ffn_norm = L.norms->as<float>() + H;
    c->norm_count += 2;
    // Optional biases (repack_cache.rs:2197-2200; decoded without large-value sanitizing).
    std::vector<float> b;
    size_t offq = 0, offk = 0, offv = 0, offo = 0;
    bool hq = false, hk = false, hv = false, ho = false;
    auto opt = [&](const char *suf, uint64_t len, size_t &off, bool &has) {
      const GgufTensor *t = g.tensor(key(l, suf));
      if (!t) return;
      std::vector<float> v = decode_1d(t, len, false);
      off = b.size();
      b.insert(b.end(), v.begin(), v.end());
      has = true;
      c->bias_count++;
    };
    opt("attn_q.bias", Q, offq, hq);
    opt("attn_k.bias", KV, offk, hk);
    opt("attn_v.bias", KV, offv, hv);
    if (pl.rank == 0) opt("attn_output.bias", H, offo, ho);  // added once, before the all-reduce
    if (!b.empty()) {
      L.biases = alloc(b.size() * 4);
      JAL_CUDA(cudaMemcpyAsync(L.biases->ptr, b.data(), b.size() * 4, cudaMemcpyHostToDevice, s));
      const float *base = L.biases->as<float>();
      if (hq) L.bq = base + offq + q0;  // this rank's heads
      if (hk) L.bk = base + offk + kv0;
      if (hv) L.bv = base + offv + kv0;
      if (ho) L.bo = base + offo;
    }
    const GgufTensor *tq = tensor2d(l, "attn_q.weight", H, Q), *tk = tensor2d(l, "attn_k.weight", H, KV),
                     *tv = tensor2d(l, "attn_v.weight", H, KV), *to = tensor2d(l, "attn_output.weight", Q, H),
                     *tg = tensor2d(l, "ffn_gate.weight", H, F), *tu = tensor2d(l, "ffn_up.weight", H, F),
                     *td = tensor2d(l, "ffn_down.weight", F, H);
    for (const GgufTensor *t : {tq, tk, tv, to, tg, tu, td})
      if (!r.supports_quant((int)t->type))
        fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported quant %u on %s", t->type, t->name.c_str());
    DevBufferPtr blk;
    std::vector<CachedMatrix> parts;
    DevMat stacked;
    const std::vector<Piece> qkv_pieces = {{tq, q0, Ql, H, 0, H}, {tk, kv0, KVl, H, 0, H}, {tv, kv0, KVl, H, 0, H}};
    if (tq->type == tk->type && tk->type == tv->type) {
      auto raws = stage_many(qkv_pieces, blk);
      repack_stacked(raws, {Ql, KVl, KVl}, (int)tq->type, H, s, parts, stacked, L.storage);
      L.wq = parts[0]; L.wk = parts[1]; L.wv = parts[2];
      L.qkv = stacked;
      L.qkv_stacked = device_quant((int)tq->type);
    } else {
      auto raws = stage_many(qkv_pieces, blk);
      std::vector<CachedMatrix> p1;
      repack_stacked({raws[0]}, {Ql}, (int)tq->type, H, s, p1, stacked, L.storage); L.wq = p1[0];
      repack_stacked({raws[1]}, {KVl}, (int)tk->type, H, s, p1, stacked, L.storage); L.wk = p1[0];
      repack_stacked({raws[2]}, {KVl}, (int)tv->type, H, s, p1, stacked, L.storage); L.wv = p1[0];
    }
    JAL_CUDA(cudaStreamSynchronize(s));
    {
      auto raws = stage_many({{to, 0, H, Q, q0, Ql}}, blk);  // input columns of this rank's heads
      repack_stacked(raws, {H}, (int)to->type, Ql, s, parts, stacked, L.storage);
      L.wo = parts[0];
    }
    JAL_CUDA(cudaStreamSynchronize(s));
    if (tg->type == tu->type) {
      auto raws = stage_many({{tg, f0, Fl, H, 0, H}, {tu, f0, Fl, H, 0, H}}, blk);
      repack_stacked(raws, {Fl, Fl}, (int)tg->type, H, s, parts, stacked, L.storage);
      L.wgate = parts[0]; L.wup = parts[1];
      L.gateup = stacked;
      L.gateup_stacked = device_quant((int)tg->type);
    } else {
      auto raws = stage_many({{tg, f0, Fl, H, 0, H}, {tu, f0, Fl, H, 0, H}}, blk);
      std::vector<CachedMatrix> p1;
      repack_stacked({raws[0]}, {Fl}, (int)tg->type, H, s, p1, stacked, L.storage); L.wgate = p1[0];
      repack_stacked({raws[1]}, {Fl}, (int)tu->type, H, s, p1, stacked, L.storage); L.wup = p1[0];
    }
    JAL_CUDA(cudaStreamSynchronize(s));
    {
      auto raws = stage_many({{td, 0, H, F, f0, Fl}}, blk);  // input columns of this rank's FFN rows
      repack_stacked(raws, {H}, (int)td->type, Fl, s, parts, stacked, L.storage);
      L.wdown = parts[0];
    }
    JAL_CUDA(cudaStreamSynchronize(s));
  }
  const GgufTensor *on = g.tensor("output_norm.weight");
  if (!on) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'output_norm.weight'");
  std::vector<float> onv = decode_1d(on, H, true);
  c->output_norm = alloc(onv.size() * 4);
  JAL_CUDA(cudaMemcpyAsync(c->output_norm->ptr, onv.data(), onv.size() * 4, cudaMemcpyHostToDevice, s));
  c->norm_count++;
  // LM head (repack_cache.rs:2226-2242) and the raw embedding table.
  {
    DevBufferPtr blk;
    auto raws = stage_many({{lm, pl.v_lo, pl.v_n, vcols, 0, vcols}}, blk);  // this rank's vocabulary rows
    std::vector<CachedMatrix> parts;
    DevMat stacked;
    std::vector<DevBufferPtr> st;
    repack_stacked(raws, {pl.v_n}, (int)lm->type, vcols, s, parts, stacked, st);
    c->lm_head = parts[0];
    c->lm_head.storage = st;
    JAL_CUDA(cudaStreamSynchronize(s));
  }
  const GgufTensor *emb = g.tensor("token_embd.weight");
  if (!emb) fail(JAL_ERR_TENSOR_BOUNDS, "missing required tensor 'token_embd.weight'");
  uint64_t erows, ecols;
  resolve_2d(emb, H, &erows, &ecols);
  if (emb->ne[0] != H) fail(JAL_ERR_CAPABILITY_MISMATCH, "token_embd.weight must be stored [hidden, vocab]");
  size_t eb = ggml_row_bytes(emb->type, H) * erows;
  c->emb_raw = alloc(eb);
  JAL_CUDA(cudaMemcpyAsync(c->emb_raw->ptr, emb->data, eb, cudaMemcpyHostToDevice, s));
  c->emb_quant = (int)emb->type;
  c->emb_rows = erows;
  JAL_CUDA(cudaStreamSynchronize(s));
  return c;
}

// ---------------------------------------------------------------------------
// RoPE tables (recipe.rs:2560-2715), host-side with libm like the reference
// ---------------------------------------------------------------------------
void fill_inv_freq(uint64_t head_dim, float theta, const RopeScaling &sc, uint64_t seq_len, float *out) {
  if (head_dim == 0 || head_dim % 2 || !std::isfinite(theta) || theta <= 0.f)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid RoPE parameters");
  uint64_t half = head_dim / 2;
  float hd = (float)head_dim;
  for (uint64_t i = 0; i < half; i++) out[i] = 1.0f / powf(theta, (float)(2 * i) / hd);
  switch (sc.kind) {
    case JAL_ROPE_SCALING_NONE: return;
    case JAL_ROPE_SCALING_LINEAR:
      if (!std::isfinite(sc.factor) || sc.factor <= 0.f) fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid linear RoPE scaling factor");
      for (uint64_t i = 0; i < half; i++) out[i] /= sc.factor;
      return;
    case JAL_ROPE_SCALING_LLAMA3: {
      float factor = sc.factor, lo = sc.low_freq_factor, hi = sc.high_freq_factor;
      if (!std::isfinite(factor) || factor <= 0.f || !std::isfinite(lo) || lo <= 0.f || !std::isfinite(hi) || hi <= lo ||
          sc.original_max_position_embeddings == 0)
        fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid Llama-3 smooth RoPE scaling parameters");
      float orig = (float)sc.original_max_position_embeddings, low_wl = orig / lo, high_wl = orig / hi;
      for (uint64_t i = 0; i < half; i++) {
        float freq = out[i], wavelen = 6.28318530717958647692f / freq;
        if (wavelen > low_wl) out[i] = freq / factor;
        else if (wavelen >= high_wl) {
          float smooth = (orig / wavelen - lo) / (hi - lo);
          out[i] = (1.0f - smooth) * (freq / factor) + smooth * freq;
        }
      }
      return;
    }
    case JAL_ROPE_SCALING_LONGROPE: {
      const std::vector<float> &f = seq_len > sc.original_max_position_embeddings ? sc.long_factor : sc.short_factor;
      if (f.size() != half) fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid LongRoPE per-dimension scaling factor table");
      for (float x : f)
        if (!std::isfinite(x) || x <= 0.f) fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid LongRoPE factor");
      for (uint64_t i = 0; i < half; i++) out[i] /= f[i];
      return;
    }
    default: fail(JAL_ERR_CAPABILITY_MISMATCH, "unknown RoPE scaling kind %d", sc.kind);
  }
}

static void build_rope_table(uint64_t n_ctx, uint64_t rot, const std::vector<float> &inv, std::vector<float> &c,
                             std::vector<float> &s) {
  uint64_t half = rot / 2;
  c.resize(n_ctx * half);
  s.resize(n_ctx * half);
  for (uint64_t p = 0; p < n_ctx; p++) {
    float pf = (float)p;
    for (uint64_t i = 0; i < half; i++) {
      float a = pf * inv[i];
      s[p * half + i] = sinf(a);
      c[p * half + i] = cosf(a);
    }
  }
}

// ---------------------------------------------------------------------------
// Context
// ---------------------------------------------------------------------------

static int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

static bool env_flag(const char *n) {
  const char *v = getenv(n);
  return v && *v && *v != '0';
}

// Persistent decode step: one cooperative launch of one CTA per SM per
// token (decode_mega.cu).  Opt-in with JAL_DECODE=mega, fast numerics only;
// the context keeps the graph path when the model shape or the device does
// not fit it.
static void setup_mega(Context &ctx, int sms) {
  const char *e = getenv("JAL_DECODE");
  if (!e || strcmp(e, "mega") != 0 || ctx.cfg.numerics != JAL_NUMERICS_RELAXED) return;
  if (ctx.cache->plan.world > 1) return;  // single-GPU kernel
  const ModelCache &c = *ctx.cache;
  const Geometry &g = ctx.g;
  int coop = 0;
  JAL_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c.device));
  if (!coop) return;
  std::vector<MegaLayer> layers(c.layers.size());
  for (size_t l = 0; l < c.layers.size(); l++) {
    const Layer &L = c.layers[l];
    MegaLayer &m = layers[l];
    m.qkv = L.qkv; m.wo = L.wo.dm; m.gateup = L.gateup; m.wdown = L.wdown.dm;
    m.attn_norm = L.attn_norm; m.ffn_norm = L.ffn_norm;
    m.bq = L.bq; m.bk = L.bk; m.bv = L.bv; m.bo = L.bo;
    m.skip_rope = ctx.recipe.should_skip_rope(l) ? 1 : 0;
    if (!w4_matrix_ok(m.qkv) || !w4_matrix_ok(m.wo) || !w4_matrix_ok(m.gateup) || !w4_matrix_ok(m.wdown)) return;
    // one weight type for every projection (the kernel is instantiated per type)
    const int q = c.lm_head.dm.quant;
    if (m.qkv.quant != q || m.wo.quant != q || m.gateup.quant != q || m.wdown.quant != q) return;
  }
  if (!w4_matrix_ok(c.lm_head.dm)) return;
  MegaArgs &a = ctx.margs;
  a.n_layers = (int)c.layers.size();
  a.H = (int64_t)g.hidden_dim; a.F = (int64_t)g.ffn_dim; a.V = (int64_t)c.vocab_size;
  a.n_heads_q = (int64_t)g.n_heads_q; a.n_kv = (int64_t)g.n_heads_kv; a.rotary_dim = (int64_t)g.rotary_dim;
  a.eps = std::max(ctx.recipe.rms_eps, 1.0e-7f);
  a.scale = 1.0f / sqrtf((float)g.head_dim);
  a.lm_head = c.lm_head.dm;
  a.out_norm = c.output_norm->as<float>();
  a.emb = c.emb_raw->as<uint8_t>(); a.emb_quant = c.emb_quant; a.emb_rows = (int64_t)c.emb_rows;
  a.cos_tab = ctx.cos_tab; a.sin_tab = ctx.sin_tab; a.cos_long = ctx.cos_long; a.sin_long = ctx.sin_long;
  a.long_threshold = ctx.recipe.scaling.kind == JAL_ROPE_SCALING_LONGROPE
                         ? (int64_t)ctx.recipe.scaling.original_max_position_embeddings : -1;
  a.neox = ctx.recipe.rope_type == JAL_ROPE_NEOX;
  a.kv = ctx.kv;
  a.window = (int64_t)ctx.cfg.sliding_window;
  a.d_pos = ctx.d_pos; a.d_token = ctx.d_token; a.d_hist = ctx.d_hist;
  a.hidden = ctx.hidden; a.qkv = ctx.qkv; a.attn = ctx.attn; a.ffn = ctx.ffn; a.logits = ctx.logits;
  a.attn_q = ctx.attn_q; a.attn_s = ctx.attn_s;
  a.ffn_q = ctx.ffn_q; a.ffn_s = ctx.ffn_s; a.ffn_cnt = ctx.ffn_cnt;
  a.am_val = ctx.am_val; a.am_idx = ctx.am_idx; a.am_cnt = ctx.am_cnt;
  a.err = ctx.d_err;
  a.splits = std::max(1, std::min(64, sms / (int)g.n_heads_kv));
  if (const char *v = getenv("JAL_MEGA_SPLIT_TOKENS")) a.attn_split_tokens = std::max(1, atoi(v));
  if (!prepare_decode_mega(a, sms)) return;
  const size_t part = mega_part_bytes(a);
  const size_t H = g.hidden_dim;
  auto lb = alloc(layers.size() * sizeof(MegaLayer) + 256 + part + 256 + g.n_heads_kv * 4 + 256 + 64 + 256 +
                  sizeof(MegaArgs) + 256 + H * 4 + 256 + H + 256 + H / 32 * 4 + 256 + H / 32 * 4 + 256 + (size_t)sms * 4 +
                  256);
  ctx.bufs.push_back(lb);
  JAL_CUDA(cudaMemset(lb->ptr, 0, lb->bytes));
  char *p = lb->as<char>();
  auto take = [&](size_t n) { char *q = p; p += (n + 255) / 256 * 256; return q; };
  MegaLayer *dl = (MegaLayer *)take(layers.size() * sizeof(MegaLayer));
  JAL_CUDA(cudaMemcpy(dl, layers.data(), layers.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice));
  a.layers = dl;
  a.attn_part = (float *)take(part);
  a.head_cnt = (unsigned *)take(g.n_heads_kv * 4);
  a.bar = (unsigned *)take(8);
  MegaArgs *da = (MegaArgs *)take(sizeof(MegaArgs));
  a.hu = (float *)take(H * 4);
  a.hq = (int8_t *)take(H);
  a.hs = (float *)take(H / 32 * 4);
  a.hcnt = (unsigned *)take(H / 32 * 4);
  a.hss = (float *)take((size_t)sms * 4);
  if ((size_t)(p - lb->as<char>()) > lb->bytes) fail(JAL_ERR_INVALID_ARGUMENT, "internal: persistent decode layout overflow");
  JAL_CUDA(cudaMemcpy(da, &a, sizeof(MegaArgs), cudaMemcpyHostToDevice));
  ctx.mega_dev_args = da;
  ctx.mega = true;
  ctx.mega_grid = sms;
}

static void setup_tp_exchange(Context &ctx, int sms);

size_t KvCache::bytes() const {
  size_t b = 0;
  for (const auto &p : bufs) b += p->bytes;
  return b;
}

// Paged layout [layer][page][kv_head][slot][head_dim], K and V pools, with an
// identity page table; zero-filled.
std::unique_ptr<KvCache> create_kv_cache(const ModelCache &c, uint64_t n_ctx, int kv_f16, uint32_t page_size) {
  if (n_ctx == 0) fail(JAL_ERR_INVALID_ARGUMENT, "n_ctx must be positive");
  if (page_size == 0) page_size = 64;
  JAL_CUDA(cudaSetDevice(c.device));
  const Geometry &g = c.lgeom;
  auto kc = std::make_unique<KvCache>();
  kc->n_ctx = n_ctx;
  kc->device = c.device;
  const uint64_t ps = page_size, n_pages = (n_ctx + ps - 1) / ps;
  KvView &kv = kc->kv;
  kv.f16 = kv_f16 ? 1 : 0;
  kv.n_pages = (int64_t)n_pages; kv.page_size = (int64_t)ps; kv.n_kv = (int64_t)g.n_heads_kv;
  kv.head_dim = (int64_t)g.head_dim; kv.n_layers = (int64_t)g.num_layers;
  const size_t kv_elems = (size_t)g.num_layers * n_pages * g.n_heads_kv * ps * g.head_dim;
  const size_t esz = kv.f16 ? 2 : 4;
  auto kb = alloc(kv_elems * esz), vb = alloc(kv_elems * esz);
  JAL_CUDA(cudaMemset(kb->ptr, 0, kb->bytes));
  JAL_CUDA(cudaMemset(vb->ptr, 0, vb->bytes));
  kv.k = kb->ptr; kv.v = vb->ptr;
  std::vector<int32_t> pt(n_pages);
  for (uint64_t i = 0; i < n_pages; i++) pt[i] = (int32_t)i;
  auto ptb = alloc(n_pages * 4);
  JAL_CUDA(cudaMemcpy(ptb->ptr, pt.data(), n_pages * 4, cudaMemcpyHostToDevice));
  kv.page_table = ptb->as<int32_t>();
  kc->bufs = {kb, vb, ptb};
  return kc;
}

std::unique_ptr<Context> create_context(const Recipe &r, const ModelCache &c, const ContextConfig &cfg0,
                                        const KvCache *ext_kv) {
  JAL_CUDA(cudaSetDevice(c.device));
  auto ctx = std::make_unique<Context>();
  static std::atomic<uint64_t> next_uid{1};
  ctx->uid = next_uid++;
  ctx->cache = &c;
  ctx->recipe = r;
  ctx->cfg = cfg0;
  if (ctx->cfg.page_size == 0) ctx->cfg.page_size = 64;
  if (ctx->cfg.n_ctx == 0) fail(JAL_ERR_INVALID_ARGUMENT, "n_ctx must be positive");
  const Geometry &g = c.lgeom;  // this rank's heads and FFN rows
  ctx->g = g;
  if (c.plan.world > 1 && ctx->cfg.numerics == JAL_NUMERICS_REFERENCE)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "tensor parallel contexts run the fast / relaxed numerics only");
  // One GPU, FAST: the reference-order kernels (xgemv / xattn / xprefill).
  ctx->exact = ctx->cfg.numerics == JAL_NUMERICS_FAST && c.plan.world == 1;
  if (g.n_heads_q / g.n_heads_kv > 8) fail(JAL_ERR_CAPABILITY_MISMATCH, "GQA group size > 8 is not supported");
  if (g.head_dim != 64 && g.head_dim != 128) fail(JAL_ERR_CAPABILITY_MISMATCH, "head_dim must be 64 or 128");
  for (const Layer &L : c.layers) {
    if (!L.qkv_stacked || !L.gateup_stacked || !device_quant(L.wo.quant) || !device_quant(L.wdown.quant))
      fail(JAL_ERR_CAPABILITY_MISMATCH, "the device forward needs Q4_0/Q8_0 layer matrices with uniform q/k/v and gate/up quants");
  }
  if (kquant(c.lm_head.quant) && (c.plan.world > 1 || ctx->cfg.numerics == JAL_NUMERICS_RELAXED))
    fail(JAL_ERR_CAPABILITY_MISMATCH, "a K-quant LM head runs the reference-order numerics on one GPU only");
  if (!device_quant(c.lm_head.quant) && !dense_quant(c.lm_head.quant) && !kquant(c.lm_head.quant))
    fail(JAL_ERR_CAPABILITY_MISMATCH, "LM head quant %d not supported on the device path", c.lm_head.quant);
  if (dense_quant(c.lm_head.quant) && g.hidden_dim % 32 != 0)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "dense LM head: hidden dim %llu not a multiple of 32", (unsigned long long)g.hidden_dim);
  gemv_init();
  if (gemv_smem_bytes(GEMV_IN_F32, 1, (int64_t)g.ffn_dim) > (size_t)kGemvMaxSmem ||
      gemv_smem_bytes(GEMV_IN_NORM, 1, (int64_t)g.hidden_dim) > (size_t)kGemvMaxSmem)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "hidden/ffn dims exceed the decode GEMV shared-memory staging");
  JAL_CUDA(cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking));
  ctx->stream = ctx->own_stream;
  const uint64_t n_ctx = ctx->cfg.n_ctx;
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv;
  const uint64_t V = c.plan.v_pad * c.plan.world;  // gathered logits (>= vocab)
  if (ext_kv) {  // a caller-owned cache: its geometry must be this model's
    const KvView &e = ext_kv->kv;
    if (ext_kv->device != c.device || e.n_layers != (int64_t)g.num_layers || e.n_kv != (int64_t)g.n_heads_kv ||
        e.head_dim != (int64_t)g.head_dim)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "KV cache was allocated for another model geometry or device");
    if (e.f16 != ctx->cfg.kv_f16 || (uint64_t)e.page_size != ctx->cfg.page_size)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "KV cache dtype / page size differ from the context configuration");
    if (n_ctx > ext_kv->n_ctx)
      fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "context n_ctx %llu exceeds the KV cache's %llu positions",
           (unsigned long long)n_ctx, (unsigned long long)ext_kv->n_ctx);
    ctx->kv = e;
  } else {
    ctx->own_kv = create_kv_cache(c, n_ctx, ctx->cfg.kv_f16, ctx->cfg.page_size);
    ctx->kv = ctx->own_kv->kv;
  }
  KvView &kv = ctx->kv;
  // RoPE tables.
  uint64_t half = g.rotary_dim / 2;
  std::vector<float> inv(half), cs, sn;
  fill_inv_freq(g.rotary_dim, r.rope_theta, r.scaling, 0, inv.data());
  build_rope_table(n_ctx, g.rotary_dim, inv, cs, sn);
  auto tb = alloc(cs.size() * 4 * 4);
  ctx->bufs.push_back(tb);
  ctx->cos_tab = tb->as<float>();
  ctx->sin_tab = ctx->cos_tab + cs.size();
  JAL_CUDA(cudaMemcpy(ctx->cos_tab, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  JAL_CUDA(cudaMemcpy(ctx->sin_tab, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  ctx->cos_long = ctx->sin_tab + sn.size();
  ctx->sin_long = ctx->cos_long + cs.size();
  if (r.scaling.kind == JAL_ROPE_SCALING_LONGROPE) {
    fill_inv_freq(g.rotary_dim, r.rope_theta, r.scaling, r.scaling.original_max_position_embeddings + 1, inv.data());
    build_rope_table(n_ctx, g.rotary_dim, inv, cs, sn);
    JAL_CUDA(cudaMemcpy(ctx->cos_long, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    JAL_CUDA(cudaMemcpy(ctx->sin_long, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }
  norm_init();
  if (ctx->exact) {
    xgemv_init();
    auto need = [&](const DevMat &w, int in_mode, int out_mode, int64_t rows, const char *what) {
      GemvArgs t;
      t.w = w; t.m = 1; t.in_mode = in_mode; t.out_mode = out_mode; t.rows = rows;
      if (!xgemv_supported(t))
        fail(JAL_ERR_CAPABILITY_MISMATCH, "%s: shape not supported by the reference-order decode GEMV", what);
    };
    for (const Layer &L : c.layers) {
      need(L.qkv, GEMV_IN_NORM, GEMV_OUT_STORE, (int64_t)(g.total_q + 2 * g.total_kv), "Q/K/V");
      need(L.wo.dm, GEMV_IN_Q8, GEMV_OUT_ADD, (int64_t)g.hidden_dim, "O");
      need(L.gateup, GEMV_IN_NORM, GEMV_OUT_SWIGLU, (int64_t)g.ffn_dim, "gate/up");
      need(L.wdown.dm, GEMV_IN_F32, GEMV_OUT_ADD, (int64_t)g.hidden_dim, "down");
    }
    if (!dense_quant(c.lm_head.quant) && !kquant(c.lm_head.quant))
      need(c.lm_head.dm, GEMV_IN_NORM, GEMV_OUT_STORE, (int64_t)c.vocab_size, "LM head");
    ctx->x_splits = xattn_cluster_size((int)g.head_dim, ctx->cfg.kv_f16, (int)(g.n_heads_q / g.n_heads_kv),
                                       (int)g.n_heads_kv, (int64_t)ctx->cfg.n_ctx);
    if (ctx->x_splits <= 0)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention: n_ctx %llu does not fit",
           (unsigned long long)ctx->cfg.n_ctx);
    const uint64_t keys = ctx->cfg.sliding_window ? std::min<uint64_t>(ctx->cfg.sliding_window, ctx->cfg.n_ctx)
                                                  : ctx->cfg.n_ctx;
    if (!xattn_prefill_supported((int64_t)g.head_dim, (int64_t)keys + 4))
      fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order prefill attention: n_ctx %llu does not fit",
           (unsigned long long)ctx->cfg.n_ctx);
    if (!xattn_v_supported((int64_t)g.head_dim, kv.page_size, (int64_t)ctx->cfg.n_ctx))
      fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention output: n_ctx %llu does not fit",
           (unsigned long long)ctx->cfg.n_ctx);
    if (!make_kv_tensor_map(kv, kv.v, ctx->tm_v))
      fail(JAL_ERR_CUDA, "reference-order decode attention: the driver refused the V tensor map");
    auto wb = alloc((size_t)g.n_heads_q * ctx->cfg.n_ctx * 4);
    ctx->bufs.push_back(wb);
    ctx->attn_w = wb->as<float>();
  }
  // Decode buffers.
  const int sms = sm_count();
  ctx->n_splits = attn_decode_cluster_size((int)g.head_dim, kv.f16, (int)(g.n_heads_q / g.n_heads_kv), n_ctx >= 512 ? 16 : 4);
  ctx->am_blocks = sms;
  size_t f32s = H + (Q + 2 * KV) + Q + Q / 32 + F + (F + 31) / 32 + V + sms;
  size_t bytes = f32s * 4 + Q + ((F + 31) / 32) * 32 + 4096 + (F / 32 + 1) * 4 + 64 + (size_t)sms * 4 + (n_ctx + 2) * 4 +
                 32 * 256 + c.plan.v_pad * 4 + H * 4 + 768;
  auto db = alloc(bytes + 1024);
  ctx->bufs.push_back(db);
  JAL_CUDA(cudaMemset(db->ptr, 0, db->bytes));
  char *p = db->as<char>();
  auto take = [&](size_t n) { char *q = p; p += (n + 255) / 256 * 256; return q; };
  ctx->d_pos = (int64_t *)take(8);
  ctx->d_token = (uint32_t *)take(4);
  ctx->d_err = (int *)take(4);
  ctx->hidden = (float *)take(H * 4);
  ctx->qkv = (float *)take((Q + 2 * KV) * 4);
  ctx->attn = (float *)take(Q * 4);
  ctx->attn_q = (int8_t *)take(Q);
  ctx->attn_s = (float *)take(Q / 32 * 4);
  ctx->ffn = (float *)take(F * 4);
  ctx->ffn_q = (int8_t *)take((F + 31) / 32 * 32);
  ctx->ffn_s = (float *)take((F + 31) / 32 * 4);
  ctx->ffn_cnt = (unsigned *)take((F + 31) / 32 * 4);
  ctx->logits = (float *)take(V * 4);
  ctx->logits_local = c.plan.world > 1 ? (float *)take(c.plan.v_pad * 4) : ctx->logits;
  ctx->am_val = (float *)take(sms * 4);
  ctx->am_idx = (int *)take(sms * 4);
  ctx->am_cnt = (unsigned *)take(4);
  ctx->d_hist = (uint32_t *)take((n_ctx + 2) * 4);
  ctx->hidden_b = (float *)take(H * 4);
  ctx->d_xepoch = (uint32_t *)take(4);
  if ((size_t)(p - db->as<char>()) > db->bytes) fail(JAL_ERR_INVALID_ARGUMENT, "internal: decode scratch layout overflow");
  if (c.tp && c.plan.world > 1) setup_tp_exchange(*ctx, sms);
  {  // reference-order scratch: normed row, int8 activations + scales, gate|up, q
    const uint64_t kmax = std::max<uint64_t>(std::max<uint64_t>(H, Q), F), kp = (kmax + 31) / 32 * 32;
    auto sb = alloc((H + kp / 32 + 2 * F + Q) * 4 + kp + 5 * 256);
    ctx->bufs.push_back(sb);
    char *q = sb->as<char>();
    auto take2 = [&](size_t n) { char *r = q; q += (n + 255) / 256 * 256; return r; };
    ctx->s_norm = (float *)take2(H * 4);
    ctx->s_sc = (float *)take2(kp / 32 * 4);
    ctx->s_gu = (float *)take2(2 * F * 4);
    ctx->s_qbuf = (float *)take2(Q * 4);
    ctx->s_q8 = (int8_t *)take2(kp);
  }
  setup_mega(*ctx, sms);
  JAL_CUDA(cudaMallocHost(&ctx->h_pos, 8));
  JAL_CUDA(cudaMallocHost(&ctx->h_token, 4 * 8));
  JAL_CUDA(cudaStreamSynchronize(ctx->stream));
  return ctx;
}

// Tensor-parallel exchange over peer memory for the decode step: a
// symmetric allocation of flagged-word slots mapped on every rank.
// Collective over the ranks; on any mismatch (a shape off the segmented
// GEMV, too many layers for the flag's phase field, no peer mapping) every
// rank keeps the NCCL all-reduce.
static void setup_tp_exchange(Context &ctx, int sms) {
  (void)sms;
  const ModelCache &c = *ctx.cache;
  const int W = c.plan.world;
  const uint64_t H = ctx.g.hidden_dim;
  const size_t L = c.layers.size();
  bool ok = W <= kPeerMax && L >= 1 && 2 * L <= 255 && !env_flag("JAL_TP_NCCL");
  if (ok) {
    const Layer &L0 = c.layers[0];
    unsigned long long *dummy = (unsigned long long *)ctx.hidden_b;
    GemvArgs pa;  // producer (O / down)
    pa.m = 1; pa.out_mode = GEMV_OUT_PEER; pa.peer_world = W; pa.rows = (int64_t)H; pa.peer_epoch = ctx.d_xepoch;
    for (int r = 0; r < W; r++) pa.peer_out[r] = dummy;
    GemvArgs po = pa, pd = pa;
    po.w = L0.wo.dm; po.in_mode = GEMV_IN_Q8;
    pd.w = L0.wdown.dm; pd.in_mode = GEMV_IN_F32;
    GemvArgs ca;  // consumers (QKV, gate / up, LM head)
    ca.m = 1; ca.in_mode = GEMV_IN_NORM; ca.peer_in = dummy; ca.peer_epoch = ctx.d_xepoch; ca.peer_world = W;
    ca.x_stride = (int64_t)H;
    GemvArgs cq = ca, cg = ca, cl = ca;
    cq.w = L0.qkv; cq.rows = L0.qkv.rows; cq.out_mode = GEMV_OUT_STORE;
    cg.w = L0.gateup; cg.rows = (int64_t)ctx.g.ffn_dim; cg.out_mode = GEMV_OUT_SWIGLU; cg.up_offset = (int64_t)ctx.g.ffn_dim;
    cl.w = c.lm_head.dm; cl.rows = (int64_t)c.plan.v_n; cl.out_mode = GEMV_OUT_STORE;
    ok = gemv_peer_supported(po) && gemv_peer_supported(pd) && gemv_peer_supported(cq) && gemv_peer_supported(cg) &&
         gemv_peer_supported(cl);
  }
  // Agree before the collective allocation (a rank that opts out by its
  // environment must not leave the others waiting in it).
  float no = ok ? 0.0f : 1.0f;
  JAL_CUDA(cudaMemcpyAsync(ctx.am_val, &no, 4, cudaMemcpyHostToDevice, ctx.stream));
  tp_all_reduce(*c.tp, ctx.am_val, 1, ctx.stream);
  JAL_CUDA(cudaMemcpyAsync(&no, ctx.am_val, 4, cudaMemcpyDeviceToHost, ctx.stream));
  JAL_CUDA(cudaStreamSynchronize(ctx.stream));
  if (no != 0.0f) return;
  ctx.tp_sym.reset(tp_symmetric_alloc(*c.tp, 2 * (size_t)W * H * 8, ctx.stream));
}

size_t decode_scratch_bytes(const Recipe &r, uint64_t seq) {  // recipe.rs:529-547 (device buffers)
  uint64_t hd = std::max<uint64_t>(r.head_dim, 2);
  if (hd % 2) hd -= 1;
  uint64_t Q = std::max<uint64_t>(r.n_heads_q, 1) * hd, KV = std::max<uint64_t>(r.n_heads_kv, 1) * hd;
  uint64_t H = std::max<uint64_t>(r.hidden_dim, 2), F = std::max<uint64_t>(r.ffn_dim, 2);
  uint64_t kv = std::max<uint64_t>(r.num_layers, 1) * 2 * std::max<uint64_t>(seq, 1) * KV * 2;
  return (size_t)(kv + 4 * (H + Q + 2 * KV + Q + F + r.vocab_size) + Q + F + 65536);
}

Context::~Context() {
  if (graph) cudaGraphExecDestroy(graph);
  if (bt_graph) cudaGraphExecDestroy(bt_graph);
  for (cudaStream_t s : bt_streams) { cudaStreamSynchronize(s); cudaStreamDestroy(s); }
  for (cudaEvent_t e : bt_events) cudaEventDestroy(e);
  if (h_pos) cudaFreeHost(h_pos);
  if (h_token) cudaFreeHost(h_token);
  if (stream) cudaStreamSynchronize(stream);
  if (own_stream) { cudaStreamSynchronize(own_stream); cudaStreamDestroy(own_stream); }
}

void Context::enqueue_decode_step(bool pdl) {
  const ModelCache &c = *cache;
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv;
  const float eps = std::max(recipe.rms_eps, 1.0e-7f);
  size_t n = 0;
  launch_embed(c.emb_raw->as<uint8_t>(), c.emb_quant, (int64_t)H, (int64_t)c.emb_rows, d_token, 1, hidden, d_err, pdl,
               stream);
  n++;
  // Tensor parallelism over peer memory: O and down (phases 2l, 2l + 1)
  // store their partial rows as flagged words into every rank's slots of
  // parity phase % 2; the next RMSNorm GEMV waits for the words of its step
  // and phase, adds them to the residual it reads (hidden for even phases,
  // hidden_b for odd ones) and writes the sum to the other buffer.  The
  // argmax at the end of the step advances the flag epoch.
  const bool xp = tp_sym != nullptr;
  const int W = c.plan.world, rank = c.plan.rank;
  auto x_slots = [&](int r, size_t parity) {  // rank r's slots [world][H] of this parity
    return (unsigned long long *)tp_sym->peer[r] + parity * (size_t)W * H;
  };
  auto produce = [&](GemvArgs &a, size_t phase) {
    a.out_mode = GEMV_OUT_PEER; a.y = nullptr; a.peer_world = W;
    a.peer_epoch = d_xepoch; a.peer_phase = (int)phase;
    for (int r = 0; r < W; r++) a.peer_out[r] = x_slots(r, phase % 2) + (size_t)rank * H;
  };
  auto consume = [&](GemvArgs &a, size_t phase) {
    a.peer_in = x_slots(rank, phase % 2); a.peer_world = W; a.err = d_err;
    a.peer_epoch = d_xepoch; a.peer_phase = (int)phase;
    a.x = phase % 2 ? hidden_b : hidden;
    a.x_out = phase % 2 ? hidden : hidden_b;
  };
  for (size_t l = 0; l < c.layers.size(); l++) {
    const Layer &L = c.layers[l];
    GemvArgs qa;
    qa.w = L.qkv; qa.rows = (int64_t)(Q + 2 * KV); qa.m = 1; qa.in_mode = GEMV_IN_NORM;
    qa.x = hidden; qa.x_stride = (int64_t)H; qa.norm_w = L.attn_norm; qa.eps = eps;
    qa.out_mode = GEMV_OUT_STORE; qa.y = qkv; qa.y_stride = (int64_t)(Q + 2 * KV); qa.pdl = pdl;
    if (xp && l > 0) consume(qa, 2 * l - 1);
    launch_gemv(qa, stream);
    AttnDecodeArgs aa;
    aa.qkv = qkv; aa.bq = L.bq; aa.bk = L.bk; aa.bv = L.bv;
    aa.cos_tab = cos_tab; aa.sin_tab = sin_tab; aa.cos_tab_long = cos_long; aa.sin_tab_long = sin_long;
    aa.long_threshold = recipe.scaling.kind == JAL_ROPE_SCALING_LONGROPE
                            ? (int64_t)recipe.scaling.original_max_position_embeddings : -1;
    aa.skip_rope = recipe.should_skip_rope(l); aa.neox = recipe.rope_type == JAL_ROPE_NEOX;
    aa.n_heads_q = (int64_t)g.n_heads_q; aa.rotary_dim = (int64_t)g.rotary_dim;
    aa.kv = kv; aa.layer = (int64_t)l; aa.d_pos = d_pos; aa.window = (int64_t)cfg.sliding_window;
    aa.scale = 1.0f / sqrtf((float)g.head_dim);
    aa.n_splits = n_splits;
    aa.out = attn; aa.out_q = attn_q; aa.out_s = attn_s; aa.err = d_err; aa.pdl = pdl;
    launch_attn_decode(aa, stream);
    GemvArgs oa;
    oa.w = L.wo.dm; oa.rows = (int64_t)H; oa.m = 1; oa.in_mode = GEMV_IN_Q8;
    oa.xq = attn_q; oa.xs = attn_s; oa.xq_stride = (int64_t)Q;
    // tensor parallel: rank 0 adds its partial to the residual, the others
    // store theirs, and the all-reduce sums them into the new residual
    oa.out_mode = c.plan.rank == 0 ? GEMV_OUT_ADD : GEMV_OUT_STORE; oa.y = hidden; oa.y_stride = (int64_t)H;
    oa.bias = L.bo; oa.pdl = pdl;
    if (xp) produce(oa, 2 * l);
    launch_gemv(oa, stream);
    if (c.tp && !xp) tp_all_reduce(*c.tp, hidden, H, stream);
    GemvArgs ga;
    ga.w = L.gateup; ga.rows = (int64_t)F; ga.m = 1; ga.in_mode = GEMV_IN_NORM;
    ga.x = hidden; ga.x_stride = (int64_t)H; ga.norm_w = L.ffn_norm; ga.eps = eps;
    ga.out_mode = GEMV_OUT_SWIGLU; ga.y = ffn; ga.y_stride = (int64_t)F; ga.up_offset = (int64_t)F; ga.pdl = pdl;
    if (xp) consume(ga, 2 * l);
    launch_gemv(ga, stream);
    GemvArgs da;
    da.w = L.wdown.dm; da.rows = (int64_t)H; da.m = 1; da.in_mode = GEMV_IN_F32;
    da.x = ffn; da.x_stride = (int64_t)F;
    da.out_mode = c.plan.rank == 0 ? GEMV_OUT_ADD : GEMV_OUT_STORE; da.y = hidden; da.y_stride = (int64_t)H;
    da.pdl = pdl;
    if (xp) produce(da, 2 * l + 1);
    launch_gemv(da, stream);
    if (c.tp && !xp) tp_all_reduce(*c.tp, hidden, H, stream);
    n += 5;
  }
  GemvArgs la;
  la.w = c.lm_head.dm; la.rows = (int64_t)c.plan.v_n; la.m = 1; la.in_mode = GEMV_IN_NORM;
  la.x = hidden; la.x_stride = (int64_t)H; la.norm_w = c.output_norm->as<float>(); la.eps = eps;
  la.out_mode = GEMV_OUT_STORE; la.y = logits_local; la.y_stride = (int64_t)c.plan.v_pad; la.pdl = pdl;
  if (xp && !c.layers.empty()) {
    consume(la, 2 * c.layers.size() - 1);
    la.x_out = nullptr;  // the residual after the last layer is not needed again
  }
  launch_gemv(la, stream);
  if (c.tp) tp_all_gather(*c.tp, logits_local, logits, c.plan.v_pad, stream);
  launch_argmax(logits, (int64_t)c.vocab_size, am_val, am_idx, am_cnt, am_blocks, d_token, d_pos, d_hist, pdl, stream,
                xp ? d_xepoch : nullptr);
  n += 2;
  launches_per_step = n;
}

// A K-quant LM head (Q4_K / Q5_K / Q6_K; llama.cpp's usual output type) in
// the reference's order for one row: the final RMSNorm, QuantizedActQ8 of
// the normed row and the repacked projection with the group-min term
// (repack_cache.rs:739-783), into logits[vocab].
static void kq_lm_head(const ModelCache &c, const float *x, int64_t H, float eps, float *s_norm, int8_t *s_q8,
                       float *s_sc, float *logits, cudaStream_t s) {
  launch_rmsnorm(x, c.output_norm->as<float>(), 1, H, eps, s_norm, s);
  launch_act_quant(s_norm, 1, H, H, s_q8, s_sc, s);
  launch_kq_gemm(c.lm_head.dm, s_norm, s_q8, s_sc, 1, logits, s);
}

// The serving step in the reference's f32 order (FAST numerics, one GPU):
// embedding, per layer Q/K/V (RMSNorm prologue) -> attention (bias, RoPE,
// append) -> O (+ bias, residual) -> gate/up (RMSNorm prologue, SwiGLU) ->
// down (residual), then the LM head (RMSNorm prologue) and the greedy argmax:
// 1 + 5L + 2 launches chained with programmatic dependent launch.
void Context::enqueue_exact_step(bool pdl) {
  const ModelCache &c = *cache;
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv;
  const float eps = std::max(recipe.rms_eps, 1.0e-7f);
  size_t n = 0;
  auto tr = [&](size_t i) { return trace_on ? d_trace + kTraceSlots * i : nullptr; };
  launch_embed(c.emb_raw->as<uint8_t>(), c.emb_quant, (int64_t)H, (int64_t)c.emb_rows, d_token, 1, hidden, d_err, pdl,
               stream);
  n++;
  for (size_t l = 0; l < c.layers.size(); l++) {
    const Layer &L = c.layers[l];
    GemvArgs qa;
    qa.trace = tr(n);
    qa.w = L.qkv; qa.rows = (int64_t)(Q + 2 * KV); qa.in_mode = GEMV_IN_NORM;
    qa.x = hidden; qa.x_stride = (int64_t)H; qa.norm_w = L.attn_norm; qa.eps = eps;
    qa.out_mode = GEMV_OUT_STORE; qa.y = qkv; qa.y_stride = (int64_t)(Q + 2 * KV); qa.pdl = pdl;
    launch_xgemv(qa, stream);
    AttnDecodeArgs aa;
    aa.qkv = qkv; aa.bq = L.bq; aa.bk = L.bk; aa.bv = L.bv;
    aa.cos_tab = cos_tab; aa.sin_tab = sin_tab; aa.cos_tab_long = cos_long; aa.sin_tab_long = sin_long;
    aa.long_threshold = recipe.scaling.kind == JAL_ROPE_SCALING_LONGROPE
                            ? (int64_t)recipe.scaling.original_max_position_embeddings : -1;
    aa.skip_rope = recipe.should_skip_rope(l); aa.neox = recipe.rope_type == JAL_ROPE_NEOX;
    aa.n_heads_q = (int64_t)g.n_heads_q; aa.rotary_dim = (int64_t)g.rotary_dim;
    aa.kv = kv; aa.layer = (int64_t)l; aa.d_pos = d_pos; aa.window = (int64_t)cfg.sliding_window;
    aa.scale = 1.0f / sqrtf((float)g.head_dim);
    aa.n_splits = x_splits;
    aa.w_out = attn_w; aa.w_stride = (int64_t)cfg.n_ctx; aa.err = d_err; aa.pdl = pdl;
    aa.trace = tr(n + 1);
    launch_xattn_decode(aa, (int64_t)cfg.n_ctx, stream);
    AttnVArgs va;
    va.kv = kv; va.layer = (int64_t)l; va.window = (int64_t)cfg.sliding_window; va.n_heads_q = (int64_t)g.n_heads_q;
    va.d_pos = d_pos; va.w = attn_w; va.w_stride = (int64_t)cfg.n_ctx;
    va.out = attn; va.out_q = attn_q; va.out_s = attn_s; va.err = d_err; va.pdl = pdl;
    va.test_extra_tx = test_stall_tx; va.wait_ns = test_wait_ns;
    va.trace = tr(n + 2);
    launch_xattn_v(tm_v, va, (int64_t)cfg.n_ctx, stream);
    GemvArgs oa;
    oa.w = L.wo.dm; oa.rows = (int64_t)H; oa.in_mode = GEMV_IN_Q8;
    oa.xq = attn_q; oa.xs = attn_s; oa.xq_stride = (int64_t)Q;
    oa.out_mode = GEMV_OUT_ADD; oa.y = hidden; oa.y_stride = (int64_t)H; oa.bias = L.bo; oa.pdl = pdl;
    oa.trace = tr(n + 3);
    launch_xgemv(oa, stream);
    GemvArgs ga;
    ga.w = L.gateup; ga.rows = (int64_t)F; ga.in_mode = GEMV_IN_NORM;
    ga.x = hidden; ga.x_stride = (int64_t)H; ga.norm_w = L.ffn_norm; ga.eps = eps;
    ga.out_mode = GEMV_OUT_SWIGLU; ga.y = ffn; ga.y_stride = (int64_t)F; ga.up_offset = (int64_t)F; ga.pdl = pdl;
    ga.trace = tr(n + 4);
    launch_xgemv(ga, stream);
    GemvArgs da;
    da.w = L.wdown.dm; da.rows = (int64_t)H; da.in_mode = GEMV_IN_F32; da.x = ffn; da.x_stride = (int64_t)F;
    da.out_mode = GEMV_OUT_ADD; da.y = hidden; da.y_stride = (int64_t)H; da.pdl = pdl;
    da.trace = tr(n + 5);
    launch_xgemv(da, stream);
    n += 6;
  }
  if (dense_quant(c.lm_head.dm.quant)) {
    launch_rmsnorm(hidden, c.output_norm->as<float>(), 1, (int64_t)H, eps, s_norm, stream);
    launch_strict_gemv_dense(c.lm_head.dm, s_norm, (int64_t)c.vocab_size, logits, stream);
    n += 2;
  } else if (kquant(c.lm_head.dm.quant)) {
    kq_lm_head(c, hidden, (int64_t)H, eps, s_norm, s_q8, s_sc, logits, stream);
    n += 3;
  } else {
    GemvArgs la;
    la.w = c.lm_head.dm; la.rows = (int64_t)c.vocab_size; la.in_mode = GEMV_IN_NORM;
    la.x = hidden; la.x_stride = (int64_t)H; la.norm_w = c.output_norm->as<float>(); la.eps = eps;
    la.out_mode = GEMV_OUT_STORE; la.y = logits; la.y_stride = (int64_t)c.vocab_size; la.pdl = pdl;
    la.trace = tr(n);
    launch_xgemv(la, stream);
    n++;
  }
  launch_argmax(logits, (int64_t)c.vocab_size, am_val, am_idx, am_cnt, am_blocks, d_token, d_pos, d_hist, pdl, stream);
  n++;
  launches_per_step = n;
}

// Batched decode of independent sequences (no counterpart in the reference,
// whose batched forward is one sequence's prompt): per layer RMSNorm +
// QuantizedActQ8 of the n rows, the Q/K/V GEMM, per sequence the two
// reference-order attention kernels on that context's KV cache and position
// (writing its row of the O input; each sequence on its own side stream),
// then the O, gate/up and down GEMMs with the residual adds, and the LM head
// over the n rows.  Every f32 sum keeps the reference's order, so each row
// equals the single-sequence step.
void batch_decode_step(Context *const *cs, size_t n, const uint32_t *d_tokens) {
  Context &c0 = *cs[0];
  const ModelCache &c = *c0.cache;
  const Geometry &g = c0.g;
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv, V = c.vocab_size;
  const float eps = std::max(c0.recipe.rms_eps, 1.0e-7f);
  const int64_t m = (int64_t)n;
  cudaStream_t s = c0.stream;
  float *hid = c0.pf_hidden, *qkv = c0.pf_qkv, *att = c0.pf_attn, *gu = c0.pf_gu, *xs = c0.pf_xs;
  int8_t *xq = c0.pf_xq;
  launch_embed(c.emb_raw->as<uint8_t>(), c.emb_quant, (int64_t)H, (int64_t)c.emb_rows, d_tokens, m, hid, c0.d_err, 0,
               s);
  for (size_t l = 0; l < c.layers.size(); l++) {
    const Layer &L = c.layers[l];
    launch_rmsnorm_quant(hid, L.attn_norm, m, (int64_t)H, eps, xq, xs, s);
    GemmArgs qa;
    qa.w = L.qkv; qa.m = m; qa.rows = (int64_t)(Q + 2 * KV); qa.xq = xq; qa.xs = xs;
    qa.y = qkv; qa.y_stride = (int64_t)(Q + 2 * KV);
    launch_gemm(qa, s);
    JAL_CUDA(cudaEventRecord(c0.bt_events[0], s));
    for (size_t b = 0; b < n; b++) {
      Context &cb = *cs[b];
      cudaStream_t sb = c0.bt_streams[b];
      JAL_CUDA(cudaStreamWaitEvent(sb, c0.bt_events[0], 0));
      AttnDecodeArgs aa;
      aa.qkv = qkv + b * (Q + 2 * KV); aa.bq = L.bq; aa.bk = L.bk; aa.bv = L.bv;
      aa.cos_tab = cb.cos_tab; aa.sin_tab = cb.sin_tab; aa.cos_tab_long = cb.cos_long; aa.sin_tab_long = cb.sin_long;
      aa.long_threshold = cb.recipe.scaling.kind == JAL_ROPE_SCALING_LONGROPE
                              ? (int64_t)cb.recipe.scaling.original_max_position_embeddings : -1;
      aa.skip_rope = cb.recipe.should_skip_rope(l); aa.neox = cb.recipe.rope_type == JAL_ROPE_NEOX;
      aa.n_heads_q = (int64_t)g.n_heads_q; aa.rotary_dim = (int64_t)g.rotary_dim;
      aa.kv = cb.kv; aa.layer = (int64_t)l; aa.d_pos = cb.d_pos; aa.window = (int64_t)cb.cfg.sliding_window;
      aa.scale = 1.0f / sqrtf((float)g.head_dim);
      aa.n_splits = cb.bt_splits;
      aa.w_out = cb.attn_w; aa.w_stride = (int64_t)cb.cfg.n_ctx; aa.err = c0.d_err; aa.pdl = 0;
      launch_xattn_decode(aa, (int64_t)cb.cfg.n_ctx, sb);
      AttnVArgs va;
      va.kv = cb.kv; va.layer = (int64_t)l; va.window = (int64_t)cb.cfg.sliding_window;
      va.n_heads_q = (int64_t)g.n_heads_q; va.d_pos = cb.d_pos; va.w = cb.attn_w; va.w_stride = (int64_t)cb.cfg.n_ctx;
      va.out = att + b * Q; va.out_q = xq + b * Q; va.out_s = xs + b * (Q / 32); va.err = c0.d_err; va.pdl = 0;
      launch_xattn_v(cb.tm_v, va, (int64_t)cb.cfg.n_ctx, sb);
      JAL_CUDA(cudaEventRecord(c0.bt_events[1 + b], sb));
    }
    for (size_t b = 0; b < n; b++) JAL_CUDA(cudaStreamWaitEvent(s, c0.bt_events[1 + b], 0));
    GemmArgs oa;
    oa.w = L.wo.dm; oa.m = m; oa.rows = (int64_t)H; oa.xq = xq; oa.xs = xs;
    oa.y = hid; oa.y_stride = (int64_t)H; oa.bias = L.bo; oa.accumulate = 1;
    launch_gemm(oa, s);
    launch_rmsnorm_quant(hid, L.ffn_norm, m, (int64_t)H, eps, xq, xs, s);
    GemmArgs ga;
    ga.w = L.gateup; ga.m = m; ga.rows = (int64_t)(2 * F); ga.xq = xq; ga.xs = xs;
    ga.y = gu; ga.y_stride = (int64_t)(2 * F);
    launch_gemm(ga, s);
    launch_swiglu_act_quant(gu, m, (int64_t)F, (int64_t)(2 * F), xq, xs, s);
    GemmArgs da;
    da.w = L.wdown.dm; da.m = m; da.rows = (int64_t)H; da.xq = xq; da.xs = xs;
    da.y = hid; da.y_stride = (int64_t)H; da.accumulate = 1;
    launch_gemm(da, s);
  }
  if (dense_quant(c.lm_head.dm.quant)) {
    for (size_t b = 0; b < n; b++) {
      launch_rmsnorm(hid + b * H, c.output_norm->as<float>(), 1, (int64_t)H, eps, c0.s_norm, s);
      launch_strict_gemv_dense(c.lm_head.dm, c0.s_norm, (int64_t)V, c0.bt_logits + b * V, s);
    }
  } else if (kquant(c.lm_head.dm.quant)) {
    for (size_t b = 0; b < n; b++)
      kq_lm_head(c, hid + b * H, (int64_t)H, eps, c0.s_norm, c0.s_q8, c0.s_sc, c0.bt_logits + b * V, s);
  } else {
    launch_rmsnorm_quant(hid, c.output_norm->as<float>(), m, (int64_t)H, eps, xq, xs, s);
    GemmArgs la;
    la.w = c.lm_head.dm; la.m = m; la.rows = (int64_t)V; la.xq = xq; la.xs = xs;
    la.y = c0.bt_logits; la.y_stride = (int64_t)V;
    launch_gemm(la, s);
  }
  JAL_CUDA(cudaGetLastError());
}

void run_batch_decode(Context *const *cs, size_t n) {
  Context &c0 = *cs[0];
  const ModelCache &c = *c0.cache;
  const uint64_t V = c.vocab_size;
  cudaStream_t s = c0.stream;
  if (c0.bt_cap < n) {
    JAL_CUDA(cudaStreamSynchronize(s));
    c0.bt_buf = alloc(n * V * 4);
    c0.pf_gen++;
    c0.bt_logits = c0.bt_buf->as<float>();
    c0.bt_cap = n;
  }
  while (c0.bt_streams.size() < n) {
    cudaStream_t t;
    JAL_CUDA(cudaStreamCreateWithFlags(&t, cudaStreamNonBlocking));
    c0.bt_streams.push_back(t);
  }
  while (c0.bt_events.size() < n + 1) {
    cudaEvent_t e;
    JAL_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    c0.bt_events.push_back(e);
  }
  std::vector<uint64_t> key = {n, c0.pf_gen};
  for (size_t b = 0; b < n; b++) {
    Context &cb = *cs[b];
    if (!cb.bt_splits) {
      cb.bt_splits = xattn_batch_cluster_size((int)cb.g.head_dim, cb.cfg.kv_f16, (int)(cb.g.n_heads_q / cb.g.n_heads_kv),
                                              (int64_t)cb.cfg.n_ctx);
      if (!cb.bt_splits) fail(JAL_ERR_CAPABILITY_MISMATCH, "batched decode: attention shape not supported");
    }
    key.push_back(cb.uid);
  }
  if (!c0.cfg.use_graphs) {
    batch_decode_step(cs, n, c0.pf_tokens);
    return;
  }
  if (!c0.bt_graph || c0.bt_key != key) {
    if (c0.bt_graph) {
      JAL_CUDA(cudaStreamSynchronize(s));
      cudaGraphExecDestroy(c0.bt_graph);
      c0.bt_graph = nullptr;
    }
    cudaGraph_t gr = nullptr;
    JAL_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      batch_decode_step(cs, n, c0.pf_tokens);
    } catch (...) {
      cudaStreamEndCapture(s, &gr);
      if (gr) cudaGraphDestroy(gr);
      cudaGetLastError();
      throw;
    }
    cudaError_t e = cudaStreamEndCapture(s, &gr);
    if (e != cudaSuccess) {
      cudaGetLastError();
      fail(JAL_ERR_CUDA, "batched decode graph capture failed: %s", cudaGetErrorString(e));
    }
    e = cudaGraphInstantiate(&c0.bt_graph, gr, 0);
    cudaGraphDestroy(gr);
    if (e != cudaSuccess) {
      c0.bt_graph = nullptr;
      fail(JAL_ERR_CUDA, "batched decode graph instantiate failed: %s", cudaGetErrorString(e));
    }
    c0.bt_key = key;
  }
  JAL_CUDA(cudaGraphLaunch(c0.bt_graph, s));
}

// Reference-order step (see strict.cu): the same layer sequence as
// forward_tokens of the reference for one token.
void Context::enqueue_strict_token(bool logits_out, bool argmax) {
  const ModelCache &c = *cache;
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv;
  const float eps = std::max(recipe.rms_eps, 1.0e-7f);
  launch_embed(c.emb_raw->as<uint8_t>(), c.emb_quant, (int64_t)H, (int64_t)c.emb_rows, d_token, 1, hidden, d_err, 0,
               stream);
  for (size_t l = 0; l < c.layers.size(); l++) {
    const Layer &L = c.layers[l];
    launch_strict_rmsnorm(hidden, L.attn_norm, (int64_t)H, eps, s_norm, stream);
    launch_act_quant(s_norm, 1, (int64_t)H, (int64_t)H, s_q8, s_sc, stream);
    launch_strict_gemv(L.qkv, s_q8, s_sc, (int64_t)(Q + 2 * KV), false, qkv, nullptr, stream);
    StrictQkvArgs qa;
    qa.qkv = qkv; qa.bq = L.bq; qa.bk = L.bk; qa.bv = L.bv;
    qa.cos_tab = cos_tab; qa.sin_tab = sin_tab; qa.cos_tab_long = cos_long; qa.sin_tab_long = sin_long;
    qa.long_threshold = recipe.scaling.kind == JAL_ROPE_SCALING_LONGROPE
                            ? (int64_t)recipe.scaling.original_max_position_embeddings : -1;
    qa.skip_rope = recipe.should_skip_rope(l); qa.neox = recipe.rope_type == JAL_ROPE_NEOX;
    qa.n_heads_q = (int64_t)g.n_heads_q; qa.rotary_dim = (int64_t)g.rotary_dim; qa.layer = (int64_t)l;
    qa.kv = kv; qa.d_pos = d_pos; qa.qbuf = s_qbuf;
    launch_strict_qkv_prep(qa, stream);
    StrictAttnArgs aa;
    aa.qbuf = s_qbuf; aa.kv = kv; aa.n_heads_q = (int64_t)g.n_heads_q; aa.layer = (int64_t)l;
    aa.window = (int64_t)cfg.sliding_window; aa.d_pos = d_pos; aa.scale = 1.0f / sqrtf((float)g.head_dim);
    aa.out = attn;
    launch_strict_attn(aa, (int64_t)cfg.n_ctx, stream);
    launch_act_quant(attn, 1, (int64_t)Q, (int64_t)Q, s_q8, s_sc, stream);
    launch_strict_gemv(L.wo.dm, s_q8, s_sc, (int64_t)H, true, hidden, L.bo, stream);
    launch_strict_rmsnorm(hidden, L.ffn_norm, (int64_t)H, eps, s_norm, stream);
    launch_act_quant(s_norm, 1, (int64_t)H, (int64_t)H, s_q8, s_sc, stream);
    launch_strict_gemv(L.gateup, s_q8, s_sc, (int64_t)(2 * F), false, s_gu, nullptr, stream);
    launch_strict_swiglu(s_gu, s_gu + F, (int64_t)F, ffn, stream);
    launch_act_quant(ffn, 1, (int64_t)F, (int64_t)F, s_q8, s_sc, stream);
    launch_strict_gemv(L.wdown.dm, s_q8, s_sc, (int64_t)H, true, hidden, nullptr, stream);
  }
  if (logits_out) {
    launch_strict_rmsnorm(hidden, c.output_norm->as<float>(), (int64_t)H, eps, s_norm, stream);
    launch_act_quant(s_norm, 1, (int64_t)H, (int64_t)H, s_q8, s_sc, stream);
    if (dense_quant(c.lm_head.dm.quant))
      launch_strict_gemv_dense(c.lm_head.dm, s_norm, (int64_t)c.vocab_size, logits, stream);
    else if (kquant(c.lm_head.dm.quant))
      launch_kq_gemm(c.lm_head.dm, s_norm, s_q8, s_sc, 1, logits, stream);
    else
      launch_strict_gemv(c.lm_head.dm, s_q8, s_sc, (int64_t)c.vocab_size, false, logits, nullptr, stream);
  }
  if (argmax)
    launch_argmax(logits, (int64_t)c.vocab_size, am_val, am_idx, am_cnt, am_blocks, d_token, d_pos, d_hist, 0, stream);
}

void Context::run_decode_step() {
  if (cfg.numerics == JAL_NUMERICS_REFERENCE) {
    enqueue_strict_token(true, true);
    JAL_CUDA(cudaGetLastError());
    return;
  }
  if (mega) {
    if (launch_decode_mega(margs, mega_dev_args, mega_grid, stream)) {
      launches_per_step = 1;
      JAL_CUDA(cudaGetLastError());
      return;
    }
    cudaGetLastError();  // launch rejected: keep the graph path from now on
    mega = false;
  }
  if (cfg.use_graphs) {
    if (!graph) {
      bool pdl = !env_flag("JAL_NO_PDL");
      cudaGraph_t gr = nullptr;
      JAL_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
      if (exact) enqueue_exact_step(pdl);
      else enqueue_decode_step(pdl);
      cudaError_t e = cudaStreamEndCapture(stream, &gr);
      if (e != cudaSuccess) {
        cudaGetLastError();
        fail(JAL_ERR_CUDA, "decode graph capture failed: %s", cudaGetErrorString(e));
      }
      e = cudaGraphInstantiate(&graph, gr, 0);
      cudaGraphDestroy(gr);
      if (e != cudaSuccess) { graph = nullptr; fail(JAL_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e)); }
    }
    JAL_CUDA(cudaGraphLaunch(graph, stream));
  } else {
    if (exact) enqueue_exact_step(!env_flag("JAL_NO_PDL"));
    else enqueue_decode_step(!env_flag("JAL_NO_PDL"));
    JAL_CUDA(cudaGetLastError());
  }
}

void Context::ensure_prefill_capacity(uint64_t m) {
  if (m <= pf_cap) return;
  JAL_CUDA(cudaStreamSynchronize(stream));  // the old scratch may still be in use
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv;
  const uint64_t K = std::max<uint64_t>(std::max<uint64_t>(H, Q), F);
  size_t bytes = m * 4 + m * H * 4 + m * (Q + 2 * KV) * 4 + m * Q * 4 + m * 2 * F * 4 +
                 m * ((K + 31) / 32) * 4 + m * ((K + 31) / 32 * 32) + 7 * 256;
  pf_buf = alloc(bytes);
  pf_gen++;
  char *p = pf_buf->as<char>();
  auto take = [&](size_t n) { char *q = p; p += (n + 255) / 256 * 256; return q; };
  pf_tokens = (uint32_t *)take(m * 4);
  pf_hidden = (float *)take(m * H * 4);
  pf_qkv = (float *)take(m * (Q + 2 * KV) * 4);
  pf_attn = (float *)take(m * Q * 4);
  pf_gu = (float *)take(m * 2 * F * 4);
  pf_xs = (float *)take(m * ((K + 31) / 32) * 4);
  pf_xq = (int8_t *)take(m * ((K + 31) / 32 * 32));
  pf_cap = m;
}

// prefill_step_with_cache (recipe.rs:564-608, execute_batch_forward :1489-1756)
void Context::prefill(const uint32_t *tokens, uint64_t n, uint64_t start_pos, bool compute_logits) {
  if (cfg.numerics == JAL_NUMERICS_REFERENCE) {
    // The reference's batched forward is per-token identical math, so the
    // reference-order path runs the prompt one token at a time.
    for (uint64_t t = 0; t < n; t++) {
      launch_set_token_pos(d_token, tokens[t], d_pos, (int64_t)(start_pos + t), stream);
      enqueue_strict_token(compute_logits && t + 1 == n, false);
    }
    JAL_CUDA(cudaGetLastError());
    return;
  }
  const ModelCache &c = *cache;
  const uint64_t H = g.hidden_dim, F = g.ffn_dim, Q = g.total_q, KV = g.total_kv;
  const float eps = std::max(recipe.rms_eps, 1.0e-7f);
  const uint64_t end_pos = start_pos + n;
  const bool use_long = recipe.scaling.kind == JAL_ROPE_SCALING_LONGROPE &&
                        end_pos > recipe.scaling.original_max_position_embeddings;
  const uint64_t chunk = std::max<uint64_t>(1, cfg.prefill_chunk);
  ensure_prefill_capacity(std::min(n, chunk));
  for (uint64_t off = 0; off < n; off += chunk) {
    const uint64_t m = std::min(chunk, n - off), sp = start_pos + off;
    JAL_CUDA(cudaMemcpyAsync(pf_tokens, tokens + off, m * 4, cudaMemcpyHostToDevice, stream));
    launch_embed(c.emb_raw->as<uint8_t>(), c.emb_quant, (int64_t)H, (int64_t)c.emb_rows, pf_tokens, (int64_t)m,
                 pf_hidden, d_err, 0, stream);
    for (size_t l = 0; l < c.layers.size(); l++) {
      const Layer &L = c.layers[l];
      launch_rmsnorm_quant(pf_hidden, L.attn_norm, (int64_t)m, (int64_t)H, eps, pf_xq, pf_xs, stream);
      GemmArgs qa;
      qa.w = L.qkv; qa.m = (int64_t)m; qa.rows = (int64_t)(Q + 2 * KV); qa.xq = pf_xq; qa.xs = pf_xs;
      qa.y = pf_qkv; qa.y_stride = (int64_t)(Q + 2 * KV);
      launch_gemm(qa, stream);
      RopeAppendArgs ra;
      ra.qkv = pf_qkv; ra.m = (int64_t)m; ra.qkv_stride = (int64_t)(Q + 2 * KV); ra.start_pos = (int64_t)sp;
      ra.bq = L.bq; ra.bk = L.bk; ra.bv = L.bv;
      ra.cos_tab = use_long ? cos_long : cos_tab; ra.sin_tab = use_long ? sin_long : sin_tab;
      ra.skip_rope = recipe.should_skip_rope(l); ra.neox = recipe.rope_type == JAL_ROPE_NEOX;
      ra.n_heads_q = (int64_t)g.n_heads_q; ra.rotary_dim = (int64_t)g.rotary_dim; ra.kv = kv; ra.layer = (int64_t)l;
      launch_rope_append(ra, stream);
      AttnPrefillArgs pa;
      pa.qkv = pf_qkv; pa.m = (int64_t)m; pa.qkv_stride = (int64_t)(Q + 2 * KV); pa.start_pos = (int64_t)sp;
      pa.n_heads_q = (int64_t)g.n_heads_q; pa.kv = kv; pa.layer = (int64_t)l; pa.window = (int64_t)cfg.sliding_window;
      pa.scale = 1.0f / sqrtf((float)g.head_dim); pa.out = pf_attn;
      if (exact) launch_xattn_prefill(pa, stream);
      else launch_attn_prefill(pa, stream);
      launch_act_quant(pf_attn, (int64_t)m, (int64_t)Q, (int64_t)Q, pf_xq, pf_xs, stream);
      GemmArgs oa;
      oa.w = L.wo.dm; oa.m = (int64_t)m; oa.rows = (int64_t)H; oa.xq = pf_xq; oa.xs = pf_xs;
      oa.y = pf_hidden; oa.y_stride = (int64_t)H; oa.bias = L.bo; oa.accumulate = c.plan.rank == 0;
      launch_gemm(oa, stream);
      if (c.tp) tp_all_reduce(*c.tp, pf_hidden, m * H, stream);
      launch_rmsnorm_quant(pf_hidden, L.ffn_norm, (int64_t)m, (int64_t)H, eps, pf_xq, pf_xs, stream);
      GemmArgs ga;
      ga.w = L.gateup; ga.m = (int64_t)m; ga.rows = (int64_t)(2 * F); ga.xq = pf_xq; ga.xs = pf_xs;
      ga.y = pf_gu; ga.y_stride = (int64_t)(2 * F);
      launch_gemm(ga, stream);
      launch_swiglu_act_quant(pf_gu, (int64_t)m, (int64_t)F, (int64_t)(2 * F), pf_xq, pf_xs, stream);
      GemmArgs da;
      da.w = L.wdown.dm; da.m = (int64_t)m; da.rows = (int64_t)H; da.xq = pf_xq; da.xs = pf_xs;
      da.y = pf_hidden; da.y_stride = (int64_t)H; da.accumulate = c.plan.rank == 0;
      launch_gemm(da, stream);
      if (c.tp) tp_all_reduce(*c.tp, pf_hidden, m * H, stream);
    }
    JAL_CUDA(cudaGetLastError());
    if (compute_logits && off + m == n) {
      GemvArgs la;
      la.w = c.lm_head.dm; la.rows = (int64_t)c.plan.v_n; la.m = 1; la.in_mode = GEMV_IN_NORM;
      la.x = pf_hidden + (m - 1) * H; la.x_stride = (int64_t)H; la.norm_w = c.output_norm->as<float>(); la.eps = eps;
      la.out_mode = GEMV_OUT_STORE; la.y = logits_local; la.y_stride = (int64_t)c.plan.v_pad;
      if (exact && dense_quant(c.lm_head.dm.quant)) {
        launch_rmsnorm(la.x, la.norm_w, 1, (int64_t)H, eps, s_norm, stream);
        launch_strict_gemv_dense(c.lm_head.dm, s_norm, (int64_t)c.vocab_size, logits, stream);
      } else if (exact && kquant(c.lm_head.dm.quant)) {
        kq_lm_head(c, la.x, (int64_t)H, eps, s_norm, s_q8, s_sc, logits, stream);
      } else if (exact) {
        launch_xgemv(la, stream);
      } else {
        launch_gemv(la, stream);
      }
      if (c.tp) tp_all_gather(*c.tp, logits_local, logits, c.plan.v_pad, stream);
      JAL_CUDA(cudaGetLastError());
    }
  }
}

}  // namespace jal
