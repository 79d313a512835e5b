// Seeded synthetic GGUF models: SplitMix64 counters -> Box-Muller normals ->
// GGML reference quantizers (Q4_0: d = max/-8, q = min(15, (i8)(x/d + 8.5));
// Q8_0: d = amax/127, q = round(x/d)), written as GGUF v3.
#include <cmath>
#include <cstring>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "common.hpp"
#include "gguf.hpp"
#include "jal_synth.h"

namespace jal {
namespace {

inline uint64_t sm64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint64_t fnv1a(const char *s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (; *s; s++) h = (h ^ (uint8_t)*s) * 0x100000001b3ull;
  return h;
}

uint64_t tensor_key(uint64_t seed, const char *name) { return sm64(seed ^ sm64(fnv1a(name))); }

// Normal pair j of the stream `key`.
inline void normal_pair(uint64_t key, uint64_t j, double *n0, double *n1) {
  uint64_t z1 = sm64(key + 2 * j), z2 = sm64(key + 2 * j + 1);
  double u1 = (double)((z1 >> 11) + 1) * (1.0 / 9007199254740992.0);  // (0, 1]
  double u2 = (double)(z2 >> 11) * (1.0 / 9007199254740992.0);        // [0, 1)
  double r = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586476925 * u2;
  *n0 = r * std::cos(th);
  *n1 = r * std::sin(th);
}

// Element i (even count chunks of 32 keep pairs inside one block).
inline void gen_block(uint64_t key, uint64_t first, size_t n, float std_dev, float *out) {
  for (size_t k = 0; k < n; k += 2) {
    double a, b;
    normal_pair(key, (first + k) / 2, &a, &b);
    out[k] = (float)(std_dev * a);
    if (k + 1 < n) out[k + 1] = (float)(std_dev * b);
  }
}

uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  x &= 0x7FFFFFFFu;
  if (x >= 0x7F800000u) return (uint16_t)(sign | (x > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (x >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (x < 0x38800000u) {
    if (x < 0x33000000u) return (uint16_t)sign;
    uint32_t mant = (x & 0x7FFFFFu) | 0x800000u;
    int e = (int)(x >> 23);
    int shift = 126 - e;
    uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = (x >> 13) - (112u << 10), rem = x & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1F, mant = h & 0x3FF, bits;
  if (exp == 0) {
    if (mant == 0) bits = sign;
    else {
      int e = -1;
      do { mant <<= 1; e++; } while (!(mant & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3FF) << 13);
    }
  } else if (exp == 31) bits = sign | 0x7F800000u | (mant << 13);
  else bits = sign | ((exp + 112u) << 23) | (mant << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

void quantize_q4_0_block(const float *x, uint8_t *out) {
  float amax = 0.f, max = 0.f;
  for (int j = 0; j < 32; j++) {
    float v = x[j];
    if (amax < std::fabs(v)) { amax = std::fabs(v); max = v; }
  }
  float d = max / -8.0f, id = d != 0.f ? 1.0f / d : 0.0f;
  uint16_t dh = f32_to_f16_rne(d);
  memcpy(out, &dh, 2);
  for (int j = 0; j < 16; j++) {
    float x0 = x[j] * id, x1 = x[16 + j] * id;
    int xi0 = (int8_t)(x0 + 8.5f), xi1 = (int8_t)(x1 + 8.5f);
    if (xi0 > 15) xi0 = 15;
    if (xi1 > 15) xi1 = 15;
    out[2 + j] = (uint8_t)(xi0 | (xi1 << 4));
  }
}

// GGML's Q5_0 reference quantizer: d = max / -16, q = min(31, (i8)(x/d + 16.5)),
// low nibbles in qs, bit 4 of element j in bit j of qh.
void quantize_q5_0_block(const float *x, uint8_t *out) {
  float amax = 0.f, max = 0.f;
  for (int j = 0; j < 32; j++) {
    float v = x[j];
    if (amax < std::fabs(v)) { amax = std::fabs(v); max = v; }
  }
  float d = max / -16.0f, id = d != 0.f ? 1.0f / d : 0.0f;
  uint16_t dh = f32_to_f16_rne(d);
  memcpy(out, &dh, 2);
  uint32_t qh = 0;
  for (int j = 0; j < 16; j++) {
    float x0 = x[j] * id, x1 = x[16 + j] * id;
    int xi0 = (int8_t)(x0 + 16.5f), xi1 = (int8_t)(x1 + 16.5f);
    if (xi0 > 31) xi0 = 31;
    if (xi1 > 31) xi1 = 31;
    out[6 + j] = (uint8_t)((xi0 & 0x0F) | ((xi1 & 0x0F) << 4));
    qh |= (uint32_t)((xi0 & 0x10) >> 4) << j;
    qh |= (uint32_t)((xi1 & 0x10) >> 4) << (j + 16);
  }
  memcpy(out + 2, &qh, 4);
}

void quantize_q8_0_block(const float *x, uint8_t *out) {
  float amax = 0.f;
  for (int j = 0; j < 32; j++) amax = std::fmax(amax, std::fabs(x[j]));
  float d = amax / 127.0f, id = d != 0.f ? 1.0f / d : 0.0f;
  uint16_t dh = f32_to_f16_rne(d);
  memcpy(out, &dh, 2);
  for (int j = 0; j < 32; j++) out[2 + j] = (uint8_t)(int8_t)std::roundf(x[j] * id);
}

// Writes `rows x cols` values of stream `key` in GGUF block order.
void write_matrix(int quant, size_t rows, size_t cols, uint64_t key, float std_dev, uint8_t *out, int nthreads) {
  size_t rb = ggml_row_bytes((uint32_t)quant, cols);
  if (!rb) fail(JAL_ERR_TENSOR_BOUNDS, "synth: cols %zu incompatible with quant %d", cols, quant);
  if (quant != JAL_Q4_0 && quant != JAL_Q5_0 && quant != JAL_Q8_0 && quant != JAL_F32 && quant != JAL_F16)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "synth: unsupported quant %d", quant);
  if (cols % 2) fail(JAL_ERR_TENSOR_BOUNDS, "synth: odd cols");
  (void)nthreads;
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads > 0 ? nthreads : 1)
  for (size_t r = 0; r < rows; r++) {
    float buf[32];
    uint8_t *row = out + r * rb;
    uint64_t base = (uint64_t)r * cols;
    if (quant == JAL_F32 || quant == JAL_F16) {
      for (size_t c = 0; c < cols; c += 32) {
        size_t n = cols - c < 32 ? cols - c : 32;
        gen_block(key, base + c, n, std_dev, buf);
        for (size_t k = 0; k < n; k++) {
          if (quant == JAL_F32) memcpy(row + (c + k) * 4, &buf[k], 4);
          else { uint16_t h = f32_to_f16_rne(buf[k]); memcpy(row + (c + k) * 2, &h, 2); }
        }
      }
      continue;
    }
    size_t bb = quant == JAL_Q4_0 ? 18 : quant == JAL_Q5_0 ? 22 : 34;
    for (size_t b = 0; b < cols / 32; b++) {
      gen_block(key, base + b * 32, 32, std_dev, buf);
      if (quant == JAL_Q4_0) quantize_q4_0_block(buf, row + b * bb);
      else if (quant == JAL_Q5_0) quantize_q5_0_block(buf, row + b * bb);
      else quantize_q8_0_block(buf, row + b * bb);
    }
  }
}

struct Plan {
  GgufWriter w;
  std::vector<float> stds;    // per tensor; NAN = constant 1.0 (norm)
};

Plan make_plan(const jal_synth_config *c) {
  Plan p;
  std::string arch(c->architecture);
  if (arch.empty()) arch = "llama";
  uint64_t H = c->hidden_dim, F = c->ffn_dim, Q = c->n_heads_q * c->head_dim, KV = c->n_heads_kv * c->head_dim;
  GgufWriter &w = p.w;
  w.add_string("general.architecture", arch);
  w.add_u32("general.alignment", 32);
  w.add_u32(arch + ".block_count", (uint32_t)c->num_layers);
  w.add_u32(arch + ".embedding_length", (uint32_t)H);
  w.add_u32(arch + ".feed_forward_length", (uint32_t)F);
  w.add_u32(arch + ".attention.head_count", (uint32_t)c->n_heads_q);
  w.add_u32(arch + ".attention.head_count_kv", (uint32_t)c->n_heads_kv);
  w.add_u32(arch + ".attention.key_length", (uint32_t)c->head_dim);
  w.add_u32(arch + ".attention.value_length", (uint32_t)c->head_dim);
  w.add_f32(arch + ".rope.freq_base", c->rope_theta);
  w.add_f32(arch + ".attention.layer_norm_rms_epsilon", c->rms_eps);
  w.add_u32(arch + ".context_length", (uint32_t)c->context_length);
  w.add_u32(arch + ".vocab_size", (uint32_t)c->vocab_size);
  auto add = [&](const std::string &n, int q, std::vector<uint64_t> d, float sd) {
    w.add_tensor(n, (uint32_t)q, std::move(d));
    p.stds.push_back(sd);
  };
  float ws = c->weight_std, bs = c->bias_std;
  add("token_embd.weight", c->embed_quant, {H, c->vocab_size}, ws);
  for (uint64_t l = 0; l < c->num_layers; l++) {
    std::string b = "blk." + std::to_string(l) + ".";
    add(b + "attn_norm.weight", JAL_F32, {H}, NAN);
    add(b + "attn_q.weight", c->weight_quant, {H, Q}, ws);
    add(b + "attn_k.weight", c->weight_quant, {H, KV}, ws);
    add(b + "attn_v.weight", c->weight_quant, {H, KV}, ws);
    if (c->qkv_bias) {
      add(b + "attn_q.bias", JAL_F32, {Q}, bs);
      add(b + "attn_k.bias", JAL_F32, {KV}, bs);
      add(b + "attn_v.bias", JAL_F32, {KV}, bs);
    }
    add(b + "attn_output.weight", c->weight_quant, {Q, H}, ws);
    add(b + "ffn_norm.weight", JAL_F32, {H}, NAN);
    add(b + "ffn_gate.weight", c->weight_quant, {H, F}, ws);
    add(b + "ffn_up.weight", c->weight_quant, {H, F}, ws);
    add(b + "ffn_down.weight", c->weight_quant, {F, H}, ws);
  }
  add("output_norm.weight", JAL_F32, {H}, NAN);
  if (c->head_quant >= 0) add("output.weight", c->head_quant, {H, c->vocab_size}, ws);
  return p;
}

}  // namespace

void set_last_error(const std::string &msg);

}  // namespace jal

using namespace jal;

extern "C" uint16_t jal_f32_to_f16_bits(float v) { return f32_to_f16_rne(v); }

extern "C" int jal_synth_gguf_size(const jal_synth_config *cfg, size_t *bytes) {
  return guard([&] {
    if (!cfg || !bytes) fail(JAL_ERR_INVALID_ARGUMENT, "null argument");
    *bytes = make_plan(cfg).w.total_size();
  });
}

extern "C" int jal_synth_gguf_write(const jal_synth_config *cfg, uint64_t seed, void *buf, size_t len, int nthreads) {
  return guard([&] {
    if (!cfg || !buf) fail(JAL_ERR_INVALID_ARGUMENT, "null argument");
    Plan p = make_plan(cfg);
    size_t total = p.w.total_size();
    if (len < total) fail(JAL_ERR_TENSOR_BOUNDS, "buffer %zu < GGUF size %zu", len, total);
    uint8_t *out = (uint8_t *)buf;
    p.w.write_header(out, len);
    size_t prev_end = 0;
    for (size_t i = 0; i < p.w.n_tensors(); i++) {
      size_t off = p.w.tensor_file_offset(i), nb = p.w.tensor_bytes(i);
      if (i > 0 && off > prev_end) memset(out + prev_end, 0, off - prev_end);
      const std::string &name = p.w.tensor_name(i);
      const std::vector<uint64_t> &d = p.w.tensor_dims(i);
      int q = (int)p.w.tensor_type(i);
      float sd = p.stds[i];
      if (std::isnan(sd)) {
        // Norm weight vector of ones.
        float one = 1.0f;
        for (size_t k = 0; k < d[0]; k++) memcpy(out + off + k * 4, &one, 4);
      } else {
        size_t rows = d.size() > 1 ? d[1] : 1;
        write_matrix(q, rows, d[0], tensor_key(seed, name.c_str()), sd, out + off, nthreads);
      }
      prev_end = off + nb;
    }
  });
}

extern "C" int jal_synth_matrix(int quant, size_t rows, size_t cols, uint64_t seed, const char *name, float std_dev,
                                void *out, size_t len, int nthreads) {
  return guard([&] {
    if (!out || !name) fail(JAL_ERR_INVALID_ARGUMENT, "null argument");
    size_t rb = ggml_row_bytes((uint32_t)quant, cols);
    if (!rb) fail(JAL_ERR_TENSOR_BOUNDS, "cols %zu incompatible with quant %d", cols, quant);
    if (len < rows * rb) fail(JAL_ERR_TENSOR_BOUNDS, "buffer %zu < %zu", len, rows * rb);
    write_matrix(quant, rows, cols, tensor_key(seed, name), std_dev, (uint8_t *)out, nthreads);
  });
}

extern "C" int jal_synth_normal_f32(uint64_t seed, const char *name, size_t n, float std_dev, float *out, int nthreads) {
  return guard([&] {
    if (!out || !name) fail(JAL_ERR_INVALID_ARGUMENT, "null argument");
    uint64_t key = tensor_key(seed, name);
    (void)nthreads;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
    for (size_t b = 0; b < (n + 31) / 32; b++) {
      size_t c = b * 32, m = n - c < 32 ? n - c : 32;
      gen_block(key, c, m, std_dev, out + c);
    }
  });
}
