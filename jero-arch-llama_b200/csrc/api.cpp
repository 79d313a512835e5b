// The C ABI (include/jal.h): thin wrappers that validate arguments, convert
// exceptions into status codes and forward to the model / kernel layers.
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "common.hpp"
#include "device.hpp"
#include "gguf.hpp"
#include "jal.h"
#include "jal_test.h"
#include "model.hpp"

namespace jal {
static thread_local std::string g_last_error;
void set_last_error(const std::string &msg) { g_last_error = msg; }
}  // namespace jal

using namespace jal;

struct jal_cached_matrix {
  CachedMatrix m;
  bool borrowed = false;
};
struct jal_recipe {
  Recipe r;
};
struct jal_model_cache {
  std::unique_ptr<ModelCache> c;
  std::vector<std::unique_ptr<jal_cached_matrix>> views;
};
struct jal_context {
  std::unique_ptr<Context> ctx;
};
struct jal_tp {
  std::unique_ptr<TpComm> t;
};
struct jal_kv_cache {
  std::unique_ptr<KvCache> kv;
};

#define NEED(p)                                                  \
  do {                                                           \
    if (!(p)) fail(JAL_ERR_INVALID_ARGUMENT, "null argument: %s", #p); \
  } while (0)

static cudaStream_t as_stream(void *s) { return (cudaStream_t)s; }

extern "C" {

const char *jal_last_error(void) { return g_last_error.c_str(); }
const char *jal_version(void) { return "jal-b200 0.1.0 (sm_100a)"; }

int jal_set_device(int device) {
  return guard([&] { JAL_CUDA(cudaSetDevice(device)); });
}

int jal_device_sm_count(int *out) {
  return guard([&] {
    NEED(out);
    int dev = 0;
    JAL_CUDA(cudaGetDevice(&dev));
    JAL_CUDA(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev));
  });
}

// ---- CachedMatrix ---------------------------------------------------------

int jal_cached_matrix_repack(const void *raw, size_t raw_len, int raw_on_device, int quant, size_t rows, size_t cols,
                             void *stream, jal_cached_matrix **out) {
  return guard([&] {
    NEED(raw);
    NEED(out);
    *out = nullptr;
    size_t elems, bb;
    if (!ggml_block_geometry((uint32_t)quant, &elems, &bb) || quant == JAL_TQ1_0 || quant == JAL_TQ2_0 || quant == 3 ||
        quant == 7 || quant == 9 || quant == 10 || quant == 11)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported quant %d", quant);
    size_t rb = ggml_row_bytes((uint32_t)quant, cols);
    if (!rb) fail(JAL_ERR_TENSOR_BOUNDS, "cols %zu incompatible with quant %d", cols, quant);
    if (rows == 0 || raw_len < rows * rb)
      fail(JAL_ERR_TENSOR_BOUNDS, "rows=%zu cols=%zu buf len %zu < required %zu", rows, cols, raw_len, rows * rb);
    cudaStream_t s = as_stream(stream);
    const uint8_t *src = (const uint8_t *)raw;
    std::unique_ptr<DevBuffer> staging;
    if (!raw_on_device) {
      staging = std::make_unique<DevBuffer>(rows * rb);
      JAL_CUDA(cudaMemcpyAsync(staging->ptr, raw, rows * rb, cudaMemcpyHostToDevice, s));
      src = staging->as<uint8_t>();
    }
    auto h = std::make_unique<jal_cached_matrix>();
    h->m = repack_matrix(src, quant, rows, cols, s);
    JAL_CUDA(cudaStreamSynchronize(s));
    *out = h.release();
  });
}

void jal_cached_matrix_free(jal_cached_matrix *m) {
  if (m && !m->borrowed) delete m;
}
size_t jal_cached_matrix_rows(const jal_cached_matrix *m) { return m ? m->m.rows : 0; }
size_t jal_cached_matrix_cols(const jal_cached_matrix *m) { return m ? m->m.cols : 0; }
int jal_cached_matrix_quant(const jal_cached_matrix *m) { return m ? m->m.quant : -1; }
size_t jal_cached_matrix_aligned_bytes(const jal_cached_matrix *m) { return m ? m->m.aligned_bytes : 0; }

int jal_cached_matrix_export_ref_layout(const jal_cached_matrix *m, int8_t *tiles, size_t tiles_len, float *scales,
                                        size_t scales_len) {
  return guard([&] {
    NEED(m);
    NEED(tiles);
    NEED(scales);
    const DevMat &w = m->m.dm;
    if (kquant(w.quant)) {
      const size_t n_tiles = (size_t)(w.rows + 7) / 8, nt = n_tiles * (w.cols / 16) * 128,
                   ns = n_tiles * (w.cols / kquant_group(w.quant)) * 8;
      if (tiles_len < nt || scales_len < ns) fail(JAL_ERR_TENSOR_BOUNDS, "export buffers too small (%zu/%zu needed)", nt, ns);
      export_kquant_ref(w, tiles, scales, nullptr);
      return;
    }
    if (w.quant != JAL_Q4_0 && w.quant != JAL_Q8_0)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "export is defined for block-scaled Q4_0/Q8_0 and K-quant matrices");
    size_t n_tiles = (size_t)(w.rows + 7) / 8, nt = n_tiles * (w.cols / 16) * 128, ns = n_tiles * (w.cols / 32) * 8;
    if (tiles_len < nt || scales_len < ns) fail(JAL_ERR_TENSOR_BOUNDS, "export buffers too small (%zu/%zu needed)", nt, ns);
    DevBuffer dt(nt), ds(ns * 4);
    launch_export_ref(w, dt.as<int8_t>(), ds.as<float>(), 0);
    JAL_CUDA(cudaGetLastError());
    JAL_CUDA(cudaMemcpy(tiles, dt.ptr, nt, cudaMemcpyDeviceToHost));
    JAL_CUDA(cudaMemcpy(scales, ds.ptr, ns * 4, cudaMemcpyDeviceToHost));
  });
}

int jal_cached_matrix_export_ref_mins(const jal_cached_matrix *m, float *mins, size_t mins_len) {
  return guard([&] {
    NEED(m);
    NEED(mins);
    const DevMat &w = m->m.dm;
    if (w.quant != JAL_Q4_K && w.quant != JAL_Q5_K)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "group mins exist for Q4_K / Q5_K matrices only");
    const size_t ns = (size_t)(w.rows + 7) / 8 * (w.cols / 32) * 8;
    if (mins_len < ns) fail(JAL_ERR_TENSOR_BOUNDS, "mins buffer too small (%zu needed)", ns);
    export_kquant_ref(w, nullptr, nullptr, mins);
  });
}

static void check_block_scaled(const jal_cached_matrix *m) {
  if (m->m.dm.quant != JAL_Q4_0 && m->m.dm.quant != JAL_Q8_0)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "device GEMV/GEMM implemented for Q4_0/Q8_0 (quant %d)", m->m.quant);
}

int jal_cached_matrix_gemm(const jal_cached_matrix *mat, const float *x, size_t m, float *y, void *stream) {
  return guard([&] {
    NEED(mat);
    NEED(x);
    NEED(y);
    if (m == 0) return;
    const DevMat &w = mat->m.dm;
    if (kquant(w.quant)) {
      cudaStream_t s = as_stream(stream);
      const int64_t K = w.cols, nb = K / 32;
      DevBuffer q8((size_t)m * K), sc((size_t)m * nb * 4);
      launch_act_quant(x, (int64_t)m, K, K, q8.as<int8_t>(), sc.as<float>(), s);
      launch_kq_gemm(w, x, q8.as<int8_t>(), sc.as<float>(), (int64_t)m, y, s);
      JAL_CUDA(cudaGetLastError());
      JAL_CUDA(cudaStreamSynchronize(s));
      return;
    }
    check_block_scaled(mat);
    cudaStream_t s = as_stream(stream);
    int64_t K = w.cols, nb = K / 32;
    DevBuffer q8((size_t)m * K), sc((size_t)m * nb * 4);
    launch_act_quant(x, (int64_t)m, K, K, q8.as<int8_t>(), sc.as<float>(), s);
    xgemv_init();
    project_q8(w, q8.as<int8_t>(), sc.as<float>(), (int64_t)m, y, s);
    JAL_CUDA(cudaGetLastError());
    JAL_CUDA(cudaStreamSynchronize(s));
  });
}

int jal_cached_matrix_gemm_noalloc(const jal_cached_matrix *mat, const float *x, size_t m, float *y, void *stream) {
  return guard([&] {
    NEED(mat);
    NEED(x);
    NEED(y);
    if (m == 0) return;
    check_block_scaled(mat);
    gemm_noalloc(mat->m.dm, x, (int64_t)m, y, as_stream(stream));
  });
}

int jal_cached_matrix_gemv_q8(const jal_cached_matrix *mat, const int8_t *q8, const float *scales, float *y,
                              void *stream) {
  return guard([&] {
    NEED(mat);
    NEED(q8);
    NEED(scales);
    NEED(y);
    check_block_scaled(mat);
    xgemv_init();
    project_q8(mat->m.dm, q8, scales, 1, y, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_cached_matrix_dot16_partials(const jal_cached_matrix *mat, const int8_t *q8, size_t r0, size_t r1, int32_t *out,
                                     void *stream) {
  return guard([&] {
    NEED(mat);
    NEED(q8);
    NEED(out);
    check_block_scaled(mat);
    if (r0 > r1 || r1 > mat->m.rows) fail(JAL_ERR_TENSOR_BOUNDS, "row range [%zu, %zu) out of bounds", r0, r1);
    launch_dot16_partials(mat->m.dm, q8, (int64_t)r0, (int64_t)r1, out, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_act_quantize_q8(const float *x, size_t m, size_t k, int8_t *q8, float *scales, void *stream) {
  return guard([&] {
    NEED(x);
    NEED(q8);
    NEED(scales);
    if (m == 0 || k == 0) fail(JAL_ERR_TENSOR_BOUNDS, "QuantizedActQ8: m and k must be non-zero");
    launch_act_quant(x, (int64_t)m, (int64_t)k, (int64_t)k, q8, scales, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_quantize_row_q8_0(const float *x, size_t n, void *blocks, void *stream) {
  return guard([&] {
    NEED(x);
    NEED(blocks);
    if (n == 0 || n % 32) fail(JAL_ERR_TENSOR_BOUNDS, "quantize_row_q8_0: length %zu must be a positive multiple of 32", n);
    launch_quantize_row_q8_0(x, (int64_t)n, blocks, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_gemv_decode_projection(const void *raw, size_t raw_len, int quant, size_t rows, size_t cols, const float *x,
                               float *y, void *stream) {
  return guard([&] {
    NEED(raw);
    NEED(x);
    NEED(y);
    const bool q32 = quant == JAL_Q4_0 || quant == JAL_Q5_0 || quant == JAL_Q8_0;
    const bool dense = quant == JAL_F16 || quant == JAL_BF16 || quant == JAL_F32;
    if (!q32 && !dense && !superblock_quant(quant))
      fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported quantization %d for M=1 GEMV projection", quant);
    size_t rb = ggml_row_bytes((uint32_t)quant, cols);
    if (!rb) fail(JAL_ERR_TENSOR_BOUNDS, "cols %zu must be a multiple of the type's block", cols);
    if (raw_len < rows * rb) fail(JAL_ERR_TENSOR_BOUNDS, "truncated weight buffer");
    if (rows == 0) return;
    cudaStream_t s = as_stream(stream);
    if (dense) {
      launch_gemv_raw_dense((const uint8_t *)raw, quant, (int64_t)rows, (int64_t)cols, x, y, s);
    } else if (q32) {
      DevBuffer xb(cols / 32 * 36);
      launch_quantize_row_q8_0(x, (int64_t)cols, xb.ptr, s);
      launch_gemv_raw((const uint8_t *)raw, quant, (int64_t)rows, (int64_t)cols, xb.ptr, y, s);
      JAL_CUDA(cudaGetLastError());
      JAL_CUDA(cudaStreamSynchronize(s));  // before xb is freed
    } else {
      DevBuffer xb(cols / 256 * kQ8KBlockBytes);
      launch_quantize_row_q8_k(x, (int64_t)cols, xb.ptr, s);
      launch_gemv_raw_superblock((const uint8_t *)raw, quant, (int64_t)rows, (int64_t)cols, xb.ptr, y, s);
      JAL_CUDA(cudaGetLastError());
      JAL_CUDA(cudaStreamSynchronize(s));  // before xb is freed
    }
    JAL_CUDA(cudaGetLastError());
    JAL_CUDA(cudaStreamSynchronize(s));
  });
}

// ---- ops ------------------------------------------------------------------

int jal_op_rmsnorm(const float *x, const float *w, size_t m, size_t n, float eps, float *out, void *stream) {
  return guard([&] {
    NEED(x); NEED(w); NEED(out);
    if (n == 0) fail(JAL_ERR_TENSOR_BOUNDS, "rmsnorm slice mismatch");
    launch_rmsnorm(x, w, (int64_t)m, (int64_t)n, eps, out, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_op_rope(float *qk, size_t m, size_t row_len, size_t head_dim, size_t rotary_dim, int neox, size_t pos0,
                const float *inv_freq, void *stream) {
  return guard([&] {
    NEED(qk); NEED(inv_freq);
    if (head_dim < 2 || head_dim % 2 || rotary_dim < 2 || rotary_dim % 2 || rotary_dim > head_dim || row_len % head_dim)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid RoPE slice bounds");
    launch_rope_rows(qk, (int64_t)m, (int64_t)row_len, (int64_t)head_dim, (int64_t)rotary_dim, neox, (int64_t)pos0,
                     inv_freq, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_op_swiglu(const float *gate, const float *up, size_t n, float *out, void *stream) {
  return guard([&] {
    NEED(gate); NEED(up); NEED(out);
    launch_swiglu(gate, up, (int64_t)n, out, as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

int jal_op_gqa_attention(const float *q, const float *k, const float *v, size_t m, size_t n_heads_q, size_t n_heads_kv,
                         size_t head_dim, size_t total_seq, size_t start_pos, size_t sliding_window, float scale,
                         float *out, void *stream) {
  return guard([&] {
    NEED(q); NEED(k); NEED(v); NEED(out);
    if (m == 0 || n_heads_kv == 0 || n_heads_q == 0 || head_dim == 0 || total_seq == 0 || n_heads_q % n_heads_kv ||
        !std::isfinite(scale) || start_pos + m > total_seq)
      fail(JAL_ERR_CAPABILITY_MISMATCH, "invalid GQA prefill dimensions or mask config");
    if (total_seq * 4 > 200 * 1024) fail(JAL_ERR_CAPABILITY_MISMATCH, "op-level attention supports total_seq <= 51200");
    launch_gqa_attention_ref(q, k, v, (int64_t)m, (int64_t)n_heads_q, (int64_t)n_heads_kv, (int64_t)head_dim,
                             (int64_t)total_seq, (int64_t)start_pos, (int64_t)sliding_window, scale, out,
                             as_stream(stream));
    JAL_CUDA(cudaGetLastError());
  });
}

// ---- recipe ---------------------------------------------------------------

int jal_recipe_new(const char *architecture, jal_recipe **out) {
  return guard([&] {
    NEED(architecture);
    NEED(out);
    std::string a(architecture);
    if (a != "llama" && a != "llama4" && a != "qwen2")
      fail(JAL_ERR_CAPABILITY_MISMATCH, "LlamaRecipe supports 'llama', 'llama4', and 'qwen2', got '%s'", architecture);
    auto r = std::make_unique<jal_recipe>();
    r->r = Recipe::for_arch(a);
    *out = r.release();
  });
}

int jal_recipe_from_gguf(const void *gguf, size_t len, jal_recipe **out) {
  return guard([&] {
    NEED(gguf);
    NEED(out);
    GgufFile g((const uint8_t *)gguf, len);
    auto r = std::make_unique<jal_recipe>();
    r->r = Recipe::from_gguf(g);
    *out = r.release();
  });
}

void jal_recipe_free(jal_recipe *r) { delete r; }

int jal_recipe_get_fields(const jal_recipe *r, jal_recipe_fields *o) {
  return guard([&] {
    NEED(r);
    NEED(o);
    memset(o, 0, sizeof(*o));
    strncpy(o->architecture, r->r.architecture.c_str(), sizeof(o->architecture) - 1);
    o->num_layers = r->r.num_layers; o->hidden_dim = r->r.hidden_dim; o->ffn_dim = r->r.ffn_dim;
    o->n_heads_q = r->r.n_heads_q; o->n_heads_kv = r->r.n_heads_kv; o->head_dim = r->r.head_dim;
    o->vocab_size = r->r.vocab_size; o->rms_eps = r->r.rms_eps; o->rope_theta = r->r.rope_theta;
    o->rope_type = r->r.rope_type; o->rotary_dim = r->r.rotary_dim;
    o->rope_scaling_kind = r->r.scaling.kind; o->rope_factor = r->r.scaling.factor;
    o->rope_low_freq_factor = r->r.scaling.low_freq_factor; o->rope_high_freq_factor = r->r.scaling.high_freq_factor;
    o->rope_original_max_position_embeddings = r->r.scaling.original_max_position_embeddings;
  });
}

int jal_recipe_set_fields(jal_recipe *r, const jal_recipe_fields *in) {
  return guard([&] {
    NEED(r);
    NEED(in);
    std::string a(in->architecture, strnlen(in->architecture, sizeof(in->architecture)));
    if (a != "llama" && a != "llama4" && a != "qwen2") fail(JAL_ERR_CAPABILITY_MISMATCH, "unsupported architecture '%s'", a.c_str());
    Recipe &x = r->r;
    x.architecture = a;
    x.num_layers = in->num_layers; x.hidden_dim = in->hidden_dim; x.ffn_dim = in->ffn_dim;
    x.n_heads_q = in->n_heads_q; x.n_heads_kv = in->n_heads_kv; x.head_dim = in->head_dim; x.vocab_size = in->vocab_size;
    x.rms_eps = in->rms_eps; x.rope_theta = in->rope_theta; x.rope_type = in->rope_type; x.rotary_dim = in->rotary_dim;
    if (in->rope_scaling_kind != JAL_ROPE_SCALING_LONGROPE) {
      x.scaling.kind = in->rope_scaling_kind;
      x.scaling.factor = in->rope_factor;
      x.scaling.low_freq_factor = in->rope_low_freq_factor;
      x.scaling.high_freq_factor = in->rope_high_freq_factor;
      x.scaling.original_max_position_embeddings = in->rope_original_max_position_embeddings;
    }
  });
}

int jal_recipe_set_irope_mask(jal_recipe *r, const uint8_t *mask, size_t n) {
  return guard([&] {
    NEED(r);
    r->r.has_irope_mask = mask != nullptr;
    r->r.irope_mask.assign(mask, mask ? mask + n : mask);
  });
}

int jal_recipe_should_skip_rope(const jal_recipe *r, size_t layer) { return r && r->r.should_skip_rope(layer) ? 1 : 0; }

int jal_recipe_set_longrope(jal_recipe *r, const float *short_factor, const float *long_factor, size_t n,
                            uint64_t original_max_position_embeddings) {
  return guard([&] {
    NEED(r);
    NEED(short_factor);
    NEED(long_factor);
    r->r.scaling.kind = JAL_ROPE_SCALING_LONGROPE;
    r->r.scaling.short_factor.assign(short_factor, short_factor + n);
    r->r.scaling.long_factor.assign(long_factor, long_factor + n);
    r->r.scaling.original_max_position_embeddings = original_max_position_embeddings;
  });
}

int jal_recipe_supports_quant(const jal_recipe *r, int quant) { return r && r->r.supports_quant(quant) ? 1 : 0; }

int jal_recipe_validate_model(const jal_recipe *r, const void *gguf, size_t len) {
  return guard([&] {
    NEED(r);
    NEED(gguf);
    GgufFile g((const uint8_t *)gguf, len);
    r->r.validate_model(g);
  });
}

size_t jal_recipe_decode_scratch_bytes(const jal_recipe *r, size_t seq_len_upper_bound) {
  return r ? decode_scratch_bytes(r->r, seq_len_upper_bound) : 0;
}

// ---- model cache ----------------------------------------------------------

int jal_model_repack_cache_build(const jal_recipe *r, const void *gguf, size_t len, int device, jal_model_cache **out) {
  return guard([&] {
    NEED(r);
    NEED(gguf);
    NEED(out);
    *out = nullptr;
    GgufFile g((const uint8_t *)gguf, len);
    auto h = std::make_unique<jal_model_cache>();
    h->c = build_model_cache(r->r, g, device);
    *out = h.release();
  });
}

void jal_model_repack_cache_free(jal_model_cache *c) { delete c; }

int jal_tp_plan(size_t n_heads_q, size_t n_heads_kv, size_t ffn_dim, size_t vocab, int rank, int world,
                jal_tp_plan_t *out) {
  return guard([&] {
    NEED(out);
    const TpPlan p = tp_plan(n_heads_q, n_heads_kv, ffn_dim, vocab, rank, world);
    out->rank = (uint64_t)p.rank; out->world = (uint64_t)p.world;
    out->q_lo = p.q_lo; out->q_n = p.q_n; out->kv_lo = p.kv_lo; out->kv_n = p.kv_n;
    out->f_lo = p.f_lo; out->f_n = p.f_n; out->v_lo = p.v_lo; out->v_n = p.v_n; out->v_pad = p.v_pad;
  });
}

int jal_tp_unique_id(uint8_t *id_out) {
  return guard([&] {
    NEED(id_out);
    tp_unique_id(id_out);
  });
}

int jal_tp_init(const uint8_t *id, int rank, int world, jal_tp **out) {
  return guard([&] {
    NEED(id);
    NEED(out);
    *out = nullptr;
    auto h = std::make_unique<jal_tp>();
    h->t.reset(tp_init(id, rank, world));
    *out = h.release();
  });
}

void jal_tp_free(jal_tp *tp) { delete tp; }

int jal_model_repack_cache_build_tp(const jal_recipe *r, const void *gguf, size_t len, int device, const jal_tp *tp,
                                    jal_model_cache **out) {
  return guard([&] {
    NEED(r);
    NEED(gguf);
    NEED(tp);
    NEED(out);
    *out = nullptr;
    GgufFile g((const uint8_t *)gguf, len);
    auto h = std::make_unique<jal_model_cache>();
    h->c = build_model_cache(r->r, g, device, tp->t.get());
    *out = h.release();
  });
}

#define CACHE_GET(name, expr) \
  size_t name(const jal_model_cache *c) { return c ? (size_t)(expr) : 0; }
CACHE_GET(jal_model_cache_num_layers, c->c->geom.num_layers)
CACHE_GET(jal_model_cache_hidden_dim, c->c->geom.hidden_dim)
CACHE_GET(jal_model_cache_ffn_dim, c->c->geom.ffn_dim)
CACHE_GET(jal_model_cache_total_q, c->c->geom.total_q)
CACHE_GET(jal_model_cache_total_kv, c->c->geom.total_kv)
CACHE_GET(jal_model_cache_vocab_size, c->c->vocab_size)
CACHE_GET(jal_model_cache_norm_count, c->c->norm_count)
CACHE_GET(jal_model_cache_bias_count, c->c->bias_count)
CACHE_GET(jal_model_cache_repacked_matrix_count, c->c->layers.size() * 7 + 1)
CACHE_GET(jal_model_cache_total_aligned_bytes, c->c->total_aligned_bytes())

const jal_cached_matrix *jal_model_cache_matrix(const jal_model_cache *cc, size_t layer, int which) {
  if (!cc) return nullptr;
  jal_model_cache *c = const_cast<jal_model_cache *>(cc);
  const CachedMatrix *src = nullptr;
  if (layer == c->c->layers.size()) src = &c->c->lm_head;
  else if (layer < c->c->layers.size()) {
    const Layer &L = c->c->layers[layer];
    const CachedMatrix *all[] = {&L.wq, &L.wk, &L.wv, &L.wo, &L.wgate, &L.wup, &L.wdown};
    if (which >= 0 && which < 7) src = all[which];
  }
  if (!src) return nullptr;
  auto v = std::make_unique<jal_cached_matrix>();
  v->m = *src;
  v->m.storage.clear();
  v->borrowed = true;
  c->views.push_back(std::move(v));
  return c->views.back().get();
}

// ---- context --------------------------------------------------------------

static ContextConfig context_config(const jal_context_config *cfg) {
  ContextConfig cc;
  cc.n_ctx = cfg->n_ctx;
  if (cfg->kv_dtype != JAL_KV_F16 && cfg->kv_dtype != JAL_KV_F32)
    fail(JAL_ERR_INVALID_ARGUMENT, "unknown KV dtype %d", cfg->kv_dtype);
  cc.kv_f16 = cfg->kv_dtype == JAL_KV_F16;
  cc.page_size = cfg->page_size ? cfg->page_size : 64;
  cc.sliding_window = cfg->sliding_window;
  cc.use_graphs = cfg->use_graphs != 0;
  if (cfg->numerics != JAL_NUMERICS_FAST && cfg->numerics != JAL_NUMERICS_REFERENCE &&
      cfg->numerics != JAL_NUMERICS_RELAXED)
    fail(JAL_ERR_INVALID_ARGUMENT, "unknown numerics mode %d", cfg->numerics);
  cc.numerics = cfg->numerics;
  return cc;
}

int jal_context_new(const jal_recipe *r, const jal_model_cache *c, const jal_context_config *cfg, jal_context **out) {
  return guard([&] {
    NEED(r);
    NEED(c);
    NEED(cfg);
    NEED(out);
    *out = nullptr;
    auto h = std::make_unique<jal_context>();
    h->ctx = create_context(r->r, *c->c, context_config(cfg));
    *out = h.release();
  });
}

int jal_kv_cache_alloc(const jal_model_cache *c, uint64_t n_ctx, int32_t kv_dtype, uint32_t page_size,
                       jal_kv_cache **out) {
  return guard([&] {
    NEED(c);
    NEED(out);
    *out = nullptr;
    if (kv_dtype != JAL_KV_F16 && kv_dtype != JAL_KV_F32) fail(JAL_ERR_INVALID_ARGUMENT, "unknown KV dtype %d", kv_dtype);
    auto h = std::make_unique<jal_kv_cache>();
    h->kv = create_kv_cache(*c->c, n_ctx, kv_dtype == JAL_KV_F16, page_size);
    *out = h.release();
  });
}

void jal_kv_cache_free(jal_kv_cache *kv) { delete kv; }

size_t jal_kv_cache_bytes(const jal_kv_cache *kv) { return kv ? kv->kv->bytes() : 0; }

int jal_context_new_with_kv(const jal_recipe *r, const jal_model_cache *c, const jal_context_config *cfg,
                            jal_kv_cache *kv, jal_context **out) {
  return guard([&] {
    NEED(r);
    NEED(c);
    NEED(cfg);
    NEED(kv);
    NEED(out);
    *out = nullptr;
    auto h = std::make_unique<jal_context>();
    h->ctx = create_context(r->r, *c->c, context_config(cfg), kv->kv.get());
    *out = h.release();
  });
}

int jal_context_set_position(jal_context *ctx, size_t pos) {
  return guard([&] {
    NEED(ctx);
    if (pos > ctx->ctx->cfg.n_ctx)
      fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "position %zu exceeds n_ctx %llu", pos,
           (unsigned long long)ctx->ctx->cfg.n_ctx);
    ctx->ctx->position = pos;
  });
}

void jal_context_free(jal_context *ctx) { delete ctx; }

size_t jal_context_position(const jal_context *ctx) { return ctx ? ctx->ctx->position : 0; }

int jal_context_reset(jal_context *ctx) {
  return guard([&] {
    NEED(ctx);
    ctx->ctx->position = 0;
  });
}

// Reads the context's device error word after a synchronised step: bit 1 =
// an embedding lookup saw an out-of-range token, bit 2 = a bounded wait for
// a KV copy in decode attention gave up, bit 8 = a persistent-step grid
// barrier wait gave up, bit 16 = a tensor-parallel exchange wait gave up.
// The word is cleared afterwards.
static void enqueue_error_read(Context &c) {
  JAL_CUDA(cudaMemcpyAsync(&c.h_token[4], c.d_err, 4, cudaMemcpyDeviceToHost, c.stream));
}
static void check_device_error(Context &c) {
  const uint32_t e = c.h_token[4];
  if (!e) return;
  c.h_token[4] = 0;
  JAL_CUDA(cudaMemsetAsync(c.d_err, 0, 4, c.stream));
  if (c.mega) {  // a step that gave up a wait may leave its arrival counters behind
    JAL_CUDA(cudaMemsetAsync(c.margs.bar, 0, 8, c.stream));
    JAL_CUDA(cudaMemsetAsync(c.margs.head_cnt, 0, (size_t)c.margs.n_kv * 4, c.stream));
    JAL_CUDA(cudaMemsetAsync(c.margs.am_cnt, 0, 4, c.stream));
    JAL_CUDA(cudaMemsetAsync(c.margs.ffn_cnt, 0, (size_t)(c.margs.F / 32) * 4, c.stream));
    JAL_CUDA(cudaMemsetAsync(c.margs.hcnt, 0, (size_t)(c.margs.H / 32) * 4, c.stream));
  }
  JAL_CUDA(cudaStreamSynchronize(c.stream));
  if (e & 8u) fail(JAL_ERR_TIMEOUT, "persistent decode step: a bounded grid barrier wait gave up");
  if (e & 16u) fail(JAL_ERR_TIMEOUT, "tensor-parallel decode step: a bounded wait for the peers' partial sums gave up");
  if (e & 2u) fail(JAL_ERR_TIMEOUT, "decode step: a bounded wait for KV-tile or weight copies gave up");
  fail(JAL_ERR_TENSOR_BOUNDS, "embedding lookup saw an out-of-range token id");
}

static void check_tokens(const Context &c, const uint32_t *t, size_t n) {
  for (size_t i = 0; i < n; i++)
    if (t[i] >= c.cache->emb_rows)
      fail(JAL_ERR_TENSOR_BOUNDS, "token_id %u out of vocabulary bounds [0..%llu)", t[i], (unsigned long long)c.cache->emb_rows);
}

int jal_prefill_step(jal_context *h, const uint32_t *tokens, size_t n, size_t start_pos, int compute_logits,
                     float *logits, size_t logits_len) {
  return guard([&] {
    NEED(h);
    Context &c = *h->ctx;
    if (n == 0) { c.position = start_pos; return; }
    NEED(tokens);
    if (start_pos + n > c.cfg.n_ctx) fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "requested %zu > n_ctx %llu", start_pos + n, (unsigned long long)c.cfg.n_ctx);
    if (compute_logits && logits && logits_len != c.cache->vocab_size)
      fail(JAL_ERR_TENSOR_BOUNDS, "logits len %zu != vocab %llu", logits_len, (unsigned long long)c.cache->vocab_size);
    check_tokens(c, tokens, n);
    JAL_CUDA(cudaSetDevice(c.cache->device));
    c.prefill(tokens, n, start_pos, compute_logits != 0);
    if (compute_logits && logits)
      JAL_CUDA(cudaMemcpyAsync(logits, c.logits, logits_len * 4, cudaMemcpyDeviceToHost, c.stream));
    enqueue_error_read(c);
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    check_device_error(c);
    c.position = start_pos + n;
  });
}

int jal_decode_step(jal_context *h, uint32_t token, float *logits, size_t logits_len) {
  return guard([&] {
    NEED(h);
    Context &c = *h->ctx;
    if (c.position + 1 > c.cfg.n_ctx)
      fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "requested %llu > n_ctx %llu", (unsigned long long)c.position + 1,
           (unsigned long long)c.cfg.n_ctx);
    if (logits && logits_len != c.cache->vocab_size)
      fail(JAL_ERR_TENSOR_BOUNDS, "logits len %zu != vocab %llu", logits_len, (unsigned long long)c.cache->vocab_size);
    check_tokens(c, &token, 1);
    JAL_CUDA(cudaSetDevice(c.cache->device));
    *c.h_pos = (int64_t)c.position;
    c.h_token[0] = token;
    JAL_CUDA(cudaMemcpyAsync(c.d_pos, c.h_pos, 8, cudaMemcpyHostToDevice, c.stream));
    JAL_CUDA(cudaMemcpyAsync(c.d_token, c.h_token, 4, cudaMemcpyHostToDevice, c.stream));
    c.run_decode_step();
    if (logits) JAL_CUDA(cudaMemcpyAsync(logits, c.logits, logits_len * 4, cudaMemcpyDeviceToHost, c.stream));
    enqueue_error_read(c);
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    check_device_error(c);
    c.position += 1;
  });
}

int jal_decode_batch(jal_context *const *hs, size_t n, const uint32_t *tokens, float *logits, size_t logits_len) {
  return guard([&] {
    NEED(hs);
    NEED(tokens);
    if (n == 0) fail(JAL_ERR_INVALID_ARGUMENT, "batch of zero sequences");
    std::vector<Context *> cs(n);
    for (size_t i = 0; i < n; i++) {
      NEED(hs[i]);
      cs[i] = hs[i]->ctx.get();
    }
    Context &c0 = *cs[0];
    for (size_t i = 0; i < n; i++) {
      Context &c = *cs[i];
      if (c.cache != c0.cache) fail(JAL_ERR_INVALID_ARGUMENT, "batched decode: context %zu runs another model cache", i);
      if (!c.exact)
        fail(JAL_ERR_CAPABILITY_MISMATCH, "batched decode needs the reference-order numerics on one GPU (context %zu)", i);
      if (c.position + 1 > c.cfg.n_ctx)
        fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "context %zu: requested %llu > n_ctx %llu", i,
             (unsigned long long)c.position + 1, (unsigned long long)c.cfg.n_ctx);
      for (size_t j = 0; j < i; j++)
        if (cs[j] == cs[i] || cs[j]->kv.k == c.kv.k)
          fail(JAL_ERR_INVALID_ARGUMENT, "batched decode: contexts %zu and %zu share a KV cache", j, i);
      check_tokens(c, &tokens[i], 1);
    }
    const size_t V = c0.cache->vocab_size;
    if (logits && logits_len != n * V)
      fail(JAL_ERR_TENSOR_BOUNDS, "logits len %zu != %zu x vocab %zu", logits_len, n, V);
    JAL_CUDA(cudaSetDevice(c0.cache->device));
    for (size_t i = 1; i < n; i++) JAL_CUDA(cudaStreamSynchronize(cs[i]->stream));  // their own work first
    c0.ensure_prefill_capacity(n);
    for (size_t i = 0; i < n; i++) {
      *cs[i]->h_pos = (int64_t)cs[i]->position;
      JAL_CUDA(cudaMemcpyAsync(cs[i]->d_pos, cs[i]->h_pos, 8, cudaMemcpyHostToDevice, c0.stream));
    }
    JAL_CUDA(cudaMemcpyAsync(c0.pf_tokens, tokens, n * 4, cudaMemcpyHostToDevice, c0.stream));
    run_batch_decode(cs.data(), n);
    if (logits) JAL_CUDA(cudaMemcpyAsync(logits, c0.bt_logits, n * V * 4, cudaMemcpyDeviceToHost, c0.stream));
    enqueue_error_read(c0);
    JAL_CUDA(cudaStreamSynchronize(c0.stream));
    check_device_error(c0);
    for (size_t i = 0; i < n; i++) cs[i]->position += 1;
  });
}

int jal_context_batch_logits_device(const jal_context *h, const float **out) {
  return guard([&] {
    NEED(h);
    NEED(out);
    *out = h->ctx->bt_logits;
  });
}

int jal_decode_greedy(jal_context *h, uint32_t token, size_t n_steps, uint32_t *tokens_out) {
  return guard([&] {
    NEED(h);
    NEED(tokens_out);
    Context &c = *h->ctx;
    if (c.position + n_steps > c.cfg.n_ctx)
      fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "requested %llu > n_ctx %llu", (unsigned long long)(c.position + n_steps),
           (unsigned long long)c.cfg.n_ctx);
    check_tokens(c, &token, 1);
    if (n_steps == 0) return;
    JAL_CUDA(cudaSetDevice(c.cache->device));
    *c.h_pos = (int64_t)c.position;
    c.h_token[0] = token;
    JAL_CUDA(cudaMemcpyAsync(c.d_pos, c.h_pos, 8, cudaMemcpyHostToDevice, c.stream));
    JAL_CUDA(cudaMemcpyAsync(c.d_token, c.h_token, 4, cudaMemcpyHostToDevice, c.stream));
    for (size_t i = 0; i < n_steps; i++) c.run_decode_step();
    JAL_CUDA(cudaMemcpyAsync(tokens_out, c.d_hist + c.position + 1, n_steps * 4, cudaMemcpyDeviceToHost, c.stream));
    enqueue_error_read(c);
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    check_device_error(c);
    c.position += n_steps;
  });
}

int jal_context_export_kv(const jal_context *h, size_t n_pos, float *out, size_t len) {
  return guard([&] {
    NEED(h);
    NEED(out);
    const Context &c = *h->ctx;
    const KvView &kv = c.kv;
    const size_t kvd = (size_t)kv.n_kv * kv.head_dim, L = (size_t)kv.n_layers;
    if (n_pos > c.cfg.n_ctx) fail(JAL_ERR_TENSOR_BOUNDS, "n_pos beyond n_ctx");
    if (len < L * 2 * n_pos * kvd) fail(JAL_ERR_TENSOR_BOUNDS, "export buffer too small");
    size_t esz = kv.f16 ? 2 : 4, elems = L * kv.n_pages * kv.n_kv * kv.page_size * kv.head_dim;
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    std::vector<uint8_t> hk(elems * esz), hv(elems * esz);
    JAL_CUDA(cudaMemcpy(hk.data(), kv.k, hk.size(), cudaMemcpyDeviceToHost));
    JAL_CUDA(cudaMemcpy(hv.data(), kv.v, hv.size(), cudaMemcpyDeviceToHost));
    auto get = [&](const std::vector<uint8_t> &b, size_t e) -> float {
      if (!kv.f16) { float f; memcpy(&f, b.data() + e * 4, 4); return f; }
      uint16_t x;
      memcpy(&x, b.data() + e * 2, 2);
      uint32_t sign = (uint32_t)(x & 0x8000u) << 16, ex = (x >> 10) & 0x1F, m = x & 0x3FF, bits;
      if (ex == 0) {
        if (m == 0) bits = sign;
        else { int k = -1; do { m <<= 1; k++; } while (!(m & 0x400)); bits = sign | ((uint32_t)(112 - k) << 23) | ((m & 0x3FF) << 13); }
      } else if (ex == 31) bits = sign | 0x7F800000u | (m << 13);
      else bits = sign | ((ex + 112u) << 23) | (m << 13);
      float f;
      memcpy(&f, &bits, 4);
      return f;
    };
    for (size_t l = 0; l < L; l++)
      for (size_t p = 0; p < n_pos; p++)
        for (size_t hh = 0; hh < (size_t)kv.n_kv; hh++)
          for (size_t d = 0; d < (size_t)kv.head_dim; d++) {
            size_t page = p / kv.page_size, slot = p % kv.page_size;  // identity page table
            size_t e = (((l * kv.n_pages + page) * kv.n_kv + hh) * kv.page_size + slot) * kv.head_dim + d;
            out[((l * 2 + 0) * n_pos + p) * kvd + hh * kv.head_dim + d] = get(hk, e);
            out[((l * 2 + 1) * n_pos + p) * kvd + hh * kv.head_dim + d] = get(hv, e);
          }
  });
}

int jal_context_logits_device(const jal_context *h, const float **out) {
  return guard([&] {
    NEED(h);
    NEED(out);
    *out = h->ctx->logits;
  });
}

int jal_context_set_stream(jal_context *h, void *stream) {
  return guard([&] {
    NEED(h);
    Context &c = *h->ctx;
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    c.stream = stream ? (cudaStream_t)stream : c.own_stream;
  });
}

int jal_context_last_step_launches(const jal_context *h, size_t *out) {
  return guard([&] {
    NEED(h);
    NEED(out);
    *out = h->ctx->launches_per_step;
  });
}

int jal_context_tp_exchange(const jal_context *h, int *out) {
  return guard([&] {
    NEED(h);
    NEED(out);
    const Context &c = *h->ctx;
    *out = c.cache->plan.world <= 1 ? JAL_TP_EXCHANGE_NONE : c.tp_sym ? JAL_TP_EXCHANGE_PEER : JAL_TP_EXCHANGE_NCCL;
  });
}

}  // extern "C"

// ---- test hooks (jal_test.h) ------------------------------------------------

int jal_context_test_stall_kv_copy(jal_context *h, uint32_t extra_bytes, uint64_t wait_ns) {
  return guard([&] {
    NEED(h);
    Context &c = *h->ctx;
    if (!c.exact) fail(JAL_ERR_CAPABILITY_MISMATCH, "the stall hook drives the FAST single-GPU decode attention");
    c.test_stall_tx = extra_bytes;
    c.test_wait_ns = wait_ns;
    if (c.graph) {  // the captured step holds the old arguments
      JAL_CUDA(cudaStreamSynchronize(c.stream));
      cudaGraphExecDestroy(c.graph);
      c.graph = nullptr;
    }
  });
}

int jal_context_trace_decode_step(jal_context *h, uint32_t token, uint64_t *out, size_t out_len, size_t *n_launches) {
  return guard([&] {
    NEED(h);
    NEED(out);
    NEED(n_launches);
    Context &c = *h->ctx;
    if (!c.exact) fail(JAL_ERR_CAPABILITY_MISMATCH, "the step trace covers the FAST single-GPU decode step");
    if (c.position + 1 > c.cfg.n_ctx)
      fail(JAL_ERR_CONTEXT_LENGTH_EXCEEDED, "requested %llu > n_ctx %llu", (unsigned long long)c.position + 1,
           (unsigned long long)c.cfg.n_ctx);
    check_tokens(c, &token, 1);
    JAL_CUDA(cudaSetDevice(c.cache->device));
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    const size_t slots = kTraceSlots * (4 + 6 * c.cache->layers.size());
    if (!c.trace_buf) {
      c.trace_buf = std::make_shared<DevBuffer>(slots * 8);
      c.d_trace = c.trace_buf->as<unsigned long long>();
    }
    std::vector<uint64_t> init(slots, 0);
    for (size_t i = 0; i < slots; i += kTraceSlots) init[i] = ~0ull;
    JAL_CUDA(cudaMemcpy(c.d_trace, init.data(), slots * 8, cudaMemcpyHostToDevice));
    auto drop_graph = [&] {
      if (c.graph) {
        JAL_CUDA(cudaStreamSynchronize(c.stream));
        cudaGraphExecDestroy(c.graph);
        c.graph = nullptr;
      }
    };
    drop_graph();  // recaptured with the trace slots
    c.trace_on = true;
    *c.h_pos = (int64_t)c.position;
    c.h_token[0] = token;
    JAL_CUDA(cudaMemcpyAsync(c.d_pos, c.h_pos, 8, cudaMemcpyHostToDevice, c.stream));
    JAL_CUDA(cudaMemcpyAsync(c.d_token, c.h_token, 4, cudaMemcpyHostToDevice, c.stream));
    try {
      c.run_decode_step();  // capture and the first replay (which pays the graph upload)
      JAL_CUDA(cudaStreamSynchronize(c.stream));
      JAL_CUDA(cudaMemcpy(c.d_trace, init.data(), slots * 8, cudaMemcpyHostToDevice));
      c.run_decode_step();  // the traced step
      JAL_CUDA(cudaStreamSynchronize(c.stream));
    } catch (...) {
      c.trace_on = false;
      drop_graph();
      throw;
    }
    c.trace_on = false;
    drop_graph();
    const size_t n = std::min(c.launches_per_step, out_len / kTraceSlots);
    *n_launches = c.launches_per_step;
    JAL_CUDA(cudaMemcpy(out, c.d_trace, n * kTraceSlots * 8, cudaMemcpyDeviceToHost));
    enqueue_error_read(c);
    JAL_CUDA(cudaStreamSynchronize(c.stream));
    check_device_error(c);
    c.position += 2;
  });
}

int jal_test_peer_exchange_timeout(const jal_cached_matrix *mat, uint64_t wait_ns, double *elapsed_ms) {
  return guard([&] {
    NEED(mat);
    check_block_scaled(mat);
    const DevMat &w = mat->m.dm;
    const int64_t K = w.cols;
    DevBuffer x((size_t)K * 4), nw((size_t)K * 4), slot((size_t)K * 8), y((size_t)w.rows * 4), words(64);
    std::vector<float> one((size_t)K, 1.0f);
    JAL_CUDA(cudaMemcpy(x.ptr, one.data(), (size_t)K * 4, cudaMemcpyHostToDevice));
    JAL_CUDA(cudaMemcpy(nw.ptr, one.data(), (size_t)K * 4, cudaMemcpyHostToDevice));
    JAL_CUDA(cudaMemset(slot.ptr, 0, slot.bytes));  // flag 0: never this step's (epoch 0, phase 0 -> flag 1)
    JAL_CUDA(cudaMemset(words.ptr, 0, words.bytes));
    GemvArgs a;
    a.w = w; a.rows = w.rows; a.m = 1; a.in_mode = GEMV_IN_NORM; a.x = x.as<float>(); a.x_stride = K;
    a.norm_w = nw.as<float>(); a.eps = 1e-5f; a.out_mode = GEMV_OUT_STORE; a.y = y.as<float>(); a.y_stride = w.rows;
    a.peer_in = slot.as<unsigned long long>(); a.peer_world = 1; a.peer_phase = 0;
    a.peer_epoch = (const uint32_t *)words.as<char>(); a.err = (int *)(words.as<char>() + 16);
    a.peer_wait_ns = wait_ns;
    if (!gemv_peer_supported(a)) fail(JAL_ERR_CAPABILITY_MISMATCH, "matrix shape not on the exchange GEMV");
    gemv_init();
    JAL_CUDA(cudaDeviceSynchronize());
    const auto t0 = std::chrono::steady_clock::now();
    launch_gemv(a, nullptr);
    JAL_CUDA(cudaGetLastError());
    JAL_CUDA(cudaDeviceSynchronize());
    const auto t1 = std::chrono::steady_clock::now();
    if (elapsed_ms) *elapsed_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    int err = 0;
    JAL_CUDA(cudaMemcpy(&err, words.as<char>() + 16, 4, cudaMemcpyDeviceToHost));
    if (err & kErrPeerWait) fail(JAL_ERR_TIMEOUT, "tensor-parallel exchange wait gave up (as arranged)");
  });
}
