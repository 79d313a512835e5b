/*
 * CPU oracle for the quantized decode/prefill hot path of jero-arch-llama.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker and the timed
 * CPU baseline.  It is a restatement, in plain C, of the reference crate's
 * portable (`--no-default-features`) Rust path; every function cites the
 * reference file:line it follows.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it.  Nothing in the product library
 * links or calls it.
 *
 * Float semantics follow the Rust code: f32 arithmetic in source order, no
 * contraction into FMA (built with -ffp-contract=off), `round` = roundf (half
 * away from zero), `powf`/`sinf`/`cosf`/`expf` from libm, and `Iterator::sum`
 * over f32 folding from -0.0.
 */
#ifndef JAL_ORACLE_H
#define JAL_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids (the on-disk GGUF tensor type field). */
enum or_quant {
  OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7,
  OR_Q8_0 = 8, OR_Q8_1 = 9, OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12,
  OR_Q5_K = 13, OR_Q6_K = 14, OR_BF16 = 30, OR_TQ1_0 = 34, OR_TQ2_0 = 35
};

/* Status codes mirror jero_core::K3Error variants. */
enum or_status {
  OR_OK = 0,
  OR_ERR_TENSOR_BOUNDS = 1,
  OR_ERR_CAPABILITY_MISMATCH = 2,
  OR_ERR_CONTEXT_LENGTH_EXCEEDED = 3
};

/* ---- converters and dequantizers ------------------------------------- */
float or_f16_to_f32_finite(uint16_t bits);
float or_bf16_to_f32_finite(uint16_t bits);
float or_sanitize_f32_weight(float v);
int or_quant_block_geometry(int quant, size_t *elems, size_t *bytes);
int or_quant_row_bytes(size_t cols, int quant, size_t *row_bytes);
int or_is_oversized_dense(int quant, size_t rows, size_t cols);
void or_dequantize_q4_0_block(const uint8_t *blk, float *out);
void or_dequantize_q5_0_block(const uint8_t *blk, float *out);
void or_dequantize_q8_0_block(const uint8_t *blk, float *out);
void or_dequantize_q4_k_block(const uint8_t *blk, float *out);
void or_dequantize_q5_k_block(const uint8_t *blk, float *out);
void or_dequantize_q6_k_block(const uint8_t *blk, float *out);
int or_decode_row_payload_to_f32(int quant, const uint8_t *row_raw, size_t cols,
                                 float *out, int sanitize_large);

/* ---- portable RepackedWeight ------------------------------------------ */
typedef struct or_repacked {
  size_t rows, cols;
  int quant;
  int dense;               /* 1 = DenseF32 storage */
  size_t blocks_per_row;   /* DenseF32: 32-float blocks per row */
  float *dense_data;       /* rows * blocks_per_row * 32 */
  size_t k_chunks, chunks_per_scale, scale_groups, n_tiles;
  int8_t *tiles;           /* n_tiles * k_chunks * 128 bytes */
  float *scales;           /* n_tiles * scale_groups * 8 */
  float *mins;             /* same size as scales, or NULL */
} or_repacked;

int or_repack(const uint8_t *raw, size_t raw_len, int quant, size_t rows,
              size_t cols, or_repacked *out);
void or_repacked_free(or_repacked *w);

/* Activation quantizer of the repack path (QuantizedActQ8). k_padded =
 * ceil(k/32)*32; f32_rows and q8 are m*k_padded, scales m*ceil(k/32). */
void or_quantize_act_rows(const float *act, size_t m, size_t k, float *f32_rows,
                          int8_t *q8, float *scales);
/* Tile evaluation for rows [r0, r1) of one token. */
void or_eval_row_range(const or_repacked *w, float *out_row, const float *a_f32,
                       const int8_t *a_q8, const float *a_sc, size_t r0,
                       size_t r1);
/* Quantize [m, cols] activations then out[m, rows] = act x W^T
 * (CachedMatrix::project_batch).  nthreads > 1 splits 64-row panels. */
int or_project_batch(const or_repacked *w, float *out, const float *act,
                     size_t m, int nthreads);
/* Integer 16-element dot partials of rows [r0,r1) for one quantized token:
 * out[(r - r0) * k_chunks + ch]. */
void or_dot16_partials(const or_repacked *w, const int8_t *a_q8, size_t r0,
                       size_t r1, int32_t *out);

/* ---- streaming raw-GGUF GEMV (decode_gemv.rs) -------------------------- */
typedef struct or_block_q8_0 { float d; int8_t qs[32]; } or_block_q8_0;
typedef struct or_block_q8_k { float d; int8_t qs[256]; int16_t bsums[16]; } or_block_q8_k;
int or_quantize_row_q8_0(const float *x, size_t n, or_block_q8_0 *out);
int or_quantize_row_q8_k(const float *x, size_t n, or_block_q8_k *out);
int or_gemv_decode_projection(const uint8_t *raw, size_t raw_len, int quant,
                              size_t rows, size_t cols, const float *x,
                              float *out, int nthreads);
float or_compute_row_dot(size_t row, size_t cols, int quant,
                         const uint8_t *raw, size_t raw_len, const float *hidden);

/* ---- elementwise / attention ops (recipe.rs) --------------------------- */
int or_rmsnorm_row(float *out, const float *in, const float *w, size_t n, float eps);
typedef struct or_rope_scaling {
  int kind;  /* 0 none, 1 linear, 2 llama3 smooth, 3 longrope */
  float factor, low_freq_factor, high_freq_factor;
  size_t original_max_position_embeddings;
  const float *short_factor, *long_factor;
  size_t n_factors;
} or_rope_scaling;
int or_fill_inv_freq(size_t head_dim, float theta, const or_rope_scaling *sc,
                     size_t seq_len, float *out);
int or_rope_cos_sin(size_t pos, size_t rotary_dim, const float *inv_freq,
                    float *cos_out, float *sin_out);
int or_apply_rope_cos_sin(float *qk, size_t len, size_t head_dim,
                          size_t rotary_dim, int neox, const float *c,
                          const float *s);
int or_apply_rope(float *qk, size_t len, size_t head_dim, size_t rotary_dim,
                  int neox, size_t pos, const float *inv_freq);
int or_gqa_attention(float *out, const float *q, const float *k_cache,
                     const float *v_cache, size_t m, size_t n_heads_q,
                     size_t n_heads_kv, size_t head_dim, size_t total_seq_len,
                     size_t start_pos, size_t sliding_window, float scale,
                     float *scores_scratch, size_t scratch_len);
int or_swiglu(float *out, const float *gate, const float *up, size_t n);

/* ---- model forward (cached recipe path) -------------------------------- */
typedef struct or_tensor {
  const char *name;
  int quant;
  int n_dims;
  uint64_t ne[4];
  const uint8_t *data;
  size_t nbytes;
} or_tensor;

typedef struct or_geometry {
  size_t num_layers, hidden_dim, ffn_dim, n_heads_q, n_heads_kv, head_dim,
      rotary_dim, vocab_size;
  float rms_eps, rope_theta;
  int neox;                        /* 0 = Norm (interleaved), 1 = NeoX */
  const uint8_t *skip_rope_layers; /* NULL or num_layers flags */
  or_rope_scaling scaling;
  size_t sliding_window;           /* 0 = none */
  int kv_f16;                      /* 1 = K/V stored rounded to f16 (round to
                                      nearest even), as a paged f16 cache holds
                                      them; attention reads them back */
} or_geometry;

typedef struct or_model or_model;
int or_model_build(const or_geometry *g, const or_tensor *tensors,
                   size_t n_tensors, int nthreads, or_model **out);
void or_model_free(or_model *m);
/* KV: f32, layout [layer][K|V][seq_cap][n_kv*head_dim]. */
int or_prefill(or_model *m, float *kv, size_t seq_cap, const uint32_t *tokens,
               size_t n, size_t start_pos, int compute_logits, float *logits);
int or_decode(or_model *m, float *kv, size_t seq_cap, uint32_t token,
              size_t pos, float *logits);
size_t or_model_vocab(const or_model *m);
/* The final normed hidden of the last forward (diagnostics). */
const float *or_model_last_hidden(const or_model *m);

/* ---- seeded synthetic tensors (synth.c; fixtures, not reference code) --- */
uint16_t or_f32_to_f16_rne(float f);
int or_synth_matrix(int quant, size_t rows, size_t cols, uint64_t seed,
                    const char *name, float std_dev, void *out, size_t len,
                    int nthreads);

#ifdef __cplusplus
}
#endif
#endif
