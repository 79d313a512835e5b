/*
 * jal.h -- C ABI of the B200-native (sm_100a) quantized decode/prefill hot
 * path of jero-arch-llama.
 *
 * Every entry point below replaces one public item of the reference crate's
 * recipe / repack_cache / decode_gemv / dispatch surface; the comment beside
 * each names the reference item it stands in for (file:line in the reference
 * crate).  Conventions:
 *   - every function returns an int status (JAL_OK = 0); the codes mirror
 *     jero_core::K3Error.  Nothing aborts; jal_last_error() gives the reason.
 *   - "device pointer" arguments point into CUDA device memory of the current
 *     device; "host pointer" arguments point into host memory.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy stream).
 *   - handles are owned by the caller and released with the matching _free.
 *   - a context is single-threaded; independent contexts may run concurrently.
 */
#ifndef JAL_H
#define JAL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (jero_core::K3Error) ---------------------------------- */
#define JAL_OK 0
#define JAL_ERR_TENSOR_BOUNDS 1           /* K3Error::TensorBoundsError */
#define JAL_ERR_CAPABILITY_MISMATCH 2     /* K3Error::CapabilityMismatch */
#define JAL_ERR_CONTEXT_LENGTH_EXCEEDED 3 /* K3Error::ContextLengthExceeded */
#define JAL_ERR_CUDA 4                    /* a CUDA runtime call failed */
#define JAL_ERR_INVALID_ARGUMENT 5        /* null handle / pointer */
#define JAL_ERR_NCCL 6                    /* an NCCL call failed */
#define JAL_ERR_TIMEOUT 7                 /* a bounded device wait gave up */

/* ---- GGML tensor types (jero_core::QuantType; GGUF type ids) ------------ */
#define JAL_F32 0
#define JAL_F16 1
#define JAL_Q4_0 2
#define JAL_Q5_0 6
#define JAL_Q8_0 8
#define JAL_Q4_K 12
#define JAL_Q5_K 13
#define JAL_Q6_K 14
#define JAL_BF16 30
#define JAL_TQ1_0 34
#define JAL_TQ2_0 35

/* Human-readable reason for the last non-zero status on this thread. */
const char *jal_last_error(void);
/* Library version string. */
const char *jal_version(void);
/* Select the CUDA device used by later calls on this thread. */
int jal_set_device(int device);
/* Number of SMs of the current device (for launch sizing by callers). */
int jal_device_sm_count(int *out);

/* ========================================================================
 * repack_cache.rs -- CachedMatrix
 * ====================================================================== */
typedef struct jal_cached_matrix jal_cached_matrix;

/* CachedMatrix::repack (repack_cache.rs:1516-1579).  `raw` holds `rows` GGUF
 * rows of `cols` elements of type `quant` (host pointer if raw_on_device == 0,
 * else a device pointer).  The device repack keeps Q4_0 at 4.5 bits per
 * weight and Q8_0 at 8.5.  Errors: JAL_ERR_CAPABILITY_MISMATCH for an
 * unsupported quant, JAL_ERR_TENSOR_BOUNDS for a length / shape mismatch. */
int jal_cached_matrix_repack(const void *raw, size_t raw_len, int raw_on_device,
                             int quant, size_t rows, size_t cols,
                             void *stream, jal_cached_matrix **out);
void jal_cached_matrix_free(jal_cached_matrix *m);
/* CachedMatrix::{rows, cols, quant, aligned_bytes, uses_repacked_storage}
 * (repack_cache.rs:1583-1628).  aligned_bytes is the device bytes held. */
size_t jal_cached_matrix_rows(const jal_cached_matrix *m);
size_t jal_cached_matrix_cols(const jal_cached_matrix *m);
int jal_cached_matrix_quant(const jal_cached_matrix *m);
size_t jal_cached_matrix_aligned_bytes(const jal_cached_matrix *m);

/* Export the device repack in the reference's portable tile layout
 * (repack_cache.rs:639-694): tiles[(r/8)*k_chunks + ch] of 128 i8 with byte
 * (r%8)*16+t = q[r][ch*16+t]; scales[((r/8)*groups+g)*8 + r%8] as f32 from
 * f16_to_f32_finite.  Host output buffers; lengths are element counts:
 * tiles_len >= ceil(rows/8)*cols/16*128, scales_len >= ceil(rows/8)*groups*8.
 * groups = cols/32, or cols/16 for Q6_K (BlockScaledI8 storage of the
 * K-quants, unpack_row_i8, repack_cache.rs:890-993).  Used to prove the
 * repack bit-exact. */
int jal_cached_matrix_export_ref_layout(const jal_cached_matrix *m,
                                        int8_t *tiles, size_t tiles_len,
                                        float *scales, size_t scales_len);
/* The group mins of a Q4_K / Q5_K repack (BlockScaledI8 mins,
 * repack_cache.rs:639-694, 890-950) in the same [(r/8)*groups+g][r%8]
 * layout: mins_len >= ceil(rows/8)*(cols/32)*8. */
int jal_cached_matrix_export_ref_mins(const jal_cached_matrix *m, float *mins,
                                      size_t mins_len);

/* CachedMatrix::project_batch / gemm_rows (repack_cache.rs:1709-1787):
 * quantize the [m, cols] f32 activations per 32-block (QuantizedActQ8,
 * repack_cache.rs:390-422) and compute y[m, rows].  Device pointers. */
int jal_cached_matrix_gemm(const jal_cached_matrix *mat, const float *x,
                           size_t m, float *y, void *stream);
/* Same result as jal_cached_matrix_gemm, for callers that cannot allocate
 * device memory while they run: a process whose free device memory belongs
 * to another allocator's pool, or a serving loop that must not call
 * cudaMalloc/cudaFree because they can synchronise the whole device.  No
 * counterpart in the reference.  The quantized activations are kept in one
 * fixed 2 MiB device array that the library holds on every GPU where its
 * kernels are loaded, until the process exits; the call allocates nothing.
 * Limit: round_up(m*cols, 256) + m*(cols/32)*4 <= 2097152 bytes (cols=4096:
 * m <= 455), else JAL_ERR_TENSOR_BOUNDS and no work.  Each call looks up the
 * array's device address on the current device; the first call on a device
 * may load the library's device code there, so make it before any stream
 * capture.
 * The work is only enqueued on `stream` (no synchronisation): every call
 * shares the array, so calls whose GPU work can overlap (other streams,
 * other threads) race; calls on one stream are ordered and safe. */
int jal_cached_matrix_gemm_noalloc(const jal_cached_matrix *mat, const float *x,
                                   size_t m, float *y, void *stream);
/* CachedMatrix::gemv_with_act_view (repack_cache.rs:1636-1672) with an
 * already quantized activation (q8: cols int8, scales: cols/32 f32). */
int jal_cached_matrix_gemv_q8(const jal_cached_matrix *mat, const int8_t *q8,
                              const float *scales, float *y, void *stream);
/* Integer 16-element block-dot partials of rows [r0, r1) against one
 * quantized activation (the i32 `dot_i32` of repack_cache.rs:759-762):
 * out[(r - r0) * (cols/16) + ch].  Device pointers. */
int jal_cached_matrix_dot16_partials(const jal_cached_matrix *mat,
                                     const int8_t *q8, size_t r0, size_t r1,
                                     int32_t *out, void *stream);

/* QuantizedActQ8::quantize_into (repack_cache.rs:491-531): per 32-block
 * scale = amax/127, inv = 1/scale, q = clamp(round(v*inv), -127, 127),
 * non-finite inputs count as 0.  x: [m, k]; q8: [m, ceil(k/32)*32];
 * scales: [m, ceil(k/32)].  Device pointers. */
int jal_act_quantize_q8(const float *x, size_t m, size_t k, int8_t *q8,
                        float *scales, void *stream);
/* quantize_row_q8_0 (decode_gemv.rs:294-313): BlockQ8_0 {f32 d; i8 qs[32]}
 * (36 bytes) with inv = 127/amax.  n % 32 == 0.  Device pointers. */
int jal_quantize_row_q8_0(const float *x, size_t n, void *blocks,
                          void *stream);

/* ========================================================================
 * decode_gemv.rs / dispatch.rs -- streaming raw-GGUF GEMV
 * ====================================================================== */
/* gemv_decode_projection (decode_gemv.rs:1395-1407) and
 * project_lm_head_row_split (dispatch.rs:191-289) for rows in raw GGUF block
 * order: y = W x.  Q4_0/Q5_0/Q8_0: BlockQ8_0 activation quantizer and
 * per-32-block f32(sumi) * (dw * dx) accumulation in block order
 * (decode_gemv.rs: 394-439, 622-642; bit-exact).  Q4_K/Q5_K/Q6_K/TQ1_0/TQ2_0: BlockQ8_K quantizer and the
 * per-super-block integer sums (decode_gemv.rs:320-346, 456-620), blocks
 * added in order (equal to the reference bit for bit).  F16/BF16/F32: the
 * 256-element chunked f32 dot of dot_dense_row_zero_alloc
 * (decode_gemv.rs:1081-1166), also bit-exact.  raw: device pointer to
 * rows*cols GGUF elements. */
int jal_gemv_decode_projection(const void *raw, size_t raw_len, int quant,
                               size_t rows, size_t cols, const float *x,
                               float *y, void *stream);

/* ========================================================================
 * recipe.rs -- fused per-op entry points (device pointers, f32)
 * ====================================================================== */
/* rmsnorm_row over m rows (recipe.rs:2534-2558, eps as given). */
int jal_op_rmsnorm(const float *x, const float *w, size_t m, size_t n,
                   float eps, float *out, void *stream);
/* apply_rope_compat (recipe.rs:2775-2834) on m rows of `row_len` floats at
 * positions pos0..pos0+m-1, using the inv_freq table (rotary_dim/2 floats,
 * device).  neox = 0: pairs (2i, 2i+1); 1: pairs (i, i+rotary_dim/2). */
int jal_op_rope(float *qk, size_t m, size_t row_len, size_t head_dim,
                size_t rotary_dim, int neox, size_t pos0,
                const float *inv_freq, void *stream);
/* swiglu_compat (recipe.rs:3024-3050): out = (g*sigmoid(g))*u. */
int jal_op_swiglu(const float *gate, const float *up, size_t n, float *out,
                  void *stream);
/* gqa_attention_prefill_portable (recipe.rs:2949-3022): m queries at
 * start_pos.. over f32 K/V planes [total_seq][n_kv*head_dim]; causal, with
 * an optional sliding window (0 = none). */
int jal_op_gqa_attention(const float *q, const float *k, const float *v,
                         size_t m, size_t n_heads_q, size_t n_heads_kv,
                         size_t head_dim, size_t total_seq, size_t start_pos,
                         size_t sliding_window, float scale, float *out,
                         void *stream);

/* ========================================================================
 * recipe.rs -- LlamaRecipe
 * ====================================================================== */
typedef struct jal_recipe jal_recipe;

#define JAL_ROPE_NORM 0 /* RopeType::Norm: interleaved pairs */
#define JAL_ROPE_NEOX 1 /* RopeType::NeoX: split-half pairs */

#define JAL_ROPE_SCALING_NONE 0
#define JAL_ROPE_SCALING_LINEAR 1
#define JAL_ROPE_SCALING_LLAMA3 2
#define JAL_ROPE_SCALING_LONGROPE 3

/* The public fields of LlamaRecipe (recipe.rs:110-139). */
typedef struct jal_recipe_fields {
  char architecture[16];
  uint64_t num_layers, hidden_dim, ffn_dim, n_heads_q, n_heads_kv, head_dim,
      vocab_size;
  float rms_eps, rope_theta;
  int32_t rope_type;   /* JAL_ROPE_NORM / JAL_ROPE_NEOX */
  int64_t rotary_dim;  /* -1 = None (use head_dim) */
  int32_t rope_scaling_kind;
  float rope_factor, rope_low_freq_factor, rope_high_freq_factor;
  uint64_t rope_original_max_position_embeddings;
} jal_recipe_fields;

/* LlamaRecipe::new / new_llama4 / new_qwen2 (recipe.rs:163-222) by
 * architecture string "llama" / "llama4" / "qwen2". */
int jal_recipe_new(const char *architecture, jal_recipe **out);
/* LlamaRecipe::from_gguf (recipe.rs:336-422): hydrate from GGUF v3 bytes. */
int jal_recipe_from_gguf(const void *gguf, size_t len, jal_recipe **out);
void jal_recipe_free(jal_recipe *r);
int jal_recipe_get_fields(const jal_recipe *r, jal_recipe_fields *out);
int jal_recipe_set_fields(jal_recipe *r, const jal_recipe_fields *in);
/* with_irope_mask (recipe.rs:452-455) / should_skip_rope (recipe.rs:466-472) */
int jal_recipe_set_irope_mask(jal_recipe *r, const uint8_t *mask, size_t n);
int jal_recipe_should_skip_rope(const jal_recipe *r, size_t layer);
/* with_rope_scaling LongRope tables (recipe.rs:56-64, 2638-2657). */
int jal_recipe_set_longrope(jal_recipe *r, const float *short_factor,
                            const float *long_factor, size_t n,
                            uint64_t original_max_position_embeddings);
/* ArchRecipe::supports_quant (recipe.rs:1819-1832): 1 / 0. */
int jal_recipe_supports_quant(const jal_recipe *r, int quant);
/* ArchRecipe::validate_model (recipe.rs:1834-1931) over GGUF bytes. */
int jal_recipe_validate_model(const jal_recipe *r, const void *gguf,
                              size_t len);
/* decode_scratch_bytes (recipe.rs:529-547): device scratch bytes one
 * context needs for decode up to seq_len_upper_bound positions. */
size_t jal_recipe_decode_scratch_bytes(const jal_recipe *r,
                                       size_t seq_len_upper_bound);

/* ========================================================================
 * repack_cache.rs -- ModelRepackCache
 * ====================================================================== */
typedef struct jal_model_cache jal_model_cache;

/* LlamaRecipe::build_repack_cache (recipe.rs:481-509) ->
 * ModelRepackCache::build (repack_cache.rs:2166-2257): upload and repack
 * every layer matrix, norm and bias of the GGUF model onto `device`. */
int jal_model_repack_cache_build(const jal_recipe *r, const void *gguf,
                                 size_t len, int device,
                                 jal_model_cache **out);
void jal_model_repack_cache_free(jal_model_cache *c);
/* ModelRepackCache accessors (repack_cache.rs:2259-2380). */
size_t jal_model_cache_num_layers(const jal_model_cache *c);
size_t jal_model_cache_hidden_dim(const jal_model_cache *c);
size_t jal_model_cache_ffn_dim(const jal_model_cache *c);
size_t jal_model_cache_total_q(const jal_model_cache *c);
size_t jal_model_cache_total_kv(const jal_model_cache *c);
size_t jal_model_cache_vocab_size(const jal_model_cache *c);
size_t jal_model_cache_norm_count(const jal_model_cache *c);
size_t jal_model_cache_bias_count(const jal_model_cache *c);
size_t jal_model_cache_repacked_matrix_count(const jal_model_cache *c);
size_t jal_model_cache_total_aligned_bytes(const jal_model_cache *c);
/* Borrow layer matrices (LayerRepackCache fields, repack_cache.rs:
 * 2084-2111): which = 0 q, 1 k, 2 v, 3 output, 4 gate, 5 up, 6 down;
 * layer = num_layers selects the LM head.  Owned by the cache. */
const jal_cached_matrix *jal_model_cache_matrix(const jal_model_cache *c,
                                                size_t layer, int which);

/* ========================================================================
 * Tensor parallelism (one process per GPU over NCCL)
 *
 * The reference runs on one host with rayon threads and has no tensor
 * parallel path; these entry points are the jal_tp_init(nccl_unique_id,
 * rank, world) the scope table asks for.  Shards: Q/K/V by whole KV heads
 * (and their query heads), gate/up by FFN rows, O and down by input columns
 * (whole 32-blocks), the LM head by vocabulary rows (per-rank slices of
 * ceil(vocab / world) rows); embedding and norms are replicated and the O
 * bias is added by rank 0.  One f32 all-reduce after O and after down per
 * layer, one all-gather of the logits per step.  Contexts on a sharded cache
 * run the fast numerics only; each rank calls the same sequence of
 * prefill / decode entry points with the same tokens.
 * ====================================================================== */
typedef struct jal_tp jal_tp;

typedef struct jal_tp_plan_t {
  uint64_t rank, world;
  uint64_t q_lo, q_n;    /* query heads */
  uint64_t kv_lo, kv_n;  /* KV heads */
  uint64_t f_lo, f_n;    /* FFN rows / down input columns */
  uint64_t v_lo, v_n;    /* LM-head vocabulary rows */
  uint64_t v_pad;        /* logits slice per rank in the all-gather */
} jal_tp_plan_t;

/* Shard plan (no GPU needed); fails with JAL_ERR_CAPABILITY_MISMATCH when
 * heads or the FFN width do not split into whole heads / 32-blocks. */
int jal_tp_plan(size_t n_heads_q, size_t n_heads_kv, size_t ffn_dim,
                size_t vocab, int rank, int world, jal_tp_plan_t *out);
/* 128-byte NCCL unique id: rank 0 creates it, the caller distributes it. */
int jal_tp_unique_id(uint8_t *id_out);
/* Joins the communicator on the current device (collective over ranks). */
int jal_tp_init(const uint8_t *id, int rank, int world, jal_tp **out);
void jal_tp_free(jal_tp *tp);
/* jal_model_repack_cache_build for this rank's shard; `tp` must outlive
 * the cache and every context made from it. */
int jal_model_repack_cache_build_tp(const jal_recipe *r, const void *gguf,
                                    size_t len, int device,
                                    const jal_tp *tp, jal_model_cache **out);

/* ========================================================================
 * ExecutionContext + prefill_step / decode_step
 * ====================================================================== */
typedef struct jal_context jal_context;

#define JAL_KV_F32 0 /* parity mode: f32 K/V like the reference */
#define JAL_KV_F16 1 /* paged fp16 K/V */

typedef struct jal_context_config {
  uint64_t n_ctx;          /* max positions (ExecutionContext::n_ctx) */
  int32_t kv_dtype;        /* JAL_KV_F32 / JAL_KV_F16 */
  uint32_t page_size;      /* tokens per KV page (0 = 64) */
  uint64_t sliding_window; /* KvGeometry::sliding_window, 0 = none */
  int32_t use_graphs;      /* capture the decode step in a CUDA graph */
  int32_t numerics;        /* JAL_NUMERICS_FAST or JAL_NUMERICS_REFERENCE */
} jal_context_config;

/* Numerics of an execution context (no counterpart setting in the
 * reference).
 *   FAST (default): the serving path.  On one GPU every f32 reduction runs in
 *     the reference's order (recipe.rs / repack_cache.rs: per-16-chunk
 *     projection terms folded left to right, sequential RMSNorm sums and
 *     softmax denominators, position-ordered attention sums), with
 *     bandwidth-oriented kernels, so logits and greedy tokens equal the
 *     reference's.  A tensor-parallel context splits each projection's sum
 *     over the ranks by construction and runs the RELAXED kernels.
 *   REFERENCE: the same order with simple one-chain-per-reduction kernels,
 *     a slow cross-check of FAST.
 *   RELAXED: reductions reordered for bandwidth (tree sums, fused
 *     multiply-adds, 32-element blocks); logits drift from the reference by
 *     up to ~1e-2 because the int8 activation quantizer amplifies one-ulp
 *     differences.  Its prefill attention runs on f16 tensor cores and
 *     rounds Q to f16, so query activations beyond +-65504 overflow there
 *     (FAST and REFERENCE keep f32). */
#define JAL_NUMERICS_FAST 0
#define JAL_NUMERICS_REFERENCE 1
#define JAL_NUMERICS_RELAXED 2

/* Creates a context over model cache c.  The device step takes Q4_0 / Q5_0
 * / Q8_0 layer matrices (uniform across q/k/v and across gate/up) and an LM
 * head in Q4_0 / Q5_0 / Q8_0, F32 / F16 / BF16 or, with the FAST or
 * REFERENCE numerics on one GPU, Q4_K / Q5_K / Q6_K (repacked, projected in
 * the reference's order with its group-min term); anything else fails with
 * JAL_ERR_CAPABILITY_MISMATCH. */
int jal_context_new(const jal_recipe *r, const jal_model_cache *c,
                    const jal_context_config *cfg, jal_context **out);
void jal_context_free(jal_context *ctx);

/* Caller-owned KV storage: the reference's KvCacheView, which the engine
 * owns and the recipe appends into (recipe.rs:2319-2326, layer_kv_mut; the
 * ExecutionContext holds only the position, lib.rs:1022-1035).  The paged
 * K / V pools of `model` (this rank's KV heads for a tensor-parallel cache)
 * for n_ctx positions, kv_dtype JAL_KV_F16 / JAL_KV_F32, page_size 0 = 64;
 * zero-filled, on the model's device.  A cache outlives every context made
 * over it and keeps its contents when a context is freed; contexts over one
 * cache must not run at the same time. */
typedef struct jal_kv_cache jal_kv_cache;
int jal_kv_cache_alloc(const jal_model_cache *model, uint64_t n_ctx,
                       int32_t kv_dtype, uint32_t page_size, jal_kv_cache **out);
void jal_kv_cache_free(jal_kv_cache *kv);
/* Device bytes the cache holds. */
size_t jal_kv_cache_bytes(const jal_kv_cache *kv);
/* jal_context_new over a caller-owned cache: cfg->kv_dtype and page_size
 * must match the cache and cfg->n_ctx must not exceed it
 * (JAL_ERR_CAPABILITY_MISMATCH / JAL_ERR_CONTEXT_LENGTH_EXCEEDED). */
int jal_context_new_with_kv(const jal_recipe *r, const jal_model_cache *c,
                            const jal_context_config *cfg, jal_kv_cache *kv,
                            jal_context **out);
/* Sets the position (ExecutionContext::position) to resume over a cache
 * whose positions [0, pos) were filled earlier, e.g. by another context. */
int jal_context_set_position(jal_context *ctx, size_t pos);
/* ExecutionContext::position. */
size_t jal_context_position(const jal_context *ctx);
/* Drop all positions (KV content becomes stale). */
int jal_context_reset(jal_context *ctx);
/* prefill_step_with_cache (recipe.rs:517-524, 564-608): n prompt tokens at
 * start_pos (chunked prefill when start_pos > 0).  When compute_logits,
 * logits (host, logits_len == vocab) receive the last token's logits.
 * Position becomes start_pos + n; unchanged on error. */
int jal_prefill_step(jal_context *ctx, const uint32_t *tokens, size_t n,
                     size_t start_pos, int compute_logits, float *logits,
                     size_t logits_len);
/* decode_step_with_cache (recipe.rs:555-562, 718-1163): one token at the
 * current position; logits (host, vocab floats) may be NULL.  Position
 * advances by one; unchanged on error. */
int jal_decode_step(jal_context *ctx, uint32_t token, float *logits,
                    size_t logits_len);
/* One decode step for n independent sequences at once, ctxs[i] holding
 * sequence i (no counterpart in the reference, whose batched forward
 * (recipe.rs:1489-1756) runs one sequence's prompt rows; this batches
 * sequences the way a serving engine does).  The contexts share one model
 * cache, run JAL_NUMERICS_FAST on one GPU and own distinct KV caches; token
 * i is decoded at ctxs[i]'s position, which then advances by one.  The
 * projections stream each weight matrix once for all n rows; every f32 sum
 * keeps the reference's order, so sequence i's logits equal what
 * jal_decode_step on ctxs[i] alone returns.  logits (host, n x vocab floats,
 * row i for sequence i) may be NULL: jal_context_batch_logits_device(ctxs[0])
 * then gives the device rows.  Work runs on ctxs[0]'s stream (replayed from
 * a CUDA graph kept for the list of contexts when graphs are on); nothing
 * changes on error. */
int jal_decode_batch(jal_context *const *ctxs, size_t n, const uint32_t *tokens,
                     float *logits, size_t logits_len);
/* Device pointer to the last jal_decode_batch logits ([n][vocab] f32) of the
 * batch whose first context is ctx. */
int jal_context_batch_logits_device(const jal_context *ctx, const float **out);
/* Greedy decode of n_steps tokens on the device, starting from `token` at
 * the current position (argmax, lowest index wins ties; the reference
 * leaves sampling to the engine).  tokens_out (host) gets n_steps ids. */
int jal_decode_greedy(jal_context *ctx, uint32_t token, size_t n_steps,
                      uint32_t *tokens_out);
/* Copy the KV cache of positions [0, n_pos) into the reference's f32 layout
 * [layer][K|V][n_pos][n_kv*head_dim] (host buffer, len floats). */
int jal_context_export_kv(const jal_context *ctx, size_t n_pos, float *out,
                          size_t len);
/* Device pointer to the last logits (vocab f32) for zero-copy callers. */
int jal_context_logits_device(const jal_context *ctx, const float **out);
/* Number of kernels one decode step launches (graph nodes when graphs are
 * on). */
int jal_context_last_step_launches(const jal_context *ctx, size_t *out);
/* How the decode step of a tensor-parallel context combines the ranks'
 * partial sums: JAL_TP_EXCHANGE_NONE (one rank), JAL_TP_EXCHANGE_NCCL
 * (all-reduce after O and down) or JAL_TP_EXCHANGE_PEER (the O / down GEMVs
 * store into every rank's slots over peer memory and the next RMSNorm GEMV
 * adds them; set JAL_TP_NCCL=1 in the environment to force NCCL). */
enum { JAL_TP_EXCHANGE_NONE = 0, JAL_TP_EXCHANGE_NCCL = 1, JAL_TP_EXCHANGE_PEER = 2 };
int jal_context_tp_exchange(const jal_context *ctx, int *out);
/* Issue the context's work on `stream` (a cudaStream_t; NULL restores the
 * context's own stream).  Lets callers order it with their own work and
 * time it with events recorded on the same stream. */
int jal_context_set_stream(jal_context *ctx, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* JAL_H */
