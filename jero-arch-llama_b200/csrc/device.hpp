// Device-side data layout shared by the host orchestration and the kernels.
//
// HBM layout of a repacked quantized matrix (B200 layout), row-interleaved:
// row r occupies qs_stride bytes at qs + r * qs_stride:
//   quants: Q4_0 the 16 nibble bytes of each GGUF block back to back (byte i
//           = elem i | elem i+16 << 4), cols/2 bytes; Q8_0 the 32 int8 of each
//           block back to back, cols bytes.  Every block starts 16-byte aligned.
//   scales: right after the quants (d = qs + quant bytes, d_stride = qs_stride
//           / 2 halves per row), one f16 bit pattern per 32-block, padded to a
//           multiple of 8 (16 bytes), sanitized at repack (f16_to_f32_finite).
// A contiguous range of rows is therefore one contiguous byte range (one
// bulk copy); weight bytes stay at 4.5 (Q4_0) / 8.5 (Q8_0) bits per weight.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace jal {

struct DevMat {
  int quant = 0;          // JAL_Q4_0, JAL_Q8_0, or JAL_F16 / JAL_BF16 / JAL_F32 for dense rows
  int64_t rows = 0, cols = 0;
  const uint8_t *qs = nullptr;
  const uint16_t *d = nullptr;
  const void *dense = nullptr;  // dense rows in their GGUF element type (cols stride)
  int64_t qs_stride = 0;  // bytes per row (quants + scales)
  int64_t d_stride = 0;   // row stride of d in halves (qs_stride / 2)
  // K-quant layout (JAL_Q4_K / Q5_K / Q6_K): qs holds one int8 quant per
  // element (qs_stride bytes per row); ks / km the f32 scale / min of each
  // group of 32 (16 for Q6_K) elements, k_stride floats per row; km null for
  // Q6_K.
  const float *ks = nullptr, *km = nullptr;
  int64_t k_stride = 0;
};

inline int64_t d_stride_for(int64_t cols) { return ((cols / 32) + 7) / 8 * 8; }

// Step trace slots per launch: {first CTA start, last warp end, 6 phase marks}.
constexpr int kTraceSlots = 8;

// ---- GEMV (decode, M tokens <= kGemvMaxM) ------------------------------
// GEMV_IN_PREQ (persistent step only): the RMSNorm input arrives already
// block-quantized as (row x norm weights) with the producers' partial sums of
// squares of the row; the norm scale is folded into the block scales.
enum GemvIn : int { GEMV_IN_Q8 = 0, GEMV_IN_F32 = 1, GEMV_IN_NORM = 2, GEMV_IN_PREQ = 3 };
// GEMV_OUT_PEER (tensor-parallel decode): each row value goes to every
// rank's partial-sum slot over peer memory as a flagged 64-bit word.
enum GemvOut : int { GEMV_OUT_STORE = 0, GEMV_OUT_ADD = 1, GEMV_OUT_SWIGLU = 2, GEMV_OUT_PEER = 3 };
constexpr int kPeerMax = 8;
constexpr int kErrPeerWait = 16;  // bit set in the context error word
constexpr int kGemvMaxM = 8;
constexpr int kGemvMaxSmem = 200 * 1024;

struct GemvArgs {
  DevMat w;
  int64_t rows = 0;        // logical output rows (pairs for SWIGLU)
  int m = 1;               // tokens
  int in_mode = GEMV_IN_Q8;
  const float *x = nullptr;     // [m][x_stride] f32 (IN_F32 / IN_NORM)
  const float *norm_w = nullptr;
  float eps = 1e-5f;
  const int8_t *xq = nullptr;   // [m][xq_stride] int8 (IN_Q8)
  const float *xs = nullptr;    // [m][xq_stride/32] f32 scales (IN_Q8)
  int64_t x_stride = 0, xq_stride = 0;
  int out_mode = GEMV_OUT_STORE;
  float *y = nullptr;           // [m][y_stride]
  int64_t y_stride = 0;
  const float *bias = nullptr;  // per output row (OUT_STORE / OUT_ADD)
  int64_t up_offset = 0;        // SWIGLU: physical row offset of the up half
  int8_t *yq = nullptr;         // SWIGLU (persistent step): y also as QuantizedActQ8,
  float *ys = nullptr;          //   each 32-block quantized by the CTA that completes it
  unsigned *ycnt = nullptr;     //   per-block row counters (zero between uses)
  const float *ss_part = nullptr;  // GEMV_IN_PREQ: partial sums of squares of the row
  int ss_n = 0;
  // GEMV_OUT_ADD in the persistent step: the finished rows also become the
  // next RMSNorm input: u = row x nx_norm (nx_u, block-quantized into nx_q /
  // nx_s through nx_cnt) and this CTA's sum of squares (nx_ss[cta]).
  const float *nx_norm = nullptr;
  float *nx_u = nullptr, *nx_s = nullptr, *nx_ss = nullptr;
  int8_t *nx_q = nullptr;
  unsigned *nx_cnt = nullptr;
  // Tensor-parallel exchange over peer memory (decode, M = 1).  A slot word
  // is (flag << 32) | f32 bits, flag = epoch * 256 + phase + 1 with epoch
  // the context's step counter (*peer_epoch) and phase < 255 the exchange
  // within the step; a 64-bit store is single-copy atomic, so a word whose
  // flag matches carries this step's value.
  // IN_NORM with peer_in: the row is x + slot row 0 + slot row 1 + ...
  // (peer_world rows of x_stride words, added in rank order, so every rank
  // gets the same bits), each word waited for until its flag matches
  // (bounded: kErrPeerWait in *err); CTA 0 stores the sum to x_out.
  // GEMV_OUT_PEER: each row value (+ bias) is stored as a word to
  // peer_out[r][row] for r < peer_world.
  const unsigned long long *peer_in = nullptr;
  const uint32_t *peer_epoch = nullptr;
  int peer_phase = 0;
  int peer_world = 0;
  float *x_out = nullptr;
  int *err = nullptr;
  uint64_t peer_wait_ns = 0;    // bound of the exchange wait (0 = 4 s)
  unsigned long long *peer_out[kPeerMax] = {};
  int grid = 0;                 // CTAs (0 = auto)
  int pdl = 0;                  // launch with programmatic dependent launch
  int64_t pf_bytes = -1;        // L2 prefetch budget per CTA (-1 = default)
  unsigned long long *trace = nullptr;  // step trace: {first CTA start, last warp end} (ns), see KernelTrace
};

void launch_gemv(const GemvArgs &a, cudaStream_t s);
// Dense rows (dense.cu): M = 1, f32 or RMSNorm input, stored output; the
// reference-order form takes the normed f32 row.
bool dense_quant(int q);
void launch_gemv_dense(const GemvArgs &a, cudaStream_t s);
void launch_strict_gemv_dense(const DevMat &w, const float *x, int64_t rows, float *y, cudaStream_t s);
// True when launch_gemv runs `a` (with peer_in or GEMV_OUT_PEER) on the
// segmented kernel whose prologue / epilogue implement the exchange.
bool gemv_peer_supported(const GemvArgs &a);
int gemv_default_grid(const GemvArgs &a);
// Sets the kernels' shared-memory limits (call before any stream capture).
void gemv_init();
size_t gemv_smem_bytes(int in_mode, int m, int64_t cols);

// Reference-order decode GEMV (xgemv.cu): M = 1, Q4_0 / Q8_0, inputs Q8 /
// F32 / RMSNorm, outputs STORE / ADD / SWIGLU.
bool xgemv_supported(const GemvArgs &a);
size_t xgemv_smem_bytes(int quant, int64_t cols, int in_mode);
void xgemv_init();
void launch_xgemv(const GemvArgs &a, cudaStream_t s);

// ---- repack / export / activation quantizers ---------------------------
void launch_repack(const uint8_t *raw, int quant, int64_t rows, int64_t cols, uint8_t *qs, uint16_t *d,
                   int64_t qs_stride, int64_t d_stride, cudaStream_t s);
void launch_export_ref(const DevMat &w, int8_t *tiles, float *scales, cudaStream_t s);
// K-quant matrices (kquant.cu).
bool kquant(int quant);
int kquant_group(int quant);  // elements per scale group: 32, or 16 for Q6_K
void launch_repack_kquant(const uint8_t *raw, int quant, int64_t rows, int64_t cols, int8_t *qs, int64_t qs_stride,
                          float *ks, float *km, int64_t k_stride, cudaStream_t s);
// y[m][rows] in the reference's order from the f32 activation x (for the
// group sums) and its QuantizedActQ8 rows xq / xs.
void launch_kq_gemm(const DevMat &w, const float *x, const int8_t *xq, const float *xs, int64_t m, float *y,
                    cudaStream_t s);
// Host copies of the reference's portable layout (tiles, scales, mins; any may be null).
void export_kquant_ref(const DevMat &w, int8_t *tiles, float *scales, float *mins);
void launch_act_quant(const float *x, int64_t m, int64_t k, int64_t x_stride, int8_t *q8, float *scales,
                      cudaStream_t s);
void launch_quantize_row_q8_0(const float *x, int64_t n, void *blocks, cudaStream_t s);
void launch_rmsnorm(const float *x, const float *w, int64_t m, int64_t n, float eps, float *out,
                    cudaStream_t s);
// Sets the RMSNorm kernels' shared-memory limit (call before any capture).
void norm_init();
// Per-row RMSNorm then QuantizedActQ8 of the normed row (prefill).
void launch_rmsnorm_quant(const float *x, const float *w, int64_t m, int64_t n, float eps, int8_t *q8,
                          float *scales, cudaStream_t s);
void launch_dot16_partials(const DevMat &w, const int8_t *q8, int64_t r0, int64_t r1, int32_t *out,
                           cudaStream_t s);
void launch_gemv_raw(const uint8_t *raw, int quant, int64_t rows, int64_t cols, const void *xblocks,
                     float *y, cudaStream_t s);
// Streaming GEMV of the super-block types (Q4_K, Q5_K, Q6_K, TQ1_0, TQ2_0)
// against BlockQ8_K activations (kQ8KBlockBytes per 256 elements), and of
// dense F16 / BF16 / F32 rows against the f32 activation (stream_gemv.cu).
constexpr int kQ8KBlockBytes = 304;
bool superblock_quant(int q);
void launch_quantize_row_q8_k(const float *x, int64_t n, void *blocks, cudaStream_t s);
void launch_gemv_raw_superblock(const uint8_t *raw, int quant, int64_t rows, int64_t cols, const void *xblocks,
                                float *y, cudaStream_t s);
void launch_gemv_raw_dense(const uint8_t *raw, int quant, int64_t rows, int64_t cols, const float *x, float *y,
                           cudaStream_t s);

// ---- GEMM (prefill) -------------------------------------------------------
// y[m][rows] (= or +=) q8[m][K] x W^T with per-16-chunk integer partials.
struct GemmArgs {
  DevMat w;
  int64_t m = 0, rows = 0;
  const int8_t *xq = nullptr;  // [m][K]
  const float *xs = nullptr;   // [m][K/32]
  float *y = nullptr;
  int64_t y_stride = 0;
  const float *bias = nullptr;
  int accumulate = 0;          // y += result
};
void launch_gemm(const GemmArgs &a, cudaStream_t s);
// y[m][rows] = quantized activations x W^T in the reference's f32 order: the
// decode GEMV for one token, the GEMM otherwise (op-level entry points).
void project_q8(const DevMat &w, const int8_t *xq, const float *xs, int64_t m, float *y, cudaStream_t s);

// Quantize-then-project with the activation scratch in a fixed file-scope
// device array (noalloc.cu) instead of a per-call allocation.
void gemm_noalloc(const DevMat &w, const float *x, int64_t m, float *y, cudaStream_t s);

// ---- elementwise / attention ---------------------------------------------
void launch_rope_rows(float *qk, int64_t m, int64_t row_len, int64_t head_dim, int64_t rotary_dim, int neox,
                      int64_t pos0, const float *inv_freq, cudaStream_t s);
void launch_swiglu(const float *g, const float *u, int64_t n, float *out, cudaStream_t s);
// SwiGLU rows straight into QuantizedActQ8 blocks (prefill down-projection input).
void launch_swiglu_act_quant(const float *gu, int64_t m, int64_t f, int64_t stride, int8_t *q8, float *scales,
                             cudaStream_t s);
void launch_gqa_attention_ref(const float *q, const float *k, const float *v, int64_t m, int64_t nq, int64_t nkv,
                              int64_t hd, int64_t total_seq, int64_t start_pos, int64_t window, float scale,
                              float *out, cudaStream_t s);

// KV cache pool: element (layer, page, head, slot, dim) at
// (((layer * n_pages + page) * n_kv + head) * page_size + slot) * head_dim + dim,
// one pool for K and one for V; dtype f32 or f16.
struct KvView {
  void *k = nullptr, *v = nullptr;
  int f16 = 1;
  int64_t n_pages = 0, page_size = 64, n_kv = 0, head_dim = 0, n_layers = 0;
  const int32_t *page_table = nullptr;  // logical page -> physical page
};

struct AttnDecodeArgs {
  const float *qkv = nullptr;  // [q | k | v] f32 of one token
  const float *bq = nullptr, *bk = nullptr, *bv = nullptr;
  const float *cos_tab = nullptr, *sin_tab = nullptr;  // [n_ctx][rot/2]
  const float *cos_tab_long = nullptr, *sin_tab_long = nullptr;
  int64_t long_threshold = -1;  // use long tables when pos + 1 > threshold
  int skip_rope = 0, neox = 0;
  int64_t n_heads_q = 0, rotary_dim = 0;
  KvView kv;
  int64_t layer = 0;
  const int64_t *d_pos = nullptr;  // current position (device)
  int64_t window = 0;
  float scale = 1.f;
  int n_splits = 1;             // CTAs per KV head = thread-block cluster size (<= 16)
  float *out = nullptr;         // [n_heads_q * head_dim]
  int8_t *out_q = nullptr;      // quantized out (QuantizedActQ8)
  float *out_s = nullptr;
  int *err = nullptr;           // error word: bit 2 = a bounded copy wait gave up
  int pdl = 0;
  uint64_t wait_ns = 0;         // bound of each copy wait (0 = 2 s)
  uint32_t test_extra_tx = 0;   // test hook: the first V copy's barrier expects this many bytes more (k_attn_decode)
  float *w_out = nullptr;       // reference-order kernel: [n_heads_q][w_stride] weights e_t / den by position
  int64_t w_stride = 0;
  unsigned long long *trace = nullptr;  // step trace slot (KernelTrace)
};
void launch_attn_decode(const AttnDecodeArgs &a, cudaStream_t s);
// Reference-order decode attention, scores (xattn.cu): clusters of
// a.n_splits CTAs per KV head build q / k / v, append k / v, and write each
// query head's weights w_t = e_t * (1 / den) to a.w_out; n_ctx bounds the
// positions (shared-memory sizing).
void launch_xattn_decode(const AttnDecodeArgs &a, int64_t n_ctx, cudaStream_t s);
// Cluster size for launch_xattn_decode (>= G), 0 when the shape does not fit.
int xattn_cluster_size(int head_dim, int f16, int G, int n_kv, int64_t n_ctx);
// The smallest cluster size (>= G) for launch_xattn_decode at n_ctx, so that
// several sequences' launches share the GPU (batched decode); 0 if none fits.
int xattn_batch_cluster_size(int head_dim, int f16, int G, int64_t n_ctx);

// Reference-order decode attention, output (xattn_v.cu): out_d = sum_t w_t
// * v_td in position order, then its QuantizedActQ8 blocks.
struct AttnVArgs {
  KvView kv;
  int64_t layer = 0, window = 0, n_heads_q = 0;
  const int64_t *d_pos = nullptr;
  const float *w = nullptr;  // [n_heads_q][w_stride], by position
  int64_t w_stride = 0;
  float *out = nullptr;
  int8_t *out_q = nullptr;
  float *out_s = nullptr;
  int *err = nullptr;  // bit value 2: a bounded copy wait gave up
  int pdl = 0;
  uint64_t wait_ns = 0;
  uint32_t test_extra_tx = 0;  // test hook: the last V stage's barrier expects this many bytes more
  unsigned long long *trace = nullptr;  // step trace slot (KernelTrace)
};
// Positions per V stage: the largest power of two <= 64 dividing the page size.
int kv_stage_rows(int64_t page_size);
bool xattn_v_supported(int64_t head_dim, int64_t page_size, int64_t n_ctx);
// Encodes the 2D tensor map of one KV plane at `base` (rows of head_dim
// elements, boxes of 32 dims x kv_stage_rows positions) into tm_out, a
// 64-byte aligned 128-byte buffer.  False if the driver refuses.
bool make_kv_tensor_map(const KvView &kv, const void *base, void *tm_out);
void launch_xattn_v(const void *tm, const AttnVArgs &a, int64_t n_ctx, cudaStream_t s);
// Largest cluster size (<= want) the decode attention kernel can run with
// for head_dim, KV element type and G query heads per KV head.
int attn_decode_cluster_size(int head_dim, int f16, int G, int want);

// ---- reference-order decode (strict.cu) -----------------------------------
struct StrictQkvArgs {
  const float *qkv = nullptr;  // [q | k | v] projection output of one token
  const float *bq = nullptr, *bk = nullptr, *bv = nullptr;
  const float *cos_tab = nullptr, *sin_tab = nullptr, *cos_tab_long = nullptr, *sin_tab_long = nullptr;
  int64_t long_threshold = -1;
  int skip_rope = 0, neox = 0;
  int64_t n_heads_q = 0, rotary_dim = 0, layer = 0;
  KvView kv;
  const int64_t *d_pos = nullptr;
  float *qbuf = nullptr;  // [n_heads_q * head_dim]
};
struct StrictAttnArgs {
  const float *qbuf = nullptr;
  KvView kv;
  int64_t n_heads_q = 0, layer = 0, window = 0;
  const int64_t *d_pos = nullptr;
  float scale = 1.f;
  float *out = nullptr;  // [n_heads_q * head_dim]
};
void launch_strict_rmsnorm(const float *x, const float *w, int64_t n, float eps, float *out, cudaStream_t s);
size_t strict_gemv_smem(int64_t cols);
void launch_strict_gemv(const DevMat &w, const int8_t *q8, const float *scales, int64_t rows, bool add, float *y,
                        const float *bias, cudaStream_t s);
void launch_strict_swiglu(const float *g, const float *u, int64_t n, float *out, cudaStream_t s);
void launch_strict_qkv_prep(const StrictQkvArgs &a, cudaStream_t s);
void launch_strict_attn(const StrictAttnArgs &a, int64_t n_ctx, cudaStream_t s);
// Sets the device token and position (stream-ordered, no host staging).
void launch_set_token_pos(uint32_t *d_token, uint32_t token, int64_t *d_pos, int64_t pos, cudaStream_t s);

// ---- persistent decode step (decode_mega.cu) --------------------------------
struct MegaLayer {
  DevMat qkv, wo, gateup, wdown;  // Q|K|V and gate|up stacked
  const float *attn_norm = nullptr, *ffn_norm = nullptr;
  const float *bq = nullptr, *bk = nullptr, *bv = nullptr, *bo = nullptr;
  int skip_rope = 0;
};
struct MegaArgs {
  int n_layers = 0;
  int64_t H = 0, F = 0, V = 0, n_heads_q = 0, n_kv = 0, rotary_dim = 0;
  float eps = 1e-5f, scale = 1.f;
  const MegaLayer *layers = nullptr;  // device array [n_layers]
  DevMat lm_head;
  const float *out_norm = nullptr;
  const uint8_t *emb = nullptr;
  int emb_quant = 0;
  int64_t emb_rows = 0;
  const float *cos_tab = nullptr, *sin_tab = nullptr, *cos_long = nullptr, *sin_long = nullptr;
  int64_t long_threshold = -1;
  int neox = 0;
  KvView kv;
  int64_t window = 0;
  int64_t *d_pos = nullptr;
  uint32_t *d_token = nullptr, *d_hist = nullptr;
  float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *ffn = nullptr, *logits = nullptr;
  int8_t *attn_q = nullptr, *ffn_q = nullptr;
  float *attn_s = nullptr, *ffn_s = nullptr;
  unsigned *ffn_cnt = nullptr;  // [F / 32] block counters of the SwiGLU output (zero between steps)
  // next RMSNorm input, formed by the phase that finishes the hidden row:
  float *hu = nullptr;          // [H] hidden x norm weights
  int8_t *hq = nullptr;         // [H] its QuantizedActQ8 blocks
  float *hs = nullptr;          // [H / 32] their scales
  unsigned *hcnt = nullptr;     // [H / 32] block counters (zero between uses)
  float *hss = nullptr;         // [grid] per-CTA sums of squares of the hidden row
  float *attn_part = nullptr;   // [n_kv][splits][4 * hd + 8] attention split partials
  unsigned *head_cnt = nullptr; // [n_kv] split arrival counters (zero between steps)
  unsigned *bar = nullptr;      // grid barrier arrival count (zero between steps)
  float *am_val = nullptr;
  int *am_idx = nullptr;
  unsigned *am_cnt = nullptr;
  int *err = nullptr;           // error word (bit 1 token, 2 copy wait, 8 grid wait)
  int splits = 1;               // attention CTAs per KV head (<= 64)
  int attn_split_tokens = 128;  // attended positions per attention split (fewer splits for short spans)
};
// Whether the persistent decode step supports this model shape at `grid`
// CTAs (head_dim, KV type, query heads per KV head, segment counts, shared
// memory).
int mega_check(const MegaArgs &a, int grid);
// Bytes of the attention split partials (MegaArgs::attn_part).
size_t mega_part_bytes(const MegaArgs &a);
// Checks the shape (mega_check) and sets the kernel's shared-memory limit;
// call once before the first launch.  Returns 0 when the shape does not fit.
int prepare_decode_mega(const MegaArgs &a, int grid);
// Launches one decode token as a cooperative kernel of `grid` CTAs; the
// kernel reads its arguments from dev_args, a device copy of `a`.  Returns 0
// when no instantiation fits or the launch was rejected.
int launch_decode_mega(const MegaArgs &a, const MegaArgs *dev_args, int grid, cudaStream_t s);
// Whether a matrix can run the segmented decode GEMV (cols a multiple of 128
// blocks of at most 16 segments, 32-byte aligned rows, Q4_0 / Q8_0).
bool w4_matrix_ok(const DevMat &w);

// Prefill: bias + RoPE on q/k rows, append k/v of m tokens into the cache.
struct RopeAppendArgs {
  float *qkv = nullptr;  // [m][qkv_stride]: q | k | v
  int64_t m = 0, qkv_stride = 0, start_pos = 0;
  const float *bq = nullptr, *bk = nullptr, *bv = nullptr;
  const float *cos_tab = nullptr, *sin_tab = nullptr;
  int skip_rope = 0, neox = 0;
  int64_t n_heads_q = 0, rotary_dim = 0;
  KvView kv;
  int64_t layer = 0;
};
void launch_rope_append(const RopeAppendArgs &a, cudaStream_t s);

struct AttnPrefillArgs {
  const float *qkv = nullptr;  // q rows at stride qkv_stride
  int64_t m = 0, qkv_stride = 0, start_pos = 0;
  int64_t n_heads_q = 0;
  KvView kv;
  int64_t layer = 0, window = 0;
  float scale = 1.f;
  float *out = nullptr;  // [m][n_heads_q*head_dim]
};
void launch_attn_prefill(const AttnPrefillArgs &a, cudaStream_t s);
// Reference-order prefill attention (xprefill.cu).
bool xattn_prefill_supported(int64_t head_dim, int64_t max_keys);
void launch_xattn_prefill(const AttnPrefillArgs &a, cudaStream_t s);

// Embedding row decode (repack_cache.rs:1166-1301 semantics) for tokens
// read from device memory.
void launch_embed(const uint8_t *emb_raw, int quant, int64_t hidden, int64_t vocab, const uint32_t *tokens,
                  int64_t m, float *out, int *err_flag, int pdl, cudaStream_t s);
// Greedy argmax over logits (lowest index wins ties); writes next token and
// advances the device position.
void launch_argmax(const float *logits, int64_t n, float *part_val, int *part_idx, unsigned *cnt, int n_blocks,
                   uint32_t *token_out, int64_t *d_pos, uint32_t *hist, int pdl, cudaStream_t s,
                   uint32_t *epoch = nullptr);  // += 1 per call when set (tensor-parallel exchange)

}  // namespace jal
