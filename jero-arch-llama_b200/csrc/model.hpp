// Host-side mirror of the reference's recipe / ModelRepackCache /
// ExecutionContext types, owning device memory and driving the kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "device.hpp"
#include "tp.hpp"
#include "gguf.hpp"
#include "jal.h"

namespace jal {

struct RopeScaling {  // RopeScalingConfig (recipe.rs:39-65)
  int kind = JAL_ROPE_SCALING_NONE;
  float factor = 1.f, low_freq_factor = 1.f, high_freq_factor = 4.f;
  uint64_t original_max_position_embeddings = 8192;
  std::vector<float> short_factor, long_factor;
};

struct Recipe {  // LlamaRecipe (recipe.rs:110-139)
  std::string architecture = "llama";
  uint64_t num_layers = 32, hidden_dim = 4096, ffn_dim = 14336, n_heads_q = 32, n_heads_kv = 8, head_dim = 128,
           vocab_size = 128256;
  float rms_eps = 1e-5f, rope_theta = 500000.f;
  int rope_type = JAL_ROPE_NORM;
  int64_t rotary_dim = -1;
  RopeScaling scaling;
  bool has_irope_mask = false;
  std::vector<uint8_t> irope_mask;

  static Recipe for_arch(const std::string &arch);
  static Recipe from_gguf(const GgufFile &g);
  bool should_skip_rope(size_t layer) const;
  bool supports_quant(int quant) const;
  void validate_model(const GgufFile &g) const;
};

// EffectiveGeometry (recipe.rs:147-158) resolved from resident tensors.
struct Geometry {
  uint64_t num_layers = 0, hidden_dim = 0, ffn_dim = 0, n_heads_q = 0, n_heads_kv = 0, head_dim = 0,
           rotary_dim = 0, total_q = 0, total_kv = 0;
};
Geometry resolve_geometry(const Recipe &r, const GgufFile &g);

struct DevBuffer {
  void *ptr = nullptr;
  size_t bytes = 0;
  DevBuffer() = default;
  explicit DevBuffer(size_t n);
  ~DevBuffer();
  DevBuffer(const DevBuffer &) = delete;
  DevBuffer &operator=(const DevBuffer &) = delete;
  template <class T> T *as() const { return (T *)ptr; }
};
using DevBufferPtr = std::shared_ptr<DevBuffer>;

// CachedMatrix (repack_cache.rs:1502-1788) on the device.
struct CachedMatrix {
  int quant = 0;
  uint64_t rows = 0, cols = 0;
  DevMat dm;
  std::vector<DevBufferPtr> storage;
  size_t aligned_bytes = 0;
};

// Repack `rows` GGUF rows of `raw` (device) into a new matrix.
CachedMatrix repack_matrix(const uint8_t *raw_dev, int quant, uint64_t rows, uint64_t cols, cudaStream_t s);
// Repack several same-quant, same-cols matrices into one stacked allocation;
// returns views for each part plus the stacked view.
void repack_stacked(const std::vector<const uint8_t *> &raws, const std::vector<uint64_t> &rows, int quant,
                    uint64_t cols, cudaStream_t s, std::vector<CachedMatrix> &parts, DevMat &stacked,
                    std::vector<DevBufferPtr> &storage);

struct Layer {  // LayerRepackCache (repack_cache.rs:2084-2111)
  DevBufferPtr norms;  // attn_norm | ffn_norm
  const float *attn_norm = nullptr, *ffn_norm = nullptr;
  DevBufferPtr biases;
  const float *bq = nullptr, *bk = nullptr, *bv = nullptr, *bo = nullptr;
  CachedMatrix wq, wk, wv, wo, wgate, wup, wdown;
  bool qkv_stacked = false, gateup_stacked = false;
  DevMat qkv, gateup;
  std::vector<DevBufferPtr> storage;
};

struct ModelCache {  // ModelRepackCache (repack_cache.rs:2129-2141)
  std::string architecture;
  int device = 0;
  Geometry geom;            // the model's geometry
  uint64_t vocab_size = 0;
  // Tensor parallelism (tp.hpp): this rank's shard.  Without it the plan is
  // rank 0 of 1 and the local geometry is the model's.
  const TpComm *tp = nullptr;  // not owned
  TpPlan plan;
  Geometry lgeom;           // heads, Q/K/V widths and FFN rows of this rank (hidden as geom)
  std::vector<Layer> layers;
  DevBufferPtr output_norm;
  CachedMatrix lm_head;
  DevBufferPtr emb_raw;  // token_embd in raw GGUF layout
  int emb_quant = 0;
  uint64_t emb_rows = 0;
  size_t norm_count = 0, bias_count = 0;
  size_t total_aligned_bytes() const;
};

std::unique_ptr<ModelCache> build_model_cache(const Recipe &r, const GgufFile &g, int device,
                                              const TpComm *tp = nullptr);

// KV storage for one model geometry (this rank's KV heads): the K and V
// page pools and the page table.  A context either owns one or runs over one
// that its caller allocated (the reference's caller-owned KvCacheView).
struct KvCache {
  KvView kv;
  uint64_t n_ctx = 0;
  int device = 0;
  std::vector<DevBufferPtr> bufs;
  size_t bytes() const;
};
std::unique_ptr<KvCache> create_kv_cache(const ModelCache &c, uint64_t n_ctx, int kv_f16, uint32_t page_size);

struct ContextConfig {
  uint64_t n_ctx = 4096;
  int kv_f16 = 1;
  uint32_t page_size = 64;
  uint64_t sliding_window = 0;
  bool use_graphs = true;
  uint64_t prefill_chunk = 2048;
  int numerics = JAL_NUMERICS_FAST;  // JAL_NUMERICS_REFERENCE: reference-order f32 (strict.cu)
};

struct Context {
  const ModelCache *cache = nullptr;
  Recipe recipe;
  ContextConfig cfg;
  Geometry g;
  cudaStream_t stream = nullptr;
  cudaStream_t own_stream = nullptr;
  uint64_t position = 0;
  // KV: a view of own_kv, or of a caller-owned cache
  KvView kv;
  std::unique_ptr<KvCache> own_kv;
  std::vector<DevBufferPtr> bufs;
  // device state
  int64_t *d_pos = nullptr;
  uint32_t *d_token = nullptr, *d_hist = nullptr;
  int *d_err = nullptr;
  float *cos_tab = nullptr, *sin_tab = nullptr, *cos_long = nullptr, *sin_long = nullptr;
  float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *attn_s = nullptr, *ffn = nullptr, *ffn_s = nullptr,
        *logits = nullptr, *am_val = nullptr;
  float *logits_local = nullptr;  // this rank's LM-head rows (== logits without tensor parallelism)
  // Tensor-parallel exchange over peer memory (decode step): symmetric
  // partial-sum slots [2 parity][world][hidden] of flagged 64-bit words;
  // d_xepoch counts the steps (the flags' epoch); hidden_b is the second
  // residual buffer (the combining prologues read one and write the other).
  // Null tp_sym: the step all-reduces through NCCL.
  std::unique_ptr<TpSymmetric> tp_sym;
  uint32_t *d_xepoch = nullptr;
  float *hidden_b = nullptr;
  int8_t *attn_q = nullptr, *ffn_q = nullptr;
  unsigned *ffn_cnt = nullptr, *am_cnt = nullptr;
  int *am_idx = nullptr;
  int n_splits = 1, am_blocks = 148;
  // Reference-order serving path (JAL_NUMERICS_FAST on one GPU): xgemv /
  // xattn kernels, x_splits CTAs per KV head in decode attention.
  bool exact = false;
  int x_splits = 0;
  // The score kernel's weights w_t = e_t / den, [n_heads_q][n_ctx], and the
  // 2D tensor map of the V plane the output kernel stages from.
  float *attn_w = nullptr;
  alignas(64) unsigned char tm_v[128] = {};
  // Test hook (jal_test.h): the decode attention's first V copy barrier
  // expects test_stall_tx bytes more than are sent, so its bounded wait
  // (test_wait_ns) runs out.
  uint32_t test_stall_tx = 0;
  uint64_t test_wait_ns = 0;
  // Step trace (jal_test.h): with trace_on, the reference-order step's
  // kernels record {start, end} of launch i in d_trace[2 i], [2 i + 1].
  bool trace_on = false;
  unsigned long long *d_trace = nullptr;
  DevBufferPtr trace_buf;
  // prefill scratch (grown on demand)
  uint64_t pf_cap = 0;
  DevBufferPtr pf_buf;
  uint32_t *pf_tokens = nullptr;
  float *pf_hidden = nullptr, *pf_qkv = nullptr, *pf_attn = nullptr, *pf_gu = nullptr,
        *pf_xs = nullptr;
  int8_t *pf_xq = nullptr;
  // batched decode scratch (batch_decode_step with this context first):
  // logits [bt_cap][vocab]
  uint64_t bt_cap = 0;
  DevBufferPtr bt_buf;
  float *bt_logits = nullptr;
  // one side stream per sequence for the attention kernels, which run
  // concurrently between the Q/K/V and O projections
  std::vector<cudaStream_t> bt_streams;
  std::vector<cudaEvent_t> bt_events;  // [0]: Q/K/V done; [1 + b]: sequence b's attention done
  int bt_splits = 0;                   // score-kernel cluster size in batched steps
  cudaGraphExec_t bt_graph = nullptr;  // the batched step of the contexts in bt_key
  std::vector<uint64_t> bt_key;        // {n, scratch generation, the contexts' ids}
  uint64_t uid = 0;                    // unique per context (graph keys)
  uint64_t pf_gen = 0;                 // bumped when the prefill scratch moves
  // host staging
  int64_t *h_pos = nullptr;
  uint32_t *h_token = nullptr;
  // reference-order decode scratch
  float *s_norm = nullptr, *s_sc = nullptr, *s_gu = nullptr, *s_qbuf = nullptr;
  int8_t *s_q8 = nullptr;
  // graph
  cudaGraphExec_t graph = nullptr;
  size_t launches_per_step = 0;
  // persistent decode step (decode_mega.cu), opt-in with JAL_DECODE=mega
  bool mega = false;
  int mega_grid = 0;
  MegaArgs margs;                         // host copy
  const MegaArgs *mega_dev_args = nullptr;  // device copy the kernel reads

  ~Context();
  void enqueue_decode_step(bool pdl);
  void enqueue_exact_step(bool pdl);
  // One token through the reference-order kernels; d_token / d_pos hold the
  // token and its position.  argmax advances d_pos like the fast step.
  void enqueue_strict_token(bool logits, bool argmax);
  void run_decode_step();
  void prefill(const uint32_t *tokens, uint64_t n, uint64_t start_pos, bool compute_logits);
  void ensure_prefill_capacity(uint64_t m);
};

// One decode step for n sequences at once, one context each (distinct KV
// caches, one model cache, reference-order numerics on one GPU): the
// projections run once over the n token rows (the reference-order GEMM), the
// attention per context at its own position.  Each sequence's logits equal
// its single-context decode step's.  Work goes on cs[0]'s stream (the
// attention on side streams joined back to it); d_pos of every context must
// hold its position; logits land in cs[0]->bt_logits.
void batch_decode_step(Context *const *cs, size_t n, const uint32_t *d_tokens);
// The batched step on cs[0]'s stream, replayed from a CUDA graph kept for
// this list of contexts (captured on first use); tokens in cs[0]->pf_tokens.
void run_batch_decode(Context *const *cs, size_t n);

// ext_kv: run over a caller-owned KV cache (must outlive the context);
// nullptr: the context allocates its own.
std::unique_ptr<Context> create_context(const Recipe &r, const ModelCache &c, const ContextConfig &cfg,
                                        const KvCache *ext_kv = nullptr);
size_t decode_scratch_bytes(const Recipe &r, uint64_t seq_len_upper_bound);

// f32 RoPE helpers shared with the op entry points (recipe.rs:2560-2660).
void fill_inv_freq(uint64_t rotary_dim, float theta, const RopeScaling &sc, uint64_t seq_len, float *out);

}  // namespace jal
