/*
 * jal_synth.h -- seeded synthetic GGUF v3 models and tensors.
 *
 * The reference has no random generator and no f32 -> Q4_0 quantizer; its
 * tests build GGUF byte buffers with jero_core::test_helpers (absent here).
 * These entry points write deterministic GGUF v3 files from a seed so the
 * oracle and the device path consume identical bytes.
 *
 * Values: SplitMix64 counters per tensor (keyed by the seed and the tensor
 * name) -> Box-Muller in double -> f32 * std.  Q4_0 / Q8_0 blocks follow the
 * public GGML reference quantizers; f16 scales use round-to-nearest-even.
 * Norm weights are 1.0.  Output is identical for any thread count.
 */
#ifndef JAL_SYNTH_H
#define JAL_SYNTH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct jal_synth_config {
  char architecture[16]; /* "llama", "llama4" or "qwen2" */
  uint64_t num_layers, hidden_dim, ffn_dim, n_heads_q, n_heads_kv, head_dim,
      vocab_size, context_length;
  float rms_eps, rope_theta;
  int32_t weight_quant; /* layer matrices: JAL_Q4_0 / JAL_Q8_0 / JAL_F32 */
  int32_t embed_quant;  /* token_embd.weight */
  int32_t head_quant;   /* output.weight; -1 = tied to token_embd */
  int32_t qkv_bias;     /* 1 = write attn_{q,k,v}.bias (F32) */
  float weight_std;     /* e.g. 0.02 */
  float bias_std;       /* e.g. 0.02 */
} jal_synth_config;

/* Total GGUF byte size for cfg. */
int jal_synth_gguf_size(const jal_synth_config *cfg, size_t *bytes);
/* Write the GGUF file into buf (len >= jal_synth_gguf_size). */
int jal_synth_gguf_write(const jal_synth_config *cfg, uint64_t seed, void *buf,
                         size_t len, int nthreads);
/* One rows x cols matrix in raw GGUF block order for `quant`, with values
 * N(0, std) keyed by (seed, name).  len >= rows * row_bytes. */
int jal_synth_matrix(int quant, size_t rows, size_t cols, uint64_t seed,
                     const char *name, float std_dev, void *out, size_t len,
                     int nthreads);
/* n f32 values N(0, std) keyed by (seed, name). */
int jal_synth_normal_f32(uint64_t seed, const char *name, size_t n,
                         float std_dev, float *out, int nthreads);
/* f32 -> f16 bits, round to nearest even. */
uint16_t jal_f32_to_f16_bits(float v);

#ifdef __cplusplus
}
#endif
#endif
