/*
 * CPU oracle for jero-arch-llama's quantized decode/prefill hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * A plain-C restatement of the reference crate's portable Rust path (built
 * without the `with-kernels` feature).  File:line citations refer to the
 * reference crate (src/repack_cache.rs, src/decode_gemv.rs, src/dispatch.rs,
 * src/recipe.rs).  Float evaluation order follows the Rust source exactly;
 * compile with -ffp-contract=off.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float f_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t *p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static inline float rdf32(const uint8_t *p) { uint32_t b = rd32(p); return f_from_bits(b); }
/* f32::max as used in the reference folds (operands are never NaN there). */
static inline float fmax_rs(float a, float b) { return a >= b ? a : b; }

/* repack_cache.rs:160-181 */
float or_f16_to_f32_finite(uint16_t bits) {
  uint32_t sign = (bits >> 15) & 1u, exp = (bits >> 10) & 0x1Fu, mant = bits & 0x3FFu;
  if (exp == 0) {
    if (mant == 0) return f_from_bits(sign << 31);
    uint32_t m = mant, e = 127u - 14u;
    while ((m & 0x400u) == 0) { m <<= 1; e -= 1; }
    m &= 0x3FFu;
    return f_from_bits((sign << 31) | (e << 23) | (m << 13));
  }
  if (exp == 31) return sign ? -0.0625f : 0.0625f;
  return f_from_bits((sign << 31) | ((exp + 127u - 15u) << 23) | (mant << 13));
}

/* repack_cache.rs:184-191 */
float or_bf16_to_f32_finite(uint16_t bits) {
  uint16_t exp = (bits >> 7) & 0xFF, sign = (bits >> 15) & 1;
  if (exp == 0xFF) return sign ? -0.0625f : 0.0625f;
  return f_from_bits((uint32_t)bits << 16);
}

/* repack_cache.rs:1028-1036 */
float or_sanitize_f32_weight(float v) {
  if (!isfinite(v)) return 0.0f;
  if (fabsf(v) > 1.0e6f) return (signbit(v) ? -1.0f : 1.0f) * 0.0625f;
  return v;
}

/* repack_cache.rs:1040-1061 */
int or_quant_block_geometry(int quant, size_t *elems, size_t *bytes) {
  size_t e = 0, b = 0;
  switch (quant) {
    case OR_F32: e = 1; b = 4; break;
    case OR_F16: case OR_BF16: e = 1; b = 2; break;
    case OR_Q8_0: e = 32; b = 34; break;
    case OR_Q4_0: e = 32; b = 18; break;
    case OR_Q5_0: e = 32; b = 22; break;
    case OR_Q4_K: e = 256; b = 144; break;
    case OR_Q5_K: e = 256; b = 176; break;
    case OR_Q6_K: e = 256; b = 210; break;
    default: return 0;
  }
  if (elems) *elems = e;
  if (bytes) *bytes = b;
  return 1;
}

/* repack_cache.rs:1065-1073 */
int or_quant_row_bytes(size_t cols, int quant, size_t *row_bytes) {
  size_t e, b;
  if (!or_quant_block_geometry(quant, &e, &b)) return 0;
  if (cols == 0 || cols % e != 0) return 0;
  *row_bytes = (cols / e) * b;
  return 1;
}

/* repack_cache.rs:1078-1085 (MAX_DENSE_F32_ELEMENTS / MAX_DENSE_HALF_ELEMENTS, :66-69) */
int or_is_oversized_dense(int quant, size_t rows, size_t cols) {
  size_t total = rows * cols;
  if (quant == OR_F32) return total > 8388608u;
  if (quant == OR_F16 || quant == OR_BF16) return total > 33554432u;
  return 0;
}

/* repack_cache.rs:194-206 */
static void unpack_q4_k_scales(const uint8_t *scales, uint8_t sc[8], uint8_t m[8]) {
  for (int j = 0; j < 4; j++) { sc[j] = scales[j] & 0x3F; m[j] = scales[j + 4] & 0x3F; }
  for (int j = 4; j < 8; j++) {
    sc[j] = (uint8_t)((scales[j + 4] & 0x0F) | ((scales[j - 4] >> 6) << 4));
    m[j] = (uint8_t)((scales[j + 4] >> 4) | ((scales[j] >> 6) << 4));
  }
}

/* repack_cache.rs:209-227 */
void or_dequantize_q4_0_block(const uint8_t *blk, float *out) {
  float d = or_f16_to_f32_finite(rd16(blk));
  if (d == 0.0f) { for (int i = 0; i < 32; i++) out[i] = 0.0f; return; }
  for (int i = 0; i < 16; i++) {
    uint8_t byte = blk[2 + i];
    int8_t q0 = (int8_t)((byte & 0x0F) - 8), q1 = (int8_t)(((byte >> 4) & 0x0F) - 8);
    out[i] = d * (float)q0;
    out[i + 16] = d * (float)q1;
  }
}

/* repack_cache.rs:231-257 */
void or_dequantize_q5_0_block(const uint8_t *blk, float *out) {
  float d = or_f16_to_f32_finite(rd16(blk));
  if (d == 0.0f) { for (int i = 0; i < 32; i++) out[i] = 0.0f; return; }
  uint32_t qh = rd32(blk + 2);
  for (int j = 0; j < 16; j++) {
    uint8_t packed = blk[6 + j];
    uint32_t xh0 = ((qh >> j) & 1u) << 4, xh1 = ((qh >> (j + 16)) & 1u) << 4;
    int8_t q0 = (int8_t)((int8_t)((packed & 0x0F) | xh0) - 16);
    int8_t q1 = (int8_t)((int8_t)((packed >> 4) | xh1) - 16);
    out[j] = d * (float)q0;
    out[j + 16] = d * (float)q1;
  }
}

/* repack_cache.rs:259-273 */
void or_dequantize_q8_0_block(const uint8_t *blk, float *out) {
  float d = or_f16_to_f32_finite(rd16(blk));
  if (d == 0.0f) { for (int i = 0; i < 32; i++) out[i] = 0.0f; return; }
  for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)blk[2 + i];
}

/* repack_cache.rs:275-293 */
void or_dequantize_q4_k_block(const uint8_t *blk, float *out) {
  float d = or_f16_to_f32_finite(rd16(blk)), dmin = or_f16_to_f32_finite(rd16(blk + 2));
  uint8_t sc[8], m[8];
  unpack_q4_k_scales(blk + 4, sc, m);
  const uint8_t *qs = blk + 16;
  for (int chunk = 0; chunk < 4; chunk++) {
    int is = chunk * 2;
    float d1 = d * (float)sc[is], m1 = dmin * (float)m[is];
    float d2 = d * (float)sc[is + 1], m2 = dmin * (float)m[is + 1];
    int out_idx = chunk * 64, q_off = chunk * 32;
    for (int l = 0; l < 32; l++) {
      out[out_idx + l] = d1 * (float)(qs[q_off + l] & 0x0F) - m1;
      out[out_idx + 32 + l] = d2 * (float)((qs[q_off + l] >> 4) & 0x0F) - m2;
    }
  }
}

/* repack_cache.rs:296-324 */
void or_dequantize_q5_k_block(const uint8_t *blk, float *out) {
  float d = or_f16_to_f32_finite(rd16(blk)), dmin = or_f16_to_f32_finite(rd16(blk + 2));
  if (d == 0.0f && dmin == 0.0f) { for (int i = 0; i < 256; i++) out[i] = 0.0f; return; }
  uint8_t sc[8], m[8];
  unpack_q4_k_scales(blk + 4, sc, m);
  const uint8_t *qh = blk + 16, *qs = blk + 48;
  uint8_t u1 = 1, u2 = 2;
  for (int chunk = 0; chunk < 4; chunk++) {
    int is = chunk * 2;
    float d1 = d * (float)sc[is], m1 = dmin * (float)m[is];
    float d2 = d * (float)sc[is + 1], m2 = dmin * (float)m[is + 1];
    int out_idx = chunk * 64, q_off = chunk * 32;
    for (int l = 0; l < 32; l++) {
      uint8_t hb1 = (qh[l] & u1) ? 16 : 0, hb2 = (qh[l] & u2) ? 16 : 0;
      out[out_idx + l] = d1 * (float)((uint8_t)((qs[q_off + l] & 0x0F) + hb1)) - m1;
      out[out_idx + 32 + l] = d2 * (float)((uint8_t)((qs[q_off + l] >> 4) + hb2)) - m2;
    }
    u1 = (uint8_t)(u1 << 2);
    u2 = (uint8_t)(u2 << 2);
  }
}

/* repack_cache.rs:326-370 */
void or_dequantize_q6_k_block(const uint8_t *blk, float *out) {
  float d = or_f16_to_f32_finite(rd16(blk + 208));
  if (d == 0.0f) { for (int i = 0; i < 256; i++) out[i] = 0.0f; return; }
  const uint8_t *ql = blk, *qh = blk + 128, *scales = blk + 192;
  for (int half = 0; half < 2; half++) {
    int n = half * 128, low = half * 64, high = half * 32, scb = half * 8;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      int8_t q1 = (int8_t)((int8_t)((ql[low + l] & 0x0F) | ((qh[high + l] & 0x03) << 4)) - 32);
      int8_t q2 = (int8_t)((int8_t)((ql[low + l + 32] & 0x0F) | (((qh[high + l] >> 2) & 0x03) << 4)) - 32);
      int8_t q3 = (int8_t)((int8_t)(((ql[low + l] >> 4) & 0x0F) | (((qh[high + l] >> 4) & 0x03) << 4)) - 32);
      int8_t q4 = (int8_t)((int8_t)(((ql[low + l + 32] >> 4) & 0x0F) | (((qh[high + l] >> 6) & 0x03) << 4)) - 32);
      float sc1 = (float)(int8_t)scales[scb + is], sc2 = (float)(int8_t)scales[scb + is + 2];
      float sc3 = (float)(int8_t)scales[scb + is + 4], sc4 = (float)(int8_t)scales[scb + is + 6];
      out[n + l] = d * sc1 * (float)q1;
      out[n + l + 32] = d * sc2 * (float)q2;
      out[n + l + 64] = d * sc3 * (float)q3;
      out[n + l + 96] = d * sc4 * (float)q4;
    }
  }
}

typedef void (*dequant_fn)(const uint8_t *, float *);

/* repack_cache.rs:1230-1242 */
static void decode_blocks_to_f32(const uint8_t *row_raw, size_t cols, size_t n, size_t b,
                                 float *out, dequant_fn f) {
  float buf[256];
  for (size_t bi = 0; bi < cols / n; bi++) {
    f(row_raw + bi * b, buf);
    memcpy(out + bi * n, buf, n * sizeof(float));
  }
}

/* repack_cache.rs:1244-1301 */
int or_decode_row_payload_to_f32(int quant, const uint8_t *row_raw, size_t cols, float *out,
                                 int sanitize_large) {
  switch (quant) {
    case OR_F32:
      for (size_t i = 0; i < cols; i++) {
        float v = rdf32(row_raw + i * 4);
        out[i] = sanitize_large ? or_sanitize_f32_weight(v) : (isfinite(v) ? v : 0.0f);
      }
      return OR_OK;
    case OR_F16:
      for (size_t i = 0; i < cols; i++) out[i] = or_f16_to_f32_finite(rd16(row_raw + i * 2));
      return OR_OK;
    case OR_BF16:
      for (size_t i = 0; i < cols; i++) out[i] = or_bf16_to_f32_finite(rd16(row_raw + i * 2));
      return OR_OK;
    case OR_Q8_0: decode_blocks_to_f32(row_raw, cols, 32, 34, out, or_dequantize_q8_0_block); return OR_OK;
    case OR_Q4_0: decode_blocks_to_f32(row_raw, cols, 32, 18, out, or_dequantize_q4_0_block); return OR_OK;
    case OR_Q5_0: decode_blocks_to_f32(row_raw, cols, 32, 22, out, or_dequantize_q5_0_block); return OR_OK;
    case OR_Q4_K: decode_blocks_to_f32(row_raw, cols, 256, 144, out, or_dequantize_q4_k_block); return OR_OK;
    case OR_Q5_K: decode_blocks_to_f32(row_raw, cols, 256, 176, out, or_dequantize_q5_k_block); return OR_OK;
    case OR_Q6_K: decode_blocks_to_f32(row_raw, cols, 256, 210, out, or_dequantize_q6_k_block); return OR_OK;
    default: return OR_ERR_CAPABILITY_MISMATCH;
  }
}

/* ---------------------------------------------------------------------- */
/* Portable RepackedWeight: repack_cache.rs:559-838                         */
/* ---------------------------------------------------------------------- */

/* repack_cache.rs:904-953 */
static void unpack_k_quants_row_i8(const uint8_t *row_raw, size_t cols, int is_q5_k, int8_t *out_q,
                                   float *out_scales, float *out_mins) {
  size_t blk_bytes = is_q5_k ? 176 : 144;
  for (size_t sb = 0; sb < cols / 256; sb++) {
    const uint8_t *blk = row_raw + sb * blk_bytes;
    float d = or_f16_to_f32_finite(rd16(blk)), dmin = or_f16_to_f32_finite(rd16(blk + 2));
    uint8_t sc[8], m[8];
    unpack_q4_k_scales(blk + 4, sc, m);
    for (int sub = 0; sub < 8; sub++) {
      out_scales[sb * 8 + sub] = d * (float)sc[sub];
      out_mins[sb * 8 + sub] = dmin * (float)m[sub];
    }
    const uint8_t *qs = is_q5_k ? blk + 48 : blk + 16;
    const uint8_t *qh = is_q5_k ? blk + 16 : NULL;
    uint8_t u1 = 1, u2 = 2;
    for (int chunk = 0; chunk < 4; chunk++) {
      size_t q_off = (size_t)chunk * 32, dst = sb * 256 + (size_t)chunk * 64;
      for (int l = 0; l < 32; l++) {
        uint8_t hb1 = 0, hb2 = 0;
        if (qh) { hb1 = (qh[l] & u1) ? 16 : 0; hb2 = (qh[l] & u2) ? 16 : 0; }
        out_q[dst + l] = (int8_t)(uint8_t)((qs[q_off + l] & 0x0F) + hb1);
        out_q[dst + 32 + l] = (int8_t)(uint8_t)((qs[q_off + l] >> 4) + hb2);
      }
      u1 = (uint8_t)(u1 << 2);
      u2 = (uint8_t)(u2 << 2);
    }
  }
}

/* repack_cache.rs:955-993 */
static void unpack_q6_k_row_i8(const uint8_t *row_raw, size_t cols, int8_t *out_q, float *out_scales) {
  for (size_t sb = 0; sb < cols / 256; sb++) {
    const uint8_t *blk = row_raw + sb * 210;
    float d = or_f16_to_f32_finite(rd16(blk + 208));
    const uint8_t *ql = blk, *qh = blk + 128, *scales = blk + 192;
    for (int sub = 0; sub < 16; sub++) out_scales[sb * 16 + sub] = d * (float)(int8_t)scales[sub];
    size_t base = sb * 256;
    for (int half = 0; half < 2; half++) {
      int n = half * 128, low = half * 64, high = half * 32;
      for (int l = 0; l < 32; l++) {
        out_q[base + n + l] = (int8_t)((int8_t)((ql[low + l] & 0x0F) | ((qh[high + l] & 0x03) << 4)) - 32);
        out_q[base + n + l + 32] =
            (int8_t)((int8_t)((ql[low + l + 32] & 0x0F) | (((qh[high + l] >> 2) & 0x03) << 4)) - 32);
        out_q[base + n + l + 64] =
            (int8_t)((int8_t)(((ql[low + l] >> 4) & 0x0F) | (((qh[high + l] >> 4) & 0x03) << 4)) - 32);
        out_q[base + n + l + 96] =
            (int8_t)((int8_t)(((ql[low + l + 32] >> 4) & 0x0F) | (((qh[high + l] >> 6) & 0x03) << 4)) - 32);
      }
    }
  }
}

/* repack_cache.rs:840-902 */
static void unpack_row_i8(const uint8_t *row_raw, size_t cols, int quant, int8_t *out_q,
                          float *out_scales, float *out_mins) {
  switch (quant) {
    case OR_Q8_0:
      for (size_t g = 0; g < cols / 32; g++) {
        const uint8_t *blk = row_raw + g * 34;
        out_scales[g] = or_f16_to_f32_finite(rd16(blk));
        for (int k = 0; k < 32; k++) out_q[g * 32 + k] = (int8_t)blk[2 + k];
      }
      break;
    case OR_Q4_0:
      for (size_t g = 0; g < cols / 32; g++) {
        const uint8_t *blk = row_raw + g * 18;
        out_scales[g] = or_f16_to_f32_finite(rd16(blk));
        for (int i = 0; i < 16; i++) {
          uint8_t byte = blk[2 + i];
          out_q[g * 32 + i] = (int8_t)((byte & 0x0F) - 8);
          out_q[g * 32 + 16 + i] = (int8_t)(((byte >> 4) & 0x0F) - 8);
        }
      }
      break;
    case OR_Q5_0:
      for (size_t g = 0; g < cols / 32; g++) {
        const uint8_t *blk = row_raw + g * 22;
        out_scales[g] = or_f16_to_f32_finite(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        for (int j = 0; j < 16; j++) {
          uint8_t packed = blk[6 + j];
          uint32_t xh0 = ((qh >> j) & 1u) << 4, xh1 = ((qh >> (j + 16)) & 1u) << 4;
          out_q[g * 32 + j] = (int8_t)((int8_t)((packed & 0x0F) | xh0) - 16);
          out_q[g * 32 + 16 + j] = (int8_t)((int8_t)((packed >> 4) | xh1) - 16);
        }
      }
      break;
    case OR_Q4_K: case OR_Q5_K:
      unpack_k_quants_row_i8(row_raw, cols, quant == OR_Q5_K, out_q, out_scales, out_mins);
      break;
    case OR_Q6_K: unpack_q6_k_row_i8(row_raw, cols, out_q, out_scales); break;
    default: break;
  }
}

/* repack_cache.rs:566-694 (from_tensor_with_half_limit, repack_dense, repack_quantized) */
int or_repack(const uint8_t *raw, size_t raw_len, int quant, size_t rows, size_t cols, or_repacked *out) {
  memset(out, 0, sizeof(*out));
  size_t row_bytes;
  if (!or_quant_block_geometry(quant, NULL, NULL)) return OR_ERR_CAPABILITY_MISMATCH;
  if (!or_quant_row_bytes(cols, quant, &row_bytes)) return OR_ERR_TENSOR_BOUNDS;
  if (rows == 0 || raw_len < rows * row_bytes) return OR_ERR_TENSOR_BOUNDS;
  out->rows = rows; out->cols = cols; out->quant = quant;
  if (quant == OR_F32 || quant == OR_F16 || quant == OR_BF16) {
    out->dense = 1;
    out->blocks_per_row = (cols + 31) / 32;
    out->dense_data = (float *)calloc(rows * out->blocks_per_row * 32, sizeof(float));
    for (size_t r = 0; r < rows; r++)
      or_decode_row_payload_to_f32(quant, raw + r * row_bytes, cols,
                                   out->dense_data + r * out->blocks_per_row * 32, 1);
    return OR_OK;
  }
  size_t group = quant == OR_Q6_K ? 16 : 32;
  out->scale_groups = cols / group;
  out->k_chunks = cols / 16;
  out->chunks_per_scale = group / 16;
  out->n_tiles = (rows + 7) / 8;
  out->tiles = (int8_t *)calloc(out->n_tiles * out->k_chunks * 128, 1);
  out->scales = (float *)calloc(out->n_tiles * out->scale_groups * 8, sizeof(float));
  int has_mins = quant == OR_Q4_K || quant == OR_Q5_K;
  if (has_mins) out->mins = (float *)calloc(out->n_tiles * out->scale_groups * 8, sizeof(float));
  int8_t *row_q = (int8_t *)calloc(cols, 1);
  float *row_sc = (float *)calloc(out->scale_groups, sizeof(float));
  float *row_mn = (float *)calloc(out->scale_groups, sizeof(float));
  for (size_t r = 0; r < rows; r++) {
    memset(row_mn, 0, out->scale_groups * sizeof(float));
    unpack_row_i8(raw + r * row_bytes, cols, quant, row_q, row_sc, row_mn);
    size_t nt = r / 8, j = r % 8;
    for (size_t g = 0; g < out->scale_groups; g++) {
      out->scales[(nt * out->scale_groups + g) * 8 + j] = row_sc[g];
      if (has_mins) out->mins[(nt * out->scale_groups + g) * 8 + j] = row_mn[g];
    }
    for (size_t ch = 0; ch < out->k_chunks; ch++)
      memcpy(out->tiles + (nt * out->k_chunks + ch) * 128 + j * 16, row_q + ch * 16, 16);
  }
  free(row_q); free(row_sc); free(row_mn);
  return OR_OK;
}

void or_repacked_free(or_repacked *w) {
  free(w->dense_data); free(w->tiles); free(w->scales); free(w->mins);
  memset(w, 0, sizeof(*w));
}

/* repack_cache.rs:390-422 (quantize_single_row_slices) */
static void quantize_single_row(const float *src, size_t k, size_t blocks, float *dst_f32,
                                int8_t *dst_q8, float *dst_scales) {
  for (size_t i = 0; i < k; i++) dst_f32[i] = isfinite(src[i]) ? src[i] : 0.0f;
  for (size_t b = 0; b < blocks; b++) {
    size_t c0 = b * 32, c1 = c0 + 32 < k ? c0 + 32 : k;
    float amax = 0.0f;
    for (size_t c = c0; c < c1; c++) amax = fmax_rs(amax, fabsf(dst_f32[c]));
    float scale = amax > 0.0f ? amax / 127.0f : 0.0f;
    float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
    for (size_t c = c0; c < c1; c++) {
      float q = roundf(dst_f32[c] * inv);
      if (q < -127.0f) q = -127.0f;
      if (q > 127.0f) q = 127.0f;
      dst_q8[c] = (int8_t)q;
    }
    dst_scales[b] = scale;
  }
}

/* repack_cache.rs:491-531 (QuantizedActQ8::quantize_into; buffers are zeroed first) */
void or_quantize_act_rows(const float *act, size_t m, size_t k, float *f32_rows, int8_t *q8,
                          float *scales) {
  size_t blocks = (k + 31) / 32, kp = blocks * 32;
  memset(f32_rows, 0, m * kp * sizeof(float));
  memset(q8, 0, m * kp);
  memset(scales, 0, m * blocks * sizeof(float));
  for (size_t t = 0; t < m; t++)
    quantize_single_row(act + t * k, k, blocks, f32_rows + t * kp, q8 + t * kp, scales + t * blocks);
}

/* repack_cache.rs:715-785 */
void or_eval_row_range(const or_repacked *w, float *out_row, const float *a_f32, const int8_t *a_q8,
                       const float *a_sc, size_t r0, size_t r1) {
  if (w->dense) {
    for (size_t r = r0; r < r1; r++) {
      const float *w_row = w->dense_data + r * w->blocks_per_row * 32;
      float acc = 0.0f;
      for (size_t c = 0; c < w->cols; c++) acc += w_row[c] * a_f32[c];
      out_row[r - r0] = acc;
    }
    return;
  }
  size_t group_elems = w->chunks_per_scale * 16;
  for (size_t r = r0; r < r1; r++) {
    size_t nt = r / 8, j = r % 8;
    float acc = 0.0f;
    for (size_t ch = 0; ch < w->k_chunks; ch++) {
      size_t sg = ch / w->chunks_per_scale, b32 = ch / 2;
      float w_sc = w->scales[(nt * w->scale_groups + sg) * 8 + j];
      const int8_t *bj = w->tiles + (nt * w->k_chunks + ch) * 128 + j * 16;
      const int8_t *ai = a_q8 + ch * 16;
      int32_t dot = 0;
      for (int i = 0; i < 16; i++) dot += (int32_t)ai[i] * (int32_t)bj[i];
      float dot_f = (float)dot;
      acc += dot_f * a_sc[b32] * w_sc;
      if (ch % w->chunks_per_scale == 0 && w->mins) {
        float w_mn = w->mins[(nt * w->scale_groups + sg) * 8 + j];
        float x_sum = 0.0f;
        for (size_t e = sg * group_elems; e < (sg + 1) * group_elems; e++) x_sum += a_f32[e];
        acc -= x_sum * w_mn;
      }
    }
    out_row[r - r0] = acc;
  }
}

void or_dot16_partials(const or_repacked *w, const int8_t *a_q8, size_t r0, size_t r1, int32_t *out) {
  for (size_t r = r0; r < r1; r++) {
    size_t nt = r / 8, j = r % 8;
    for (size_t ch = 0; ch < w->k_chunks; ch++) {
      const int8_t *bj = w->tiles + (nt * w->k_chunks + ch) * 128 + j * 16;
      const int8_t *ai = a_q8 + ch * 16;
      int32_t dot = 0;
      for (int i = 0; i < 16; i++) dot += (int32_t)ai[i] * (int32_t)bj[i];
      out[(r - r0) * w->k_chunks + ch] = dot;
    }
  }
}

/* repack_cache.rs:808-837 (gemm_rows) driven by 64-row panels as in
 * run_repacked_gemm_panels (repack_cache.rs:1931-1972); results per row do not
 * depend on the panel split. */
int or_project_batch(const or_repacked *w, float *out, const float *act, size_t m, int nthreads) {
  if (m == 0) return OR_OK;
  size_t k = w->cols, blocks = (k + 31) / 32, kp = blocks * 32;
  float *f32_rows = (float *)malloc(m * kp * sizeof(float));
  int8_t *q8 = (int8_t *)malloc(m * kp);
  float *sc = (float *)malloc(m * blocks * sizeof(float));
  or_quantize_act_rows(act, m, k, f32_rows, q8, sc);
  size_t rows = w->rows, panels = (rows + 63) / 64;
  (void)nthreads;
#pragma omp parallel for schedule(dynamic) num_threads(nthreads > 0 ? nthreads : 1) if (nthreads > 1)
  for (size_t p = 0; p < panels; p++) {
    size_t r0 = p * 64, r1 = r0 + 64 < rows ? r0 + 64 : rows;
    float tmp[64];
    for (size_t t = 0; t < m; t++) {
      or_eval_row_range(w, tmp, f32_rows + t * kp, q8 + t * kp, sc + t * blocks, r0, r1);
      memcpy(out + t * rows + r0, tmp, (r1 - r0) * sizeof(float));
    }
  }
  free(f32_rows); free(q8); free(sc);
  return OR_OK;
}

/* ---------------------------------------------------------------------- */
/* Streaming raw-GGUF GEMV: decode_gemv.rs:168-891, 1289-1407               */
/* ---------------------------------------------------------------------- */

/* decode_gemv.rs:251-257 */
static int8_t round_scaled_to_i8(float v, float inv) {
  if (!isfinite(v)) return 0;
  float q = roundf(v * inv);
  if (q < -127.0f) q = -127.0f;
  if (q > 127.0f) q = 127.0f;
  return (int8_t)q;
}

/* decode_gemv.rs:294-313 */
int or_quantize_row_q8_0(const float *x, size_t n, or_block_q8_0 *out) {
  if (n == 0 || n % 32 != 0) return OR_ERR_TENSOR_BOUNDS;
  for (size_t b = 0; b < n / 32; b++) {
    const float *c = x + b * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) if (isfinite(c[i])) amax = fmax_rs(amax, fabsf(c[i]));
    if (amax == 0.0f || !isfinite(amax)) { memset(&out[b], 0, sizeof(out[b])); continue; }
    out[b].d = amax / 127.0f;
    float inv = 127.0f / amax;
    for (int i = 0; i < 32; i++) out[b].qs[i] = round_scaled_to_i8(c[i], inv);
  }
  return OR_OK;
}

/* decode_gemv.rs:320-346 */
int or_quantize_row_q8_k(const float *x, size_t n, or_block_q8_k *out) {
  if (n == 0 || n % 256 != 0) return OR_ERR_TENSOR_BOUNDS;
  for (size_t b = 0; b < n / 256; b++) {
    const float *c = x + b * 256;
    float amax = 0.0f;
    for (int i = 0; i < 256; i++) if (isfinite(c[i])) amax = fmax_rs(amax, fabsf(c[i]));
    if (amax == 0.0f || !isfinite(amax)) { memset(&out[b], 0, sizeof(out[b])); continue; }
    out[b].d = amax / 127.0f;
    float inv = 127.0f / amax;
    for (int s = 0; s < 16; s++) {
      int16_t bsum = 0;
      for (int j = 0; j < 16; j++) {
        int8_t q = round_scaled_to_i8(c[s * 16 + j], inv);
        out[b].qs[s * 16 + j] = q;
        bsum = (int16_t)(bsum + q);
      }
      out[b].bsums[s] = bsum;
    }
  }
  return OR_OK;
}

/* decode_gemv.rs:394-407 */
static float dot_q4_0_q8_0_blk(const uint8_t *w, const or_block_q8_0 *x) {
  float dw = or_f16_to_f32_finite(rd16(w));
  if (dw == 0.0f || x->d == 0.0f) return 0.0f;
  int32_t sumi = 0;
  for (int i = 0; i < 16; i++) {
    uint8_t byte = w[2 + i];
    int32_t q0 = (int32_t)(byte & 0x0F) - 8, q1 = (int32_t)((byte >> 4) & 0x0F) - 8;
    sumi += q0 * x->qs[i] + q1 * x->qs[i + 16];
  }
  return (float)sumi * (dw * x->d);
}

/* decode_gemv.rs:409-425 */
static float dot_q5_0_q8_0_blk(const uint8_t *w, const or_block_q8_0 *x) {
  float dw = or_f16_to_f32_finite(rd16(w));
  if (dw == 0.0f || x->d == 0.0f) return 0.0f;
  uint32_t qh = rd32(w + 2);
  int32_t sumi = 0;
  for (int j = 0; j < 16; j++) {
    uint8_t byte = w[6 + j];
    int32_t h0 = (int32_t)(((qh >> j) & 1u) << 4), h1 = (int32_t)(((qh >> (j + 16)) & 1u) << 4);
    int32_t q0 = ((int32_t)(byte & 0x0F) | h0) - 16, q1 = ((int32_t)((byte >> 4) & 0x0F) | h1) - 16;
    sumi += q0 * x->qs[j] + q1 * x->qs[j + 16];
  }
  return (float)sumi * (dw * x->d);
}

/* decode_gemv.rs:427-439 */
static float dot_q8_0_q8_0_blk(const uint8_t *w, const or_block_q8_0 *x) {
  float dw = or_f16_to_f32_finite(rd16(w));
  if (dw == 0.0f || x->d == 0.0f) return 0.0f;
  int32_t sumi = 0;
  for (int i = 0; i < 32; i++) sumi += (int32_t)(int8_t)w[2 + i] * x->qs[i];
  return (float)sumi * (dw * x->d);
}

/* decode_gemv.rs:456-523 (Q4_K and Q5_K share the body) */
static float dot_q45_k_q8_k_blk(const uint8_t *w, const or_block_q8_k *x, int q5) {
  float d = or_f16_to_f32_finite(rd16(w)), dmin = or_f16_to_f32_finite(rd16(w + 2));
  if ((d == 0.0f && dmin == 0.0f) || x->d == 0.0f) return 0.0f;
  uint8_t sc[8], mins[8];
  unpack_q4_k_scales(w + 4, sc, mins);
  const uint8_t *qh = q5 ? w + 16 : NULL, *qs = q5 ? w + 48 : w + 16;
  int32_t sumi = 0, sum_mins = 0;
  for (int chunk = 0; chunk < 4; chunk++) {
    int is = chunk * 2;
    uint8_t u1 = (uint8_t)(1u << (chunk * 2)), u2 = (uint8_t)(2u << (chunk * 2));
    const uint8_t *q_sub = qs + chunk * 32;
    const int8_t *x_lo = x->qs + chunk * 64, *x_hi = x->qs + chunk * 64 + 32;
    int32_t s_lo = 0, s_hi = 0;
    for (int l = 0; l < 32; l++) {
      uint8_t b = q_sub[l];
      int32_t hb1 = 0, hb2 = 0;
      if (qh) { hb1 = (qh[l] & u1) ? 16 : 0; hb2 = (qh[l] & u2) ? 16 : 0; }
      s_lo += ((int32_t)(b & 0x0F) | hb1) * x_lo[l];
      s_hi += ((int32_t)(b >> 4) | hb2) * x_hi[l];
    }
    sumi += (int32_t)sc[is] * s_lo + (int32_t)sc[is + 1] * s_hi;
    int32_t bsum_lo = (int32_t)x->bsums[chunk * 4] + x->bsums[chunk * 4 + 1];
    int32_t bsum_hi = (int32_t)x->bsums[chunk * 4 + 2] + x->bsums[chunk * 4 + 3];
    sum_mins += (int32_t)mins[is] * bsum_lo + (int32_t)mins[is + 1] * bsum_hi;
  }
  return (d * x->d) * (float)sumi - (dmin * x->d) * (float)sum_mins;
}

/* decode_gemv.rs:525-564 */
static float dot_q6_k_q8_k_blk(const uint8_t *w, const or_block_q8_k *x) {
  float d = or_f16_to_f32_finite(rd16(w + 208));
  if (d == 0.0f || x->d == 0.0f) return 0.0f;
  const uint8_t *ql = w, *qh = w + 128, *scales = w + 192;
  int32_t sumi = 0;
  for (int half = 0; half < 2; half++) {
    int n = half * 128, qlo = half * 64, qhi = half * 32, scb = half * 8;
    for (int is = 0; is < 2; is++) {
      int lb = is * 16;
      int32_t sc1 = (int8_t)scales[scb + is], sc2 = (int8_t)scales[scb + is + 2];
      int32_t sc3 = (int8_t)scales[scb + is + 4], sc4 = (int8_t)scales[scb + is + 6];
      int32_t s1 = 0, s2 = 0, s3 = 0, s4 = 0;
      for (int l = lb; l < lb + 16; l++) {
        uint8_t b_lo = ql[qlo + l], b_hi = ql[qlo + l + 32], hb = qh[qhi + l];
        int32_t q1 = ((int32_t)(b_lo & 0x0F) | ((int32_t)(hb & 0x03) << 4)) - 32;
        int32_t q2 = ((int32_t)(b_hi & 0x0F) | ((int32_t)((hb >> 2) & 0x03) << 4)) - 32;
        int32_t q3 = ((int32_t)(b_lo >> 4) | ((int32_t)((hb >> 4) & 0x03) << 4)) - 32;
        int32_t q4 = ((int32_t)(b_hi >> 4) | ((int32_t)((hb >> 6) & 0x03) << 4)) - 32;
        s1 += q1 * x->qs[n + l];
        s2 += q2 * x->qs[n + l + 32];
        s3 += q3 * x->qs[n + l + 64];
        s4 += q4 * x->qs[n + l + 96];
      }
      sumi += sc1 * s1 + sc2 * s2 + sc3 * s3 + sc4 * s4;
    }
  }
  return (d * x->d) * (float)sumi;
}

/* decode_gemv.rs:566-603 */
static float dot_tq1_0_q8_k_blk(const uint8_t *w, const or_block_q8_k *x) {
  float d = or_f16_to_f32_finite(rd16(w));
  if (d == 0.0f || x->d == 0.0f) return 0.0f;
  int32_t sumi = 0;
  for (int i = 0; i < 51; i++) {
    unsigned cur = w[2 + i];
    for (int j = 0; j < 5; j++) {
      int32_t trit = (int32_t)(cur % 3) - 1;
      sumi += trit * x->qs[i * 5 + j];
      cur /= 3;
    }
  }
  sumi += ((int32_t)(w[53] % 3) - 1) * x->qs[255];
  return (float)sumi * (d * x->d);
}

/* decode_gemv.rs:605-620 */
static float dot_tq2_0_q8_k_blk(const uint8_t *w, const or_block_q8_k *x) {
  float d = or_bf16_to_f32_finite(rd16(w + 64));
  if (d == 0.0f || x->d == 0.0f) return 0.0f;
  int32_t sumi = 0;
  for (int i = 0; i < 64; i++)
    for (int sub = 0; sub < 4; sub++) sumi += ((int32_t)((w[i] >> (sub * 2)) & 0x03) - 1) * x->qs[i * 4 + sub];
  return (float)sumi * (d * x->d);
}

/* decode_gemv.rs:1155-1166 and the Rust f32 Sum fold (start -0.0) */
static float dot_f32_sum(const float *a, const float *b, size_t n) {
  float s = -0.0f;
  for (size_t i = 0; i < n; i++) s += a[i] * b[i];
  return s;
}

/* decode_gemv.rs:1081-1153 */
static float dot_dense_row_zero_alloc(int quant, const uint8_t *row, const float *x, size_t cols) {
  float buf[256], act[256], sum = 0.0f;
  for (size_t col = 0; col < cols;) {
    size_t n = cols - col < 256 ? cols - col : 256;
    for (size_t i = 0; i < n; i++) {
      if (quant == OR_F32) buf[i] = or_sanitize_f32_weight(rdf32(row + (col + i) * 4));
      else if (quant == OR_BF16) buf[i] = or_bf16_to_f32_finite(rd16(row + (col + i) * 2));
      else buf[i] = or_f16_to_f32_finite(rd16(row + (col + i) * 2));
    }
    int all_finite = 1;
    for (size_t i = 0; i < n; i++) if (!isfinite(x[col + i])) { all_finite = 0; break; }
    float term;
    if (all_finite) term = dot_f32_sum(buf, x + col, n);
    else {
      for (size_t i = 0; i < n; i++) act[i] = isfinite(x[col + i]) ? x[col + i] : 0.0f;
      term = dot_f32_sum(buf, act, n);
    }
    if (isfinite(term)) sum += term;
    col += n;
  }
  return sum;
}

/* dispatch.rs:79-105 */
static float block_dequant_dot(size_t row, size_t cols, size_t n, size_t b, const uint8_t *raw,
                               size_t raw_len, const float *hidden, dequant_fn f) {
  size_t bpr = cols / n, row_off = row * bpr * b;
  float sum = 0.0f, buf[256];
  for (size_t bi = 0; bi < bpr; bi++) {
    size_t off = row_off + bi * b;
    if (off + b > raw_len) continue;
    f(raw + off, buf);
    for (size_t k = 0; k < n; k++) sum += buf[k] * hidden[bi * n + k];
  }
  return sum;
}

/* dispatch.rs:107-177 */
float or_compute_row_dot(size_t row, size_t cols, int quant, const uint8_t *raw, size_t raw_len,
                         const float *hidden) {
  float sum = 0.0f;
  switch (quant) {
    case OR_F32:
      for (size_t i = 0; i < cols; i++) {
        size_t off = row * cols * 4 + i * 4;
        if (off + 4 <= raw_len) sum += or_sanitize_f32_weight(rdf32(raw + off)) * hidden[i];
      }
      return sum;
    case OR_F16: case OR_BF16:
      for (size_t i = 0; i < cols; i++) {
        size_t off = row * cols * 2 + i * 2;
        if (off + 2 <= raw_len) {
          uint16_t bits = rd16(raw + off);
          float v = quant == OR_BF16 ? or_bf16_to_f32_finite(bits) : or_f16_to_f32_finite(bits);
          sum += v * hidden[i];
        }
      }
      return sum;
    case OR_Q8_0: return block_dequant_dot(row, cols, 32, 34, raw, raw_len, hidden, or_dequantize_q8_0_block);
    case OR_Q4_0: return block_dequant_dot(row, cols, 32, 18, raw, raw_len, hidden, or_dequantize_q4_0_block);
    case OR_Q5_0: return block_dequant_dot(row, cols, 32, 22, raw, raw_len, hidden, or_dequantize_q5_0_block);
    case OR_Q4_K: return block_dequant_dot(row, cols, 256, 144, raw, raw_len, hidden, or_dequantize_q4_k_block);
    case OR_Q5_K: return block_dequant_dot(row, cols, 256, 176, raw, raw_len, hidden, or_dequantize_q5_k_block);
    case OR_Q6_K: return block_dequant_dot(row, cols, 256, 210, raw, raw_len, hidden, or_dequantize_q6_k_block);
    default: return 0.0f;
  }
}

/* decode_gemv.rs:1289-1388 (gemv_decode_projection_with_workers).  Each row is
 * evaluated by run_gemv (decode_gemv.rs:622-642), independent of the split. */
int or_gemv_decode_projection(const uint8_t *raw, size_t raw_len, int quant, size_t rows,
                              size_t cols, const float *x, float *out, int nthreads) {
  size_t blk_e = 0, blk_b = 0;
  switch (quant) {
    case OR_F32: case OR_F16: case OR_BF16: case OR_Q4_0: case OR_Q5_0: case OR_Q8_0:
    case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: case OR_TQ1_0: case OR_TQ2_0: break;
    default: return OR_ERR_CAPABILITY_MISMATCH;
  }
  if (rows == 0) return OR_OK;
  if (quant == OR_TQ1_0) { blk_e = 256; blk_b = 54; }
  else if (quant == OR_TQ2_0) { blk_e = 256; blk_b = 66; }
  else or_quant_block_geometry(quant, &blk_e, &blk_b);
  if (cols == 0 || cols % blk_e != 0) return OR_ERR_TENSOR_BOUNDS;
  size_t stride = (cols / blk_e) * blk_b;
  if (raw_len < rows * stride) return OR_ERR_TENSOR_BOUNDS;
  (void)nthreads;
  if (quant == OR_Q4_0 || quant == OR_Q5_0 || quant == OR_Q8_0) {
    size_t nb = cols / 32;
    or_block_q8_0 *xb = (or_block_q8_0 *)calloc(nb, sizeof(or_block_q8_0));
    or_quantize_row_q8_0(x, cols, xb);
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1) if (nthreads > 1)
    for (size_t r = 0; r < rows; r++) {
      const uint8_t *row = raw + r * stride;
      float acc = 0.0f;
      for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * blk_b;
        float t = quant == OR_Q4_0 ? dot_q4_0_q8_0_blk(blk, &xb[b])
                  : quant == OR_Q5_0 ? dot_q5_0_q8_0_blk(blk, &xb[b]) : dot_q8_0_q8_0_blk(blk, &xb[b]);
        acc += t;
      }
      out[r] = acc;
    }
    free(xb);
    return OR_OK;
  }
  if (quant == OR_Q4_K || quant == OR_Q5_K || quant == OR_Q6_K || quant == OR_TQ1_0 || quant == OR_TQ2_0) {
    size_t nb = cols / 256;
    or_block_q8_k *xb = (or_block_q8_k *)calloc(nb, sizeof(or_block_q8_k));
    or_quantize_row_q8_k(x, cols, xb);
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1) if (nthreads > 1)
    for (size_t r = 0; r < rows; r++) {
      const uint8_t *row = raw + r * stride;
      float acc = 0.0f;
      for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * blk_b;
        float t;
        switch (quant) {
          case OR_Q4_K: t = dot_q45_k_q8_k_blk(blk, &xb[b], 0); break;
          case OR_Q5_K: t = dot_q45_k_q8_k_blk(blk, &xb[b], 1); break;
          case OR_Q6_K: t = dot_q6_k_q8_k_blk(blk, &xb[b]); break;
          case OR_TQ1_0: t = dot_tq1_0_q8_k_blk(blk, &xb[b]); break;
          default: t = dot_tq2_0_q8_k_blk(blk, &xb[b]); break;
        }
        acc += t;
      }
      out[r] = acc;
    }
    free(xb);
    return OR_OK;
  }
  for (size_t r = 0; r < rows; r++) out[r] = dot_dense_row_zero_alloc(quant, raw + r * stride, x, cols);
  return OR_OK;
}

/* ---------------------------------------------------------------------- */
/* Elementwise / attention ops: recipe.rs:2534-3050                         */
/* ---------------------------------------------------------------------- */

/* recipe.rs:2534-2558 */
int or_rmsnorm_row(float *out, const float *in, const float *w, size_t n, float eps) {
  if (n == 0) return OR_ERR_TENSOR_BOUNDS;
  float sum_sq = -0.0f;
  for (size_t i = 0; i < n; i++) sum_sq += in[i] * in[i];
  float inv = 1.0f / sqrtf(sum_sq / (float)n + eps);
  for (size_t i = 0; i < n; i++) out[i] = in[i] * inv * w[i];
  return OR_OK;
}

/* recipe.rs:2560-2660 */
int or_fill_inv_freq(size_t head_dim, float theta, const or_rope_scaling *sc, size_t seq_len, float *out) {
  if (head_dim == 0 || head_dim % 2 != 0 || !isfinite(theta) || theta <= 0.0f) return OR_ERR_CAPABILITY_MISMATCH;
  size_t half = head_dim / 2;
  float hd = (float)head_dim;
  for (size_t i = 0; i < half; i++) {
    float e = (float)(2 * i) / hd;
    out[i] = 1.0f / powf(theta, e);
  }
  if (!sc || sc->kind == 0) return OR_OK;
  if (sc->kind == 1) {
    if (!isfinite(sc->factor) || sc->factor <= 0.0f) return OR_ERR_CAPABILITY_MISMATCH;
    for (size_t i = 0; i < half; i++) out[i] /= sc->factor;
    return OR_OK;
  }
  if (sc->kind == 2) {
    float factor = sc->factor, lo = sc->low_freq_factor, hi = sc->high_freq_factor;
    if (!isfinite(factor) || factor <= 0.0f || !isfinite(lo) || lo <= 0.0f || !isfinite(hi) || hi <= lo ||
        sc->original_max_position_embeddings == 0)
      return OR_ERR_CAPABILITY_MISMATCH;
    float orig = (float)sc->original_max_position_embeddings;
    float low_wl = orig / lo, high_wl = orig / hi;
    for (size_t i = 0; i < half; i++) {
      float freq = out[i];
      float wavelen = 6.28318530717958647692f / freq;
      if (wavelen > low_wl) out[i] = freq / factor;
      else if (wavelen >= high_wl) {
        float smooth = (orig / wavelen - lo) / (hi - lo);
        out[i] = (1.0f - smooth) * (freq / factor) + smooth * freq;
      }
    }
    return OR_OK;
  }
  if (sc->kind == 3) {
    const float *f = seq_len > sc->original_max_position_embeddings ? sc->long_factor : sc->short_factor;
    if (sc->n_factors != half || !f) return OR_ERR_CAPABILITY_MISMATCH;
    for (size_t i = 0; i < half; i++) if (!isfinite(f[i]) || f[i] <= 0.0f) return OR_ERR_CAPABILITY_MISMATCH;
    for (size_t i = 0; i < half; i++) out[i] /= f[i];
    return OR_OK;
  }
  return OR_ERR_CAPABILITY_MISMATCH;
}

/* recipe.rs:2680-2715 */
int or_rope_cos_sin(size_t pos, size_t rotary_dim, const float *inv_freq, float *c, float *s) {
  if (rotary_dim < 2 || rotary_dim % 2 != 0) return OR_ERR_CAPABILITY_MISMATCH;
  float p = (float)pos;
  for (size_t i = 0; i < rotary_dim / 2; i++) {
    float a = p * inv_freq[i];
    s[i] = sinf(a);
    c[i] = cosf(a);
  }
  return OR_OK;
}

static void rotate_head(float *head, size_t half, int neox, const float *c, const float *s) {
  for (size_t i = 0; i < half; i++) {
    size_t i0 = neox ? i : 2 * i, i1 = neox ? i + half : 2 * i + 1;
    float x0 = head[i0], x1 = head[i1];
    head[i0] = x0 * c[i] - x1 * s[i];
    head[i1] = x0 * s[i] + x1 * c[i];
  }
}

/* recipe.rs:2717-2773 */
int or_apply_rope_cos_sin(float *qk, size_t len, size_t head_dim, size_t rotary_dim, int neox,
                          const float *c, const float *s) {
  if (head_dim < 2 || head_dim % 2 || rotary_dim < 2 || rotary_dim % 2 || rotary_dim > head_dim ||
      len % head_dim)
    return OR_ERR_CAPABILITY_MISMATCH;
  for (size_t h = 0; h < len / head_dim; h++) rotate_head(qk + h * head_dim, rotary_dim / 2, neox, c, s);
  return OR_OK;
}

/* recipe.rs:2775-2834 */
int or_apply_rope(float *qk, size_t len, size_t head_dim, size_t rotary_dim, int neox, size_t pos,
                  const float *inv_freq) {
  if (head_dim < 2 || head_dim % 2 || rotary_dim < 2 || rotary_dim % 2 || rotary_dim > head_dim ||
      len % head_dim)
    return OR_ERR_CAPABILITY_MISMATCH;
  if (pos == 0) return OR_OK;
  float c[512], s[512];
  size_t half = rotary_dim / 2;
  float p = (float)pos;
  for (size_t i = 0; i < half; i++) { float a = p * inv_freq[i]; s[i] = sinf(a); c[i] = cosf(a); }
  for (size_t h = 0; h < len / head_dim; h++) rotate_head(qk + h * head_dim, half, neox, c, s);
  return OR_OK;
}

/* recipe.rs:2892-3022 (validate_gqa_prefill_portable + gqa_attention_prefill_portable) */
int or_gqa_attention(float *out, const float *q, const float *k_cache, const float *v_cache, size_t m,
                     size_t nq, size_t nkv, size_t hd, size_t total_seq, size_t start_pos,
                     size_t sliding_window, float scale, float *scratch, size_t scratch_len) {
  size_t query_end = start_pos + m;
  if (m == 0 || nkv == 0 || nq == 0 || hd == 0 || total_seq == 0 || nq % nkv != 0 || !isfinite(scale) ||
      query_end > total_seq)
    return OR_ERR_CAPABILITY_MISMATCH;
  size_t min_scratch = sliding_window ? (sliding_window < query_end ? sliding_window : query_end) : query_end;
  if (scratch_len < min_scratch) return OR_ERR_TENSOR_BOUNDS;
  size_t kv_stride = nkv * hd, group = nq / nkv;
  for (size_t hkv = 0; hkv < nkv; hkv++) {
    size_t kv_off = hkv * hd;
    for (size_t tok = 0; tok < m; tok++) {
      size_t qpos = start_pos + tok;
      size_t vend = qpos + 1 < total_seq ? qpos + 1 : total_seq;
      size_t vstart = 0;
      if (sliding_window) vstart = qpos + 1 > sliding_window ? qpos + 1 - sliding_window : 0;
      size_t active = vend > vstart ? vend - vstart : 0;
      for (size_t g = 0; g < group; g++) {
        size_t hq = hkv * group + g;
        const float *qh = q + (tok * nq + hq) * hd;
        float maxs = -INFINITY;
        for (size_t i = 0; i < active; i++) {
          const float *kh = k_cache + (vstart + i) * kv_stride + kv_off;
          float d = -0.0f;
          for (size_t e = 0; e < hd; e++) d += qh[e] * kh[e];
          float sc = d * scale;
          scratch[i] = sc;
          if (sc > maxs) maxs = sc;
        }
        float denom = 0.0f;
        for (size_t i = 0; i < active; i++) { scratch[i] = expf(scratch[i] - maxs); denom += scratch[i]; }
        float inv = denom > 0.0f ? 1.0f / denom : 0.0f;
        float *oh = out + (tok * nq + hq) * hd;
        for (size_t e = 0; e < hd; e++) oh[e] = 0.0f;
        for (size_t i = 0; i < active; i++) {
          float w = scratch[i] * inv;
          const float *vh = v_cache + (vstart + i) * kv_stride + kv_off;
          for (size_t e = 0; e < hd; e++) oh[e] += w * vh[e];
        }
      }
    }
  }
  return OR_OK;
}

/* recipe.rs:3024-3050 */
int or_swiglu(float *out, const float *gate, const float *up, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float g = gate[i], sig;
    if (g <= -20.0f) sig = 0.0f;
    else if (g >= 20.0f) sig = 1.0f;
    else sig = 1.0f / (1.0f + expf(-g));
    out[i] = (g * sig) * up[i];
  }
  return OR_OK;
}

/* ---------------------------------------------------------------------- */
/* Model forward: ModelRepackCache::build (repack_cache.rs:2166-2257),      */
/* execute_decode_in_scope (recipe.rs:807-1163) and execute_batch_forward   */
/* + project_logits (recipe.rs:1489-1807).                                   */
/* ---------------------------------------------------------------------- */

typedef struct or_layer {
  float *attn_norm, *ffn_norm;
  or_repacked wq, wk, wv, wo, wgate, wup, wdown;
  float *bq, *bk, *bv, *bo;
} or_layer;

struct or_model {
  or_geometry g;
  size_t total_q, total_kv;
  or_layer *layers;
  float *output_norm;
  or_repacked lm_head;
  or_tensor emb;  /* copied: caller owns only the payload bytes */
  size_t emb_rows;
  int nthreads;
  float *last_hidden;
  uint8_t *skip_rope;
  float *short_f, *long_f;
};

static const or_tensor *find_tensor(const or_tensor *t, size_t n, const char *name) {
  for (size_t i = 0; i < n; i++) if (strcmp(t[i].name, name) == 0) return &t[i];
  return NULL;
}

/* repack_cache.rs:1094-1158 */
static int resolve_2d(const or_tensor *t, size_t expected_cols, size_t *rows, size_t *cols) {
  if (t->n_dims != 2) return OR_ERR_TENSOR_BOUNDS;
  size_t d0 = t->ne[0], d1 = t->ne[1];
  if (d0 == expected_cols) { *rows = d1; *cols = d0; }
  else if (d1 == expected_cols) { *rows = d0; *cols = d1; }
  else return OR_ERR_TENSOR_BOUNDS;
  size_t rb;
  if (!or_quant_row_bytes(*cols, t->quant, &rb)) return OR_ERR_TENSOR_BOUNDS;
  if (t->nbytes < *rows * rb) return OR_ERR_TENSOR_BOUNDS;
  return OR_OK;
}

/* Aligned128F32::from_tensor (repack_cache.rs:1321-1353) */
static int decode_1d(const or_tensor *t, size_t len, int sanitize, float **out) {
  size_t ne = 1;
  for (int i = 0; i < t->n_dims; i++) ne *= t->ne[i];
  if (ne != len) return OR_ERR_TENSOR_BOUNDS;
  size_t rb;
  if (!or_quant_row_bytes(len, t->quant, &rb)) return OR_ERR_CAPABILITY_MISMATCH;
  if (t->nbytes < rb) return OR_ERR_TENSOR_BOUNDS;
  *out = (float *)calloc(len, sizeof(float));
  return or_decode_row_payload_to_f32(t->quant, t->data, len, *out, sanitize);
}

static int repack_checked(const or_tensor *ts, size_t n, const char *name, size_t exp_cols,
                          size_t exp_rows, or_repacked *out) {
  const or_tensor *t = find_tensor(ts, n, name);
  if (!t) return OR_ERR_TENSOR_BOUNDS;
  size_t rows, cols;
  int rc = resolve_2d(t, exp_cols, &rows, &cols);
  if (rc) return rc;
  if (rows != exp_rows) return OR_ERR_TENSOR_BOUNDS;
  return or_repack(t->data, t->nbytes, t->quant, rows, cols, out);
}

static int opt_1d(const or_tensor *ts, size_t n, const char *name, size_t len, float **out) {
  *out = NULL;
  const or_tensor *t = find_tensor(ts, n, name);
  if (!t) return OR_OK;
  return decode_1d(t, len, 0, out);
}

int or_model_build(const or_geometry *g, const or_tensor *ts, size_t n, int nthreads, or_model **out) {
  or_model *m = (or_model *)calloc(1, sizeof(or_model));
  m->g = *g;
  m->nthreads = nthreads;
  m->total_q = g->n_heads_q * g->head_dim;
  m->total_kv = g->n_heads_kv * g->head_dim;
  if (g->skip_rope_layers) {
    m->skip_rope = (uint8_t *)malloc(g->num_layers);
    memcpy(m->skip_rope, g->skip_rope_layers, g->num_layers);
    m->g.skip_rope_layers = m->skip_rope;
  }
  if (g->scaling.kind == 3) {
    m->short_f = (float *)malloc(g->scaling.n_factors * sizeof(float));
    m->long_f = (float *)malloc(g->scaling.n_factors * sizeof(float));
    memcpy(m->short_f, g->scaling.short_factor, g->scaling.n_factors * sizeof(float));
    memcpy(m->long_f, g->scaling.long_factor, g->scaling.n_factors * sizeof(float));
    m->g.scaling.short_factor = m->short_f;
    m->g.scaling.long_factor = m->long_f;
  }
  m->layers = (or_layer *)calloc(g->num_layers, sizeof(or_layer));
  m->last_hidden = (float *)calloc(g->hidden_dim, sizeof(float));
  char nm[128];
  int rc = OR_OK;
  size_t H = g->hidden_dim, F = g->ffn_dim, Q = m->total_q, KV = m->total_kv;
  for (size_t l = 0; l < g->num_layers && rc == OR_OK; l++) {
    or_layer *L = &m->layers[l];
    const or_tensor *t;
    snprintf(nm, sizeof nm, "blk.%zu.attn_norm.weight", l);
    if (!(t = find_tensor(ts, n, nm))) { rc = OR_ERR_TENSOR_BOUNDS; break; }
    if ((rc = decode_1d(t, H, 1, &L->attn_norm))) break;
    snprintf(nm, sizeof nm, "blk.%zu.ffn_norm.weight", l);
    if (!(t = find_tensor(ts, n, nm))) { rc = OR_ERR_TENSOR_BOUNDS; break; }
    if ((rc = decode_1d(t, H, 1, &L->ffn_norm))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_q.weight", l);
    if ((rc = repack_checked(ts, n, nm, H, Q, &L->wq))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_k.weight", l);
    if ((rc = repack_checked(ts, n, nm, H, KV, &L->wk))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_v.weight", l);
    if ((rc = repack_checked(ts, n, nm, H, KV, &L->wv))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_output.weight", l);
    if ((rc = repack_checked(ts, n, nm, Q, H, &L->wo))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_q.bias", l);
    if ((rc = opt_1d(ts, n, nm, Q, &L->bq))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_k.bias", l);
    if ((rc = opt_1d(ts, n, nm, KV, &L->bk))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_v.bias", l);
    if ((rc = opt_1d(ts, n, nm, KV, &L->bv))) break;
    snprintf(nm, sizeof nm, "blk.%zu.attn_output.bias", l);
    if ((rc = opt_1d(ts, n, nm, H, &L->bo))) break;
    snprintf(nm, sizeof nm, "blk.%zu.ffn_gate.weight", l);
    if ((rc = repack_checked(ts, n, nm, H, F, &L->wgate))) break;
    snprintf(nm, sizeof nm, "blk.%zu.ffn_up.weight", l);
    if ((rc = repack_checked(ts, n, nm, H, F, &L->wup))) break;
    snprintf(nm, sizeof nm, "blk.%zu.ffn_down.weight", l);
    if ((rc = repack_checked(ts, n, nm, F, H, &L->wdown))) break;
  }
  if (rc == OR_OK) {
    const or_tensor *t = find_tensor(ts, n, "output_norm.weight");
    if (!t) rc = OR_ERR_TENSOR_BOUNDS;
    else rc = decode_1d(t, H, 1, &m->output_norm);
  }
  if (rc == OR_OK) {
    const or_tensor *emb = find_tensor(ts, n, "token_embd.weight");
    const or_tensor *head = find_tensor(ts, n, "output.weight");
    if (!head) head = emb;
    if (!head || !emb) rc = OR_ERR_TENSOR_BOUNDS;
    else {
      size_t rows, cols;
      rc = resolve_2d(head, H, &rows, &cols);
      if (rc == OR_OK) rc = or_repack(head->data, head->nbytes, head->quant, rows, cols, &m->lm_head);
      if (rc == OR_OK) { m->emb = *emb; m->emb.name = NULL; rc = resolve_2d(emb, H, &m->emb_rows, &cols); }
    }
  }
  if (rc != OR_OK) { or_model_free(m); *out = NULL; return rc; }
  *out = m;
  return OR_OK;
}

void or_model_free(or_model *m) {
  if (!m) return;
  for (size_t l = 0; l < m->g.num_layers && m->layers; l++) {
    or_layer *L = &m->layers[l];
    free(L->attn_norm); free(L->ffn_norm); free(L->bq); free(L->bk); free(L->bv); free(L->bo);
    or_repacked_free(&L->wq); or_repacked_free(&L->wk); or_repacked_free(&L->wv); or_repacked_free(&L->wo);
    or_repacked_free(&L->wgate); or_repacked_free(&L->wup); or_repacked_free(&L->wdown);
  }
  free(m->layers); free(m->output_norm); or_repacked_free(&m->lm_head);
  free(m->last_hidden); free(m->skip_rope); free(m->short_f); free(m->long_f);
  free(m);
}

size_t or_model_vocab(const or_model *m) { return m->lm_head.rows; }
const float *or_model_last_hidden(const or_model *m) { return m->last_hidden; }

/* recipe.rs:1395-1440 */
static int embed(const or_model *m, const uint32_t *toks, size_t n, float *hidden) {
  size_t H = m->g.hidden_dim, rb;
  if (!or_quant_row_bytes(H, m->emb.quant, &rb)) return OR_ERR_CAPABILITY_MISMATCH;
  for (size_t i = 0; i < n; i++) {
    if (toks[i] >= m->emb_rows) return OR_ERR_TENSOR_BOUNDS;
    int rc = or_decode_row_payload_to_f32(m->emb.quant, m->emb.data + (size_t)toks[i] * rb, H,
                                          hidden + i * H, 1);
    if (rc) return rc;
  }
  return OR_OK;
}

static void add_bias(float *batch, const float *b, size_t dim, size_t m) {
  if (!b) return;
  for (size_t t = 0; t < m; t++)
    for (size_t i = 0; i < dim; i++) batch[t * dim + i] += b[i];
}

/* f32 -> f16 (round to nearest even) -> f32, for the f16 KV cache option. */
static float f16_round(float v) {
  uint16_t h = or_f32_to_f16_rne(v);
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1F, mant = h & 0x3FF, bits;
  if (e == 0) {
    if (mant == 0) bits = sign;
    else {
      int sh = 0;
      while (!(mant & 0x400)) { mant <<= 1; sh++; }
      bits = sign | ((uint32_t)(113 - sh) << 23) | ((mant & 0x3FF) << 13);
    }
  } else if (e == 31) bits = sign | 0x7F800000u | (mant << 13);
  else bits = sign | ((e + 112u) << 23) | (mant << 13);
  return f_from_bits(bits);
}

/* Shared per-layer body for M tokens at positions start..start+M (the cached
 * batched forward; decode is the M = 1 case and produces identical math). */
static int forward_tokens(or_model *m, float *kv, size_t seq_cap, const uint32_t *toks, size_t M,
                          size_t start, int compute_logits, float *logits) {
  const or_geometry *g = &m->g;
  size_t H = g->hidden_dim, F = g->ffn_dim, Q = m->total_q, KV = m->total_kv, hd = g->head_dim;
  size_t end = start + M;
  if (end > seq_cap) return OR_ERR_CONTEXT_LENGTH_EXCEEDED;
  float *hidden = (float *)calloc(M * H, sizeof(float));
  int rc = embed(m, toks, M, hidden);
  if (rc) { free(hidden); return rc; }
  float *inv_freq = (float *)calloc(g->rotary_dim / 2, sizeof(float));
  rc = or_fill_inv_freq(g->rotary_dim, g->rope_theta, &g->scaling, end, inv_freq);
  if (rc) { free(hidden); free(inv_freq); return rc; }
  float *norm = (float *)malloc(M * H * sizeof(float));
  float *q = (float *)malloc(M * Q * sizeof(float));
  float *k = (float *)malloc(M * KV * sizeof(float));
  float *v = (float *)malloc(M * KV * sizeof(float));
  float *att = (float *)malloc(M * Q * sizeof(float));
  float *proj = (float *)malloc(M * H * sizeof(float));
  float *gate = (float *)malloc(M * F * sizeof(float));
  float *up = (float *)malloc(M * F * sizeof(float));
  float *act = (float *)malloc(M * F * sizeof(float));
  float *scores = (float *)malloc((end + 1) * sizeof(float));
  float eps = g->rms_eps > 1.0e-7f ? g->rms_eps : 1.0e-7f;
  float scale = 1.0f / sqrtf((float)hd);
  for (size_t l = 0; l < g->num_layers && rc == OR_OK; l++) {
    or_layer *L = &m->layers[l];
    for (size_t t = 0; t < M; t++) or_rmsnorm_row(norm + t * H, hidden + t * H, L->attn_norm, H, eps);
    or_project_batch(&L->wq, q, norm, M, m->nthreads);
    add_bias(q, L->bq, Q, M);
    or_project_batch(&L->wk, k, norm, M, m->nthreads);
    add_bias(k, L->bk, KV, M);
    or_project_batch(&L->wv, v, norm, M, m->nthreads);
    add_bias(v, L->bv, KV, M);
    int skip = g->skip_rope_layers && g->skip_rope_layers[l];
    if (!skip) {
      for (size_t t = 0; t < M; t++) {
        or_apply_rope(q + t * Q, Q, hd, g->rotary_dim, g->neox, start + t, inv_freq);
        or_apply_rope(k + t * KV, KV, hd, g->rotary_dim, g->neox, start + t, inv_freq);
      }
    }
    /* KV append (recipe.rs:2319-2326); layout [layer][K|V][seq_cap][KV] */
    float *kp = kv + (l * 2 + 0) * seq_cap * KV, *vp = kv + (l * 2 + 1) * seq_cap * KV;
    memcpy(kp + start * KV, k, M * KV * sizeof(float));
    memcpy(vp + start * KV, v, M * KV * sizeof(float));
    if (g->kv_f16) /* an f16 cache holds the appended rows rounded to f16 */
      for (size_t i = start * KV; i < end * KV; i++) {
        kp[i] = f16_round(kp[i]);
        vp[i] = f16_round(vp[i]);
      }
    rc = or_gqa_attention(att, q, kp, vp, M, g->n_heads_q, g->n_heads_kv, hd, end, start,
                          g->sliding_window, scale, scores, end + 1);
    if (rc) break;
    or_project_batch(&L->wo, proj, att, M, m->nthreads);
    add_bias(proj, L->bo, H, M);
    for (size_t i = 0; i < M * H; i++) hidden[i] += proj[i];
    for (size_t t = 0; t < M; t++) or_rmsnorm_row(norm + t * H, hidden + t * H, L->ffn_norm, H, eps);
    or_project_batch(&L->wgate, gate, norm, M, m->nthreads);
    or_project_batch(&L->wup, up, norm, M, m->nthreads);
    or_swiglu(act, gate, up, M * F);
    or_project_batch(&L->wdown, proj, act, M, m->nthreads);
    for (size_t i = 0; i < M * H; i++) hidden[i] += proj[i];
  }
  if (rc == OR_OK && compute_logits) {
    or_rmsnorm_row(m->last_hidden, hidden + (M - 1) * H, m->output_norm, H, eps);
    if (logits) or_project_batch(&m->lm_head, logits, m->last_hidden, 1, m->nthreads);
  }
  free(hidden); free(inv_freq); free(norm); free(q); free(k); free(v); free(att); free(proj);
  free(gate); free(up); free(act); free(scores);
  return rc;
}

/* recipe.rs:564-608 (prefill_step_inner with cache) */
int or_prefill(or_model *m, float *kv, size_t seq_cap, const uint32_t *tokens, size_t n, size_t start_pos,
               int compute_logits, float *logits) {
  if (n == 0) return OR_OK;
  return forward_tokens(m, kv, seq_cap, tokens, n, start_pos, compute_logits, logits);
}

/* recipe.rs:718-797, 807-1163 (decode_step_inner with cache) */
int or_decode(or_model *m, float *kv, size_t seq_cap, uint32_t token, size_t pos, float *logits) {
  return forward_tokens(m, kv, seq_cap, &token, 1, pos, 1, logits);
}
