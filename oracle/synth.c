/*
 * Seeded synthetic tensors for the CPU side (TEST INFRASTRUCTURE ONLY).
 *
 * The reference has no random generator and no f32 -> Q4_0 quantizer, so the
 * synthetic models of the benchmark and the tests are new fixtures.  This file
 * restates, in plain C, the generator whose bytes the device side consumes:
 * per tensor a SplitMix64 counter stream keyed by (seed, FNV-1a of the tensor
 * name), Box-Muller in double, value = (float)(std * normal), then the public
 * GGML reference quantizers (Q4_0: d = max / -8, q = min(15, (i8)(x/d + 8.5));
 * Q8_0: d = amax / 127, q = round(x / d)), f16 scales rounded to nearest even.
 * It lets the CPU baseline build its model without loading the product
 * library; a CPU test checks that both produce identical bytes.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "oracle.h"

static uint64_t sm64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

static uint64_t fnv1a(const char *s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (; *s; s++) h = (h ^ (uint8_t)*s) * 0x100000001b3ull;
  return h;
}

static void normal_pair(uint64_t key, uint64_t j, double *n0, double *n1) {
  uint64_t z1 = sm64(key + 2 * j), z2 = sm64(key + 2 * j + 1);
  double u1 = (double)((z1 >> 11) + 1) * (1.0 / 9007199254740992.0);
  double u2 = (double)(z2 >> 11) * (1.0 / 9007199254740992.0);
  double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586476925 * u2;
  *n0 = r * cos(th);
  *n1 = r * sin(th);
}

static void gen_block(uint64_t key, uint64_t first, size_t n, float sd, float *out) {
  for (size_t k = 0; k < n; k += 2) {
    double a, b;
    normal_pair(key, (first + k) / 2, &a, &b);
    out[k] = (float)(sd * a);
    if (k + 1 < n) out[k + 1] = (float)(sd * b);
  }
}

uint16_t or_f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  x &= 0x7FFFFFFFu;
  if (x >= 0x7F800000u) return (uint16_t)(sign | (x > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (x >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (x < 0x38800000u) {
    if (x < 0x33000000u) return (uint16_t)sign;
    uint32_t mant = (x & 0x7FFFFFu) | 0x800000u;
    int shift = 126 - (int)(x >> 23);
    uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = (x >> 13) - (112u << 10), rem = x & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static void quant_q4_0(const float *x, uint8_t *out) {
  float amax = 0.f, max = 0.f;
  for (int j = 0; j < 32; j++)
    if (amax < fabsf(x[j])) { amax = fabsf(x[j]); max = x[j]; }
  float d = max / -8.0f, id = d != 0.f ? 1.0f / d : 0.0f;
  uint16_t dh = or_f32_to_f16_rne(d);
  memcpy(out, &dh, 2);
  for (int j = 0; j < 16; j++) {
    int a = (int8_t)(x[j] * id + 8.5f), b = (int8_t)(x[16 + j] * id + 8.5f);
    if (a > 15) a = 15;
    if (b > 15) b = 15;
    out[2 + j] = (uint8_t)(a | (b << 4));
  }
}

static void quant_q8_0(const float *x, uint8_t *out) {
  float amax = 0.f;
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
  float d = amax / 127.0f, id = d != 0.f ? 1.0f / d : 0.0f;
  uint16_t dh = or_f32_to_f16_rne(d);
  memcpy(out, &dh, 2);
  for (int j = 0; j < 32; j++) out[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

int or_synth_matrix(int quant, size_t rows, size_t cols, uint64_t seed, const char *name, float sd, void *out,
                    size_t len, int nthreads) {
  size_t rb;
  if (!out || !name || cols % 32) return OR_ERR_TENSOR_BOUNDS;
  if (quant != OR_Q4_0 && quant != OR_Q8_0 && quant != OR_F32) return OR_ERR_CAPABILITY_MISMATCH;
  if (!or_quant_row_bytes(cols, quant, &rb) || len < rows * rb) return OR_ERR_TENSOR_BOUNDS;
  const uint64_t key = sm64(seed ^ sm64(fnv1a(name)));
  (void)nthreads;
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads > 0 ? nthreads : 1) if (nthreads > 1)
  for (size_t r = 0; r < rows; r++) {
    float buf[32];
    uint8_t *row = (uint8_t *)out + r * rb;
    for (size_t b = 0; b < cols / 32; b++) {
      gen_block(key, (uint64_t)r * cols + b * 32, 32, sd, buf);
      if (quant == OR_F32) memcpy(row + b * 128, buf, 128);
      else if (quant == OR_Q4_0) quant_q4_0(buf, row + b * 18);
      else quant_q8_0(buf, row + b * 34);
    }
  }
  return OR_OK;
}
