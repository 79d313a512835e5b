// Streaming raw-GGUF GEMV for the super-block and dense types
// (gemv_decode_projection, decode_gemv.rs:1289-1388): Q4_K / Q5_K / Q6_K /
// TQ1_0 / TQ2_0 rows against the BlockQ8_K activation (decode_gemv.rs:
// 320-346, 456-620), and F16 / BF16 / F32 rows against the f32 activation in
// 256-element chunks (dot_dense_row_zero_alloc, decode_gemv.rs:1081-1166).
//
// A warp takes one row; lane l evaluates super-blocks (or 256-element
// chunks) l, l + 32, ... with the reference's per-block integer sums and
// float combination, and the block results are then added in block order
// through shuffles, so every output equals the reference's sequential sum
// bit for bit.  Weights are read in place (no repack); the Q8_K activation
// is a 304-byte device block per 256 elements: qs[256], bsums[16], d, pad.
#include <cuda_fp16.h>

#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

struct alignas(16) Q8KBlock {
  int8_t qs[256];
  int16_t bsums[16];
  float d;
  float pad[3];
};
static_assert(sizeof(Q8KBlock) == kQ8KBlockBytes, "Q8_K device block size");

__device__ __forceinline__ uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// quantize_row_q8_k (decode_gemv.rs:320-346): one CTA of 256 threads per
// super-block; amax over the finite values, d = amax / 127, bsums per 16.
__global__ void k_quantize_row_q8_k(const float *__restrict__ x, Q8KBlock *__restrict__ out) {
  __shared__ float red[8];
  const int t = threadIdx.x, lane = t % 32, warp = t / 32;
  const float v = x[(int64_t)blockIdx.x * 256 + t];
  const bool fin = isfinite(v);
  float a = warp_max(fin ? fabsf(v) : 0.0f);
  if (lane == 0) red[warp] = a;
  __syncthreads();
  float amax = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) amax = fmaxf(amax, red[w]);
  Q8KBlock &o = out[blockIdx.x];
  if (amax == 0.0f || !isfinite(amax)) {
    o.qs[t] = 0;
    if (t < 16) o.bsums[t] = 0;
    if (t == 0) o.d = 0.0f;
    return;
  }
  const float inv = __fdiv_rn(127.0f, amax);
  const int q = fin ? (int)act_quant_one(v, inv) : 0;
  o.qs[t] = (int8_t)q;
  int s = q;  // sum over the 16 consecutive elements of this half-warp
#pragma unroll
  for (int m = 1; m < 16; m <<= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  if ((t & 15) == 0) o.bsums[t / 16] = (int16_t)s;
  if (t == 0) o.d = __fdiv_rn(amax, 127.0f);
}

// unpack_q4_k_scales: six-bit scales and mins of a Q4_K / Q5_K super-block.
__device__ __forceinline__ void q4k_scales(const uint8_t *s, int (&sc)[8], int (&m)[8]) {
#pragma unroll
  for (int j = 0; j < 4; j++) {
    sc[j] = s[j] & 0x3F;
    m[j] = s[j + 4] & 0x3F;
  }
#pragma unroll
  for (int j = 4; j < 8; j++) {
    sc[j] = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
    m[j] = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// One super-block of `QUANT` against one Q8_K block; the float expression of
// each type is the reference's, without contraction.
template <int QUANT>
__device__ float superblock_dot(const uint8_t *w, const Q8KBlock &x) {
  const float xd = x.d;
  if (QUANT == JAL_Q4_K || QUANT == JAL_Q5_K) {  // decode_gemv.rs:456-523
    const float d = f16_finite(rd16(w)), dmin = f16_finite(rd16(w + 2));
    if ((d == 0.0f && dmin == 0.0f) || xd == 0.0f) return 0.0f;
    int sc[8], mn[8];
    q4k_scales(w + 4, sc, mn);
    const uint8_t *qh = QUANT == JAL_Q5_K ? w + 16 : nullptr;
    const uint8_t *qs = QUANT == JAL_Q5_K ? w + 48 : w + 16;
    int sumi = 0, sum_mins = 0;
    for (int chunk = 0; chunk < 4; chunk++) {
      const int u1 = 1 << (2 * chunk), u2 = 2 << (2 * chunk);
      const int8_t *xlo = x.qs + chunk * 64, *xhi = xlo + 32;
      int slo = 0, shi = 0;
      for (int l = 0; l < 32; l++) {
        const int b = qs[chunk * 32 + l];
        int hb1 = 0, hb2 = 0;
        if (QUANT == JAL_Q5_K) {
          hb1 = (qh[l] & u1) ? 16 : 0;
          hb2 = (qh[l] & u2) ? 16 : 0;
        }
        slo += ((b & 0x0F) | hb1) * xlo[l];
        shi += ((b >> 4) | hb2) * xhi[l];
      }
      sumi += sc[2 * chunk] * slo + sc[2 * chunk + 1] * shi;
      const int blo = (int)x.bsums[chunk * 4] + x.bsums[chunk * 4 + 1];
      const int bhi = (int)x.bsums[chunk * 4 + 2] + x.bsums[chunk * 4 + 3];
      sum_mins += mn[2 * chunk] * blo + mn[2 * chunk + 1] * bhi;
    }
    return __fsub_rn(__fmul_rn(__fmul_rn(d, xd), (float)sumi), __fmul_rn(__fmul_rn(dmin, xd), (float)sum_mins));
  } else if (QUANT == JAL_Q6_K) {  // decode_gemv.rs:525-564
    const float d = f16_finite(rd16(w + 208));
    if (d == 0.0f || xd == 0.0f) return 0.0f;
    const uint8_t *ql = w, *qh = w + 128;
    const int8_t *scales = (const int8_t *)(w + 192);
    int sumi = 0;
    for (int half = 0; half < 2; half++) {
      const int n = half * 128, qlo = half * 64, qhi = half * 32, scb = half * 8;
      for (int is = 0; is < 2; is++) {
        const int lb = is * 16;
        const int sc1 = scales[scb + is], sc2 = scales[scb + is + 2];
        const int sc3 = scales[scb + is + 4], sc4 = scales[scb + is + 6];
        int s1 = 0, s2 = 0, s3 = 0, s4 = 0;
        for (int l = lb; l < lb + 16; l++) {
          const int blo = ql[qlo + l], bhi = ql[qlo + l + 32], hb = qh[qhi + l];
          s1 += (((blo & 0x0F) | ((hb & 0x03) << 4)) - 32) * x.qs[n + l];
          s2 += (((bhi & 0x0F) | (((hb >> 2) & 0x03) << 4)) - 32) * x.qs[n + l + 32];
          s3 += (((blo >> 4) | (((hb >> 4) & 0x03) << 4)) - 32) * x.qs[n + l + 64];
          s4 += (((bhi >> 4) | (((hb >> 6) & 0x03) << 4)) - 32) * x.qs[n + l + 96];
        }
        sumi += sc1 * s1 + sc2 * s2 + sc3 * s3 + sc4 * s4;
      }
    }
    return __fmul_rn(__fmul_rn(d, xd), (float)sumi);
  } else if (QUANT == JAL_TQ1_0) {  // decode_gemv.rs:566-603
    const float d = f16_finite(rd16(w));
    if (d == 0.0f || xd == 0.0f) return 0.0f;
    int sumi = 0;
    for (int i = 0; i < 51; i++) {
      unsigned cur = w[2 + i];
#pragma unroll
      for (int j = 0; j < 5; j++) {
        sumi += ((int)(cur % 3u) - 1) * x.qs[i * 5 + j];
        cur /= 3u;
      }
    }
    sumi += ((int)(w[53] % 3u) - 1) * x.qs[255];
    return __fmul_rn((float)sumi, __fmul_rn(d, xd));
  } else {  // TQ2_0, decode_gemv.rs:605-620
    const float d = bf16_finite(rd16(w + 64));
    if (d == 0.0f || xd == 0.0f) return 0.0f;
    int sumi = 0;
    for (int i = 0; i < 64; i++) {
      const int b = w[i];
#pragma unroll
      for (int sub = 0; sub < 4; sub++) sumi += (((b >> (2 * sub)) & 0x03) - 1) * x.qs[i * 4 + sub];
    }
    return __fmul_rn((float)sumi, __fmul_rn(d, xd));
  }
}

template <int QUANT>
constexpr int superblock_bytes() {
  return QUANT == JAL_Q4_K ? 144 : QUANT == JAL_Q5_K ? 176 : QUANT == JAL_Q6_K ? 210 : QUANT == JAL_TQ1_0 ? 54 : 66;
}

// Adds the lanes' block results t (block b0 + lane) in block order.
__device__ __forceinline__ float add_in_order(float acc, float t, int64_t b0, int64_t nb) {
  for (int k = 0; k < 32; k++) {
    const float v = __shfl_sync(0xffffffffu, t, k);
    if (b0 + k < nb) acc = __fadd_rn(acc, v);
  }
  return acc;
}

template <int QUANT>
__global__ void k_gemv_raw_superblock(const uint8_t *__restrict__ raw, int64_t rows, int64_t nb,
                                      const Q8KBlock *__restrict__ xb, float *__restrict__ y) {
  constexpr int BB = superblock_bytes<QUANT>();
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;  // whole warps leave together
  const uint8_t *rp = raw + row * nb * BB;
  float acc = 0.0f;
  for (int64_t b0 = 0; b0 < nb; b0 += 32) {
    const int64_t b = b0 + lane;
    const float t = b < nb ? superblock_dot<QUANT>(rp + b * BB, xb[b]) : 0.0f;
    acc = add_in_order(acc, t, b0, nb);
  }
  if (lane == 0) y[row] = acc;
}

// dot_dense_row_zero_alloc: per 256-element chunk, a -0.0-started
// sequential f32 sum of sanitised weight x (finite-masked) activation; the
// finite chunk sums are added in order.
template <int QUANT>
__global__ void k_gemv_raw_dense(const uint8_t *__restrict__ raw, int64_t rows, int64_t cols,
                                 const float *__restrict__ x, float *__restrict__ y) {
  constexpr int ES = QUANT == JAL_F32 ? 4 : 2;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const uint8_t *rp = raw + row * cols * ES;
  const int64_t nc = (cols + 255) / 256;
  float sum = 0.0f;
  for (int64_t c0 = 0; c0 < nc; c0 += 32) {
    const int64_t c = c0 + lane;
    float term = -0.0f;
    bool ok = false;
    if (c < nc) {
      const int64_t e0 = c * 256, e1 = e0 + 256 < cols ? e0 + 256 : cols;
      for (int64_t e = e0; e < e1; e++) {
        float wv;
        if (QUANT == JAL_F32) wv = sanitize_weight(((const float *)rp)[e]);
        else if (QUANT == JAL_F16) wv = f16_finite(((const uint16_t *)rp)[e]);
        else wv = bf16_finite(((const uint16_t *)rp)[e]);
        const float xv = x[e];
        term = __fadd_rn(term, __fmul_rn(wv, isfinite(xv) ? xv : 0.0f));
      }
      ok = isfinite(term);
    }
    for (int k = 0; k < 32; k++) {
      const float v = __shfl_sync(0xffffffffu, term, k);
      const int vk = __shfl_sync(0xffffffffu, ok ? 1 : 0, k);
      if (c0 + k < nc && vk) sum = __fadd_rn(sum, v);
    }
  }
  if (lane == 0) y[row] = sum;
}

}  // namespace

bool superblock_quant(int q) {
  return q == JAL_Q4_K || q == JAL_Q5_K || q == JAL_Q6_K || q == JAL_TQ1_0 || q == JAL_TQ2_0;
}

void launch_quantize_row_q8_k(const float *x, int64_t n, void *blocks, cudaStream_t s) {
  if (n < 256) return;
  k_quantize_row_q8_k<<<(unsigned)(n / 256), 256, 0, s>>>(x, (Q8KBlock *)blocks);
}

void launch_gemv_raw_superblock(const uint8_t *raw, int quant, int64_t rows, int64_t cols, const void *xblocks,
                                float *y, cudaStream_t s) {
  if (!rows) return;
  const unsigned grid = (unsigned)((rows * 32 + 255) / 256);
  const int64_t nb = cols / 256;
  const Q8KBlock *xb = (const Q8KBlock *)xblocks;
  switch (quant) {
    case JAL_Q4_K: k_gemv_raw_superblock<JAL_Q4_K><<<grid, 256, 0, s>>>(raw, rows, nb, xb, y); break;
    case JAL_Q5_K: k_gemv_raw_superblock<JAL_Q5_K><<<grid, 256, 0, s>>>(raw, rows, nb, xb, y); break;
    case JAL_Q6_K: k_gemv_raw_superblock<JAL_Q6_K><<<grid, 256, 0, s>>>(raw, rows, nb, xb, y); break;
    case JAL_TQ1_0: k_gemv_raw_superblock<JAL_TQ1_0><<<grid, 256, 0, s>>>(raw, rows, nb, xb, y); break;
    default: k_gemv_raw_superblock<JAL_TQ2_0><<<grid, 256, 0, s>>>(raw, rows, nb, xb, y); break;
  }
}

void launch_gemv_raw_dense(const uint8_t *raw, int quant, int64_t rows, int64_t cols, const float *x, float *y,
                           cudaStream_t s) {
  if (!rows) return;
  const unsigned grid = (unsigned)((rows * 32 + 255) / 256);
  if (quant == JAL_F16) k_gemv_raw_dense<JAL_F16><<<grid, 256, 0, s>>>(raw, rows, cols, x, y);
  else if (quant == JAL_BF16) k_gemv_raw_dense<JAL_BF16><<<grid, 256, 0, s>>>(raw, rows, cols, x, y);
  else k_gemv_raw_dense<JAL_F32><<<grid, 256, 0, s>>>(raw, rows, cols, x, y);
}

}  // namespace jal
