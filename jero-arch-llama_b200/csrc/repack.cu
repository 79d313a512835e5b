// One-time device repack of GGUF Q4_0 / Q8_0 blocks into the B200 layout,
// the export back to the reference's portable tile layout, the activation
// quantizers, RMSNorm, the raw-GGUF streaming GEMV and the embedding
// gather.
#include <cuda_fp16.h>

#include "common.hpp"
#include "dev_util.cuh"
#include "exact.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

// The reference decodes block scales with f16_to_f32_finite (Inf/NaN ->
// +-0.0625).  0.0625 = 2^-4 is exactly representable in f16 (0x2C00), so the
// repack stores the sanitized half and every kernel may convert it plainly.
__device__ __forceinline__ uint16_t sanitize_f16(uint16_t h) {
  return (h & 0x7C00u) == 0x7C00u ? (uint16_t)((h & 0x8000u) | 0x2C00u) : h;
}

// ---- repack: GGUF block rows -> qs plane + f16 scale plane ---------------
// unpack_row_i8 (repack_cache.rs:840-871) keeps the nibbles/bytes and the
// f16 scale of every block; the B200 layout stores them split into two
// 16-byte aligned planes instead of the reference's 8x16 i8 tiles.
__global__ void k_repack_q4_0(const uint8_t *__restrict__ raw, int64_t rows, int64_t nb, uint8_t *__restrict__ qs,
                              uint16_t *__restrict__ d, int64_t qs_stride, int64_t d_stride) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nb) return;
  int64_t r = idx / nb, g = idx % nb;
  const uint16_t *src = (const uint16_t *)(raw + (r * nb + g) * 18);
  uint16_t h[9];
#pragma unroll
  for (int i = 0; i < 9; i++) h[i] = src[i];
  uint4 v;
  v.x = (uint32_t)h[1] | ((uint32_t)h[2] << 16);
  v.y = (uint32_t)h[3] | ((uint32_t)h[4] << 16);
  v.z = (uint32_t)h[5] | ((uint32_t)h[6] << 16);
  v.w = (uint32_t)h[7] | ((uint32_t)h[8] << 16);
  *(uint4 *)(qs + r * qs_stride + g * 16) = v;
  d[r * d_stride + g] = sanitize_f16(h[0]);
}

__global__ void k_repack_q8_0(const uint8_t *__restrict__ raw, int64_t rows, int64_t nb, uint8_t *__restrict__ qs,
                              uint16_t *__restrict__ d, int64_t qs_stride, int64_t d_stride) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nb) return;
  int64_t r = idx / nb, g = idx % nb;
  const uint16_t *src = (const uint16_t *)(raw + (r * nb + g) * 34);
  uint16_t h[17];
#pragma unroll
  for (int i = 0; i < 17; i++) h[i] = src[i];
  uint4 a, b;
  a.x = (uint32_t)h[1] | ((uint32_t)h[2] << 16);
  a.y = (uint32_t)h[3] | ((uint32_t)h[4] << 16);
  a.z = (uint32_t)h[5] | ((uint32_t)h[6] << 16);
  a.w = (uint32_t)h[7] | ((uint32_t)h[8] << 16);
  b.x = (uint32_t)h[9] | ((uint32_t)h[10] << 16);
  b.y = (uint32_t)h[11] | ((uint32_t)h[12] << 16);
  b.z = (uint32_t)h[13] | ((uint32_t)h[14] << 16);
  b.w = (uint32_t)h[15] | ((uint32_t)h[16] << 16);
  uint4 *dst = (uint4 *)(qs + r * qs_stride + g * 32);
  dst[0] = a;
  dst[1] = b;
  d[r * d_stride + g] = sanitize_f16(h[0]);
}

// Q5_0 (unpack_row_i8, repack_cache.rs:840-871): the 5-bit values become
// int8 (q = (nibble | qh bit << 4) - 16), so a Q5_0 matrix takes the Q8_0
// device layout and runs the Q8_0 kernels (the reference evaluates both as
// int8 blocks with one scale per 32).
__global__ void k_repack_q5_0(const uint8_t *__restrict__ raw, int64_t rows, int64_t nb, uint8_t *__restrict__ qs,
                              uint16_t *__restrict__ d, int64_t qs_stride, int64_t d_stride) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * nb) return;
  int64_t r = idx / nb, g = idx % nb;
  const uint8_t *blk = raw + (r * nb + g) * 22;
  const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const int e = 4 * k + b, j = e & 15;
      const uint32_t nib = e < 16 ? (blk[6 + j] & 15u) : (uint32_t)(blk[6 + j] >> 4);
      const uint32_t hb = ((qh >> (e < 16 ? j : j + 16)) & 1u) << 4;
      word |= (uint32_t)(uint8_t)(int8_t)((int)(nib | hb) - 16) << (8 * b);
    }
    w[k] = word;
  }
  uint4 *dst = (uint4 *)(qs + r * qs_stride + g * 32);
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  d[r * d_stride + g] = sanitize_f16((uint16_t)(blk[0] | (blk[1] << 8)));
}

void launch_repack(const uint8_t *raw, int quant, int64_t rows, int64_t cols, uint8_t *qs, uint16_t *d,
                   int64_t qs_stride, int64_t d_stride, cudaStream_t s) {
  int64_t nb = cols / 32, n = rows * nb;
  if (n == 0) return;
  int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (quant == JAL_Q4_0)
    k_repack_q4_0<<<(unsigned)blocks, threads, 0, s>>>(raw, rows, nb, qs, d, qs_stride, d_stride);
  else if (quant == JAL_Q5_0)
    k_repack_q5_0<<<(unsigned)blocks, threads, 0, s>>>(raw, rows, nb, qs, d, qs_stride, d_stride);
  else
    k_repack_q8_0<<<(unsigned)blocks, threads, 0, s>>>(raw, rows, nb, qs, d, qs_stride, d_stride);
}


// ---- export to the reference's portable layout (repack_cache.rs:639-694) --
__device__ __forceinline__ int8_t weight_q(const DevMat &w, int64_t r, int64_t e) {
  int64_t g = e / 32, i = e % 32;
  if (w.quant == JAL_Q4_0) {
    uint8_t byte = w.qs[r * w.qs_stride + g * 16 + (i & 15)];
    return (int8_t)((i < 16 ? (byte & 15) : (byte >> 4)) - 8);
  }
  return (int8_t)w.qs[r * w.qs_stride + e];
}

__global__ void k_export_tiles(DevMat w, int64_t n_tiles, int8_t *__restrict__ tiles) {
  int64_t k_chunks = w.cols / 16;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (padded row, chunk)
  if (idx >= n_tiles * 8 * k_chunks) return;
  int64_t rp = idx / k_chunks, ch = idx % k_chunks;
  int64_t nt = rp / 8, j = rp % 8;
  int8_t *dst = tiles + (nt * k_chunks + ch) * 128 + j * 16;
  for (int t = 0; t < 16; t++) dst[t] = rp < w.rows ? weight_q(w, rp, ch * 16 + t) : (int8_t)0;
}

__global__ void k_export_scales(DevMat w, int64_t n_tiles, float *__restrict__ scales) {
  int64_t groups = w.cols / 32;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_tiles * 8 * groups) return;
  int64_t rp = idx / groups, g = idx % groups, nt = rp / 8, j = rp % 8;
  scales[(nt * groups + g) * 8 + j] = rp < w.rows ? f16_finite(w.d[rp * w.d_stride + g]) : 0.0f;
}

void launch_export_ref(const DevMat &w, int8_t *tiles, float *scales, cudaStream_t s) {
  int64_t n_tiles = (w.rows + 7) / 8;
  int64_t n1 = n_tiles * 8 * (w.cols / 16), n2 = n_tiles * 8 * (w.cols / 32);
  if (n1) k_export_tiles<<<(unsigned)((n1 + 255) / 256), 256, 0, s>>>(w, n_tiles, tiles);
  if (n2) k_export_scales<<<(unsigned)((n2 + 255) / 256), 256, 0, s>>>(w, n_tiles, scales);
}

// ---- QuantizedActQ8 (repack_cache.rs:390-422, 491-531) -------------------
// One warp per 32-block; lane i owns element i.
__global__ void k_act_quant(const float *__restrict__ x, int64_t m, int64_t k, int64_t x_stride,
                            int8_t *__restrict__ q8, float *__restrict__ scales) {
  int64_t nb = (k + 31) / 32;
  int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (wid >= m * nb) return;
  int64_t t = wid / nb, b = wid % nb, c = b * 32 + lane;
  float v = c < k ? x[t * x_stride + c] : 0.0f;
  if (!isfinite(v)) v = 0.0f;
  float amax = warp_max(fabsf(v));
  float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
  q8[t * nb * 32 + c] = c < k ? act_quant_one(v, inv) : (int8_t)0;
  if (lane == 0) scales[t * nb + b] = scale;
}

void launch_act_quant(const float *x, int64_t m, int64_t k, int64_t x_stride, int8_t *q8, float *scales,
                      cudaStream_t s) {
  int64_t warps = m * ((k + 31) / 32);
  if (!warps) return;
  k_act_quant<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(x, m, k, x_stride, q8, scales);
}

// ---- quantize_row_q8_0 (decode_gemv.rs:294-313): inv = 127/amax ----------
__global__ void k_quantize_row_q8_0(const float *__restrict__ x, int64_t n, uint8_t *__restrict__ blocks) {
  int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (wid >= n / 32) return;
  float v = x[wid * 32 + lane];
  bool fin = isfinite(v);
  float amax = warp_max(fin ? fabsf(v) : 0.0f);
  uint8_t *blk = blocks + wid * 36;
  if (amax == 0.0f || !isfinite(amax)) {
    blk[4 + lane] = 0;
    if (lane == 0) *(float *)blk = 0.0f;
    return;
  }
  float inv = __fdiv_rn(127.0f, amax);
  int8_t q = fin ? act_quant_one(v, inv) : (int8_t)0;
  blk[4 + lane] = (uint8_t)q;
  if (lane == 0) *(float *)blk = __fdiv_rn(amax, 127.0f);
}

void launch_quantize_row_q8_0(const float *x, int64_t n, void *blocks, cudaStream_t s) {
  int64_t warps = n / 32;
  if (!warps) return;
  k_quantize_row_q8_0<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(x, n, (uint8_t *)blocks);
}

// ---- RMSNorm (recipe.rs:2534-2558) ---------------------------------------
__device__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  int w = threadIdx.x / 32, l = threadIdx.x % 32, nw = blockDim.x / 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < nw ? red[l] : 0.0f;
    t = warp_sum(t);
    if (l == 0) red[32] = t;
  }
  __syncthreads();
  float r = red[32];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float rms_inv(float ss, int64_t n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// RMSNorm rows in the reference's order (rmsnorm_row, recipe.rs:2534-2558):
// the sum of squares is the left-to-right f32 sum from -0.0 (computed exactly
// by exact::seq_sum_nonneg over the squares staged in shared memory), then
// inv = 1 / sqrt(sum / n + eps) and out = (x * inv) * w.  One CTA per row.
constexpr int kNormThreads = 256;

__device__ float row_inv_ref(const float *xr, int64_t n, float eps, float *sq) {
  __shared__ exact::SumSmem<kNormThreads> sm;
  for (int64_t i = threadIdx.x; i < n; i += kNormThreads) sq[i] = __fmul_rn(xr[i], xr[i]);
  __syncthreads();
  const float ss = exact::seq_sum_nonneg<kNormThreads>(sq, (int)n, -0.0f, sm);
  return rms_inv(ss, n, eps);
}

__global__ void __launch_bounds__(kNormThreads) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w,
                                                         int64_t n, float eps, float *__restrict__ out) {
  extern __shared__ float sq[];
  const float *xr = x + blockIdx.x * n;
  const float inv = row_inv_ref(xr, n, eps, sq);
  for (int64_t i = threadIdx.x; i < n; i += kNormThreads) out[blockIdx.x * n + i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

constexpr int kNormMaxSmem = 160 * 1024;  // rows up to 40944 elements

static size_t norm_smem(int64_t n) { return ((size_t)n + exact::kSumSlack) * 4; }  // squares + the sum's read slack
static bool norm_fits(int64_t n) { return norm_smem(n) <= (size_t)kNormMaxSmem; }

void launch_rmsnorm(const float *x, const float *w, int64_t m, int64_t n, float eps, float *out, cudaStream_t s) {
  if (!m) return;
  norm_init();
  if (!norm_fits(n)) fail(JAL_ERR_CAPABILITY_MISMATCH, "rmsnorm: row of %lld elements too long", (long long)n);
  k_rmsnorm<<<(unsigned)m, kNormThreads, norm_smem(n), s>>>(x, w, n, eps, out);
}


// One CTA per row: RMSNorm (reference order, as above), then QuantizedActQ8
// per 32-block of the normed row.
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm_quant(const float *__restrict__ x,
                                                               const float *__restrict__ w, int64_t n, float eps,
                                                               int8_t *__restrict__ q8, float *__restrict__ scales) {
  extern __shared__ float sq[];
  const float *xr = x + blockIdx.x * n;
  const float inv = row_inv_ref(xr, n, eps, sq);
  int64_t nb = (n + 31) / 32;
  int lane = threadIdx.x % 32;
  for (int64_t b = threadIdx.x / 32; b < nb; b += kNormThreads / 32) {
    int64_t c = b * 32 + lane;
    float v = c < n ? __fmul_rn(__fmul_rn(xr[c], inv), w[c]) : 0.0f;
    if (!isfinite(v)) v = 0.0f;
    float amax = warp_max(fabsf(v));
    float scale = act_scale_from_amax(amax), qi = act_inv_from_scale(scale);
    q8[blockIdx.x * nb * 32 + c] = c < n ? act_quant_one(v, qi) : (int8_t)0;
    if (lane == 0) scales[blockIdx.x * nb + b] = scale;
  }
}

void norm_init() {
  static bool done = false;
  if (done) return;
  cudaFuncSetAttribute(k_rmsnorm, cudaFuncAttributeMaxDynamicSharedMemorySize, kNormMaxSmem);
  cudaFuncSetAttribute(k_rmsnorm_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, kNormMaxSmem);
  done = true;
}

void launch_rmsnorm_quant(const float *x, const float *w, int64_t m, int64_t n, float eps, int8_t *q8,
                          float *scales, cudaStream_t s) {
  if (!m) return;
  norm_init();
  if (!norm_fits(n)) fail(JAL_ERR_CAPABILITY_MISMATCH, "rmsnorm: row of %lld elements too long", (long long)n);
  k_rmsnorm_quant<<<(unsigned)m, kNormThreads, norm_smem(n), s>>>(x, w, n, eps, q8, scales);
}

// ---- integer 16-element partials (repack_cache.rs:759-762) ---------------
__global__ void k_dot16(DevMat w, const int8_t *__restrict__ q8, int64_t r0, int64_t r1, int32_t *__restrict__ out) {
  int64_t kc = w.cols / 16;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (r1 - r0) * kc) return;
  int64_t r = r0 + idx / kc, ch = idx % kc;
  int32_t dot = 0;
  for (int t = 0; t < 16; t++) dot += (int32_t)q8[ch * 16 + t] * (int32_t)weight_q(w, r, ch * 16 + t);
  out[idx] = dot;
}

void launch_dot16_partials(const DevMat &w, const int8_t *q8, int64_t r0, int64_t r1, int32_t *out, cudaStream_t s) {
  int64_t n = (r1 - r0) * (w.cols / 16);
  if (!n) return;
  k_dot16<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w, q8, r0, r1, out);
}

// ---- streaming raw-GGUF GEMV (decode_gemv.rs:394-439, 622-642) -----------
// One warp per row; each lane takes whole 32-blocks; per-block term
// f32(sumi) * (dw * dx) with the reference's zero short-circuit.
// Lane l evaluates blocks l, l + 32, ...; the block results are added in
// block order through shuffles, so each output equals run_gemv's sequential
// sum (decode_gemv.rs:622-642) bit for bit.
__global__ void k_gemv_raw(const uint8_t *__restrict__ raw, int quant, int64_t rows, int64_t cols,
                           const uint8_t *__restrict__ xb, float *__restrict__ y) {
  int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  int lane = threadIdx.x % 32;
  if (row >= rows) return;  // whole warps leave together
  int64_t nb = cols / 32, bb = quant == JAL_Q4_0 ? 18 : quant == JAL_Q5_0 ? 22 : 34;
  const uint8_t *rp = raw + row * nb * bb;
  float acc = 0.0f;
  for (int64_t b0 = 0; b0 < nb; b0 += 32) {
    const int64_t b = b0 + lane;
    float t = 0.0f;
    if (b < nb) {
      const uint8_t *w = rp + b * bb;
      const uint8_t *xbk = xb + b * 36;
      float dx = *(const float *)xbk;
      const int8_t *xq = (const int8_t *)(xbk + 4);
      float dw = f16_finite((uint16_t)(w[0] | (w[1] << 8)));
      if (dw != 0.0f && dx != 0.0f) {
        int32_t sumi = 0;
        if (quant == JAL_Q4_0) {
          for (int i = 0; i < 16; i++) {
            int32_t q0 = (int32_t)(w[2 + i] & 15) - 8, q1 = (int32_t)(w[2 + i] >> 4) - 8;
            sumi += q0 * xq[i] + q1 * xq[i + 16];
          }
        } else if (quant == JAL_Q5_0) {
          uint32_t qh = (uint32_t)w[2] | ((uint32_t)w[3] << 8) | ((uint32_t)w[4] << 16) | ((uint32_t)w[5] << 24);
          for (int j = 0; j < 16; j++) {
            int32_t h0 = (int32_t)(((qh >> j) & 1u) << 4), h1 = (int32_t)(((qh >> (j + 16)) & 1u) << 4);
            int32_t q0 = ((int32_t)(w[6 + j] & 15) | h0) - 16, q1 = ((int32_t)(w[6 + j] >> 4) | h1) - 16;
            sumi += q0 * xq[j] + q1 * xq[j + 16];
          }
        } else {
          for (int i = 0; i < 32; i++) sumi += (int32_t)(int8_t)w[2 + i] * xq[i];
        }
        t = __fmul_rn((float)sumi, __fmul_rn(dw, dx));
      }
    }
    for (int k = 0; k < 32; k++) {
      const float v = __shfl_sync(0xffffffffu, t, k);
      if (b0 + k < nb) acc = __fadd_rn(acc, v);
    }
  }
  if (lane == 0) y[row] = acc;
}

void launch_gemv_raw(const uint8_t *raw, int quant, int64_t rows, int64_t cols, const void *xblocks, float *y,
                     cudaStream_t s) {
  if (!rows) return;
  k_gemv_raw<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(raw, quant, rows, cols, (const uint8_t *)xblocks, y);
}

// ---- embedding gather (recipe.rs:1395-1440, repack_cache.rs:1244-1301) ---
__global__ void k_embed(const uint8_t *__restrict__ emb, int quant, int64_t hidden, int64_t vocab,
                        const uint32_t *__restrict__ tokens, float *__restrict__ out, int *err_flag, int pdl) {
  if (pdl) pdl_wait();
  uint32_t tok = tokens[blockIdx.x];
  float *o = out + (int64_t)blockIdx.x * hidden;
  if (tok >= vocab) {
    if (threadIdx.x == 0 && err_flag) atomicOr(err_flag, 1);
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = 0.0f;
    if (pdl) pdl_trigger();
    return;
  }
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = embed_value(emb, quant, hidden, tok, i);
  if (pdl) pdl_trigger();
}

void launch_embed(const uint8_t *emb_raw, int quant, int64_t hidden, int64_t vocab, const uint32_t *tokens, int64_t m,
                  float *out, int *err_flag, int pdl, cudaStream_t s) {
  if (!m) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_embed, emb_raw, quant, hidden, vocab, tokens, out, err_flag, pdl);
}

}  // namespace jal
