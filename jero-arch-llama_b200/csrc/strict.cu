// Reference-order decode kernels (JAL_NUMERICS_REFERENCE).
//
// The fast decode path reorders f32 reductions (tree sums, fused multiply
// adds, per-32-block terms, CUDA's expf).  The int8 activation quantizer
// makes the model output discontinuous in its inputs, so a one-ulp change
// can flip a rounding and move logits by ~1e-2 a few layers later.  These
// kernels reproduce the reference's f32 operation order exactly so a whole
// decode run can be compared with the CPU oracle:
//   - RMSNorm: sum of squares from -0.0 in element order, inv = 1 /
//     sqrt(sum / n + eps), out = (x * inv) * w (or_rmsnorm_row,
//     recipe.rs rmsnorm_row);
//   - projections: acc += (f32(dot16) * a_sc) * w_sc over 16-element chunks
//     in order, no fused multiply-add (repack_cache.rs:715-785);
//   - attention: sequential q.k from -0.0, exp(s - max), sequential
//     denominator, out[e] += (p * inv) * v[e] in position order
//     (recipe.rs:2949-3022);
//   - SwiGLU: (g * (1 / (1 + exp(-g)))) * u with the +-20 clamps
//     (recipe.rs:3037-3047).
// exp is glibc's expf evaluation (libm_expf.h), which the reference calls.
#include <cuda_fp16.h>

#include "dev_util.cuh"
#include "device.hpp"
#include "libm_expf.h"
#include "jal.h"

namespace jal {

namespace {

__device__ __forceinline__ float exp_ref(float x) { return libm::expf_ref(x); }

__global__ void k_strict_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, int64_t n, float eps,
                                 float *__restrict__ out) {
  __shared__ float inv_s;
  if (threadIdx.x == 0) {
    float ss = -0.0f;
    for (int64_t i = 0; i < n; i++) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
    inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  }
  __syncthreads();
  const float inv = inv_s;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// One warp per row: lane l forms the two 16-element chunk terms of blocks
// l, l+32, ... into shared memory, then lane 0 adds them in chunk order.
template <int QUANT>
__global__ void k_strict_gemv(const DevMat w, const int8_t *__restrict__ q8, const float *__restrict__ asc,
                              int64_t rows, int add, float *__restrict__ y, const float *__restrict__ bias) {
  extern __shared__ float terms[];  // [warps][2 * nb]
  const int nb = (int)(w.cols / 32), warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int W = blockDim.x / 32;
  float *tw = terms + (size_t)warp * 2 * nb;
  for (int64_t r = (int64_t)blockIdx.x * W + warp; r < rows; r += (int64_t)gridDim.x * W) {
    const uint8_t *qrow = w.qs + r * w.qs_stride;
    const uint16_t *drow = w.d + r * w.d_stride;
    for (int b = lane; b < nb; b += 32) {
      const int4 alo = *(const int4 *)(q8 + b * 32), ahi = *(const int4 *)(q8 + b * 32 + 16);
      const float ws = __half2float(__ushort_as_half(drow[b])), as = asc[b];
      int d0, d1;
      if (QUANT == JAL_Q4_0) {
        const uint4 v = *(const uint4 *)(qrow + b * 16);
        d0 = dp4a_us(v.x & 0x0F0F0F0Fu, alo.x, 0);
        d0 = dp4a_us(v.y & 0x0F0F0F0Fu, alo.y, d0);
        d0 = dp4a_us(v.z & 0x0F0F0F0Fu, alo.z, d0);
        d0 = dp4a_us(v.w & 0x0F0F0F0Fu, alo.w, d0);
        d1 = dp4a_us(v.x & 0xF0F0F0F0u, ahi.x, 0);
        d1 = dp4a_us(v.y & 0xF0F0F0F0u, ahi.y, d1);
        d1 = dp4a_us(v.z & 0xF0F0F0F0u, ahi.z, d1);
        d1 = dp4a_us(v.w & 0xF0F0F0F0u, ahi.w, d1);
        int s0 = dp4a_ss(alo.x, 0x01010101, 0), s1 = dp4a_ss(ahi.x, 0x01010101, 0);
        s0 = dp4a_ss(alo.y, 0x01010101, s0);
        s1 = dp4a_ss(ahi.y, 0x01010101, s1);
        s0 = dp4a_ss(alo.z, 0x01010101, s0);
        s1 = dp4a_ss(ahi.z, 0x01010101, s1);
        s0 = dp4a_ss(alo.w, 0x01010101, s0);
        s1 = dp4a_ss(ahi.w, 0x01010101, s1);
        d0 -= 8 * s0;              // nibble n encodes n - 8
        d1 = (d1 >> 4) - 8 * s1;   // high nibbles were multiplied by 16 in place
      } else {
        const uint4 v0 = *(const uint4 *)(qrow + b * 32), v1 = *(const uint4 *)(qrow + b * 32 + 16);
        d0 = dp4a_ss((int)v0.x, alo.x, 0);
        d0 = dp4a_ss((int)v0.y, alo.y, d0);
        d0 = dp4a_ss((int)v0.z, alo.z, d0);
        d0 = dp4a_ss((int)v0.w, alo.w, d0);
        d1 = dp4a_ss((int)v1.x, ahi.x, 0);
        d1 = dp4a_ss((int)v1.y, ahi.y, d1);
        d1 = dp4a_ss((int)v1.z, ahi.z, d1);
        d1 = dp4a_ss((int)v1.w, ahi.w, d1);
      }
      tw[2 * b] = __fmul_rn(__fmul_rn(__int2float_rn(d0), as), ws);
      tw[2 * b + 1] = __fmul_rn(__fmul_rn(__int2float_rn(d1), as), ws);
    }
    __syncwarp();
    if (lane == 0) {
      float acc = 0.0f;
      for (int c = 0; c < 2 * nb; c++) acc = __fadd_rn(acc, tw[c]);
      const float p = bias ? __fadd_rn(acc, bias[r]) : acc;
      y[r] = add ? __fadd_rn(y[r], p) : p;
    }
    __syncwarp();
  }
}

__global__ void k_strict_swiglu(const float *__restrict__ g, const float *__restrict__ u, int64_t n,
                                float *__restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = g[i];
  const float sig = x <= -20.0f ? 0.0f : (x >= 20.0f ? 1.0f : __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_ref(-x))));
  out[i] = __fmul_rn(__fmul_rn(x, sig), u[i]);
}

__device__ __forceinline__ int64_t kv_index(const KvView &kv, int64_t layer, int64_t h, int64_t pos) {
  const int64_t page = kv.page_table[pos / kv.page_size], slot = pos % kv.page_size;
  return (((layer * kv.n_pages + page) * kv.n_kv + h) * kv.page_size + slot) * kv.head_dim;
}

// q (+ bias, RoPE) into qbuf; new k (+ bias, RoPE) and v (+ bias) appended
// to the cache at the current position (recipe.rs:2319-2326).
__global__ void k_strict_qkv_prep(const StrictQkvArgs a) {
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t HD = a.kv.head_dim, Q = a.n_heads_q * HD, KVD = a.kv.n_kv * HD;
  const bool rope = !a.skip_rope && pos > 0;
  const int64_t half = a.rotary_dim / 2;
  const bool use_long = a.long_threshold >= 0 && seq > a.long_threshold;
  const float *ct = (use_long ? a.cos_tab_long : a.cos_tab) + pos * half;
  const float *st = (use_long ? a.sin_tab_long : a.sin_tab) + pos * half;
  for (int64_t i = threadIdx.x; i < Q + 2 * KVD; i += blockDim.x) {
    const int region = i < Q ? 0 : (i < Q + KVD ? 1 : 2);
    const int64_t base = region == 0 ? 0 : (region == 1 ? Q : Q + KVD);
    const float *bias = region == 0 ? a.bq : (region == 1 ? a.bk : a.bv);
    const int64_t li = i - base, hh = li / HD, d = li % HD;
    auto ld = [&](int64_t dd) {
      const float x = a.qkv[base + hh * HD + dd];
      return bias ? __fadd_rn(x, bias[hh * HD + dd]) : x;
    };
    float o = ld(d);
    if (rope && region < 2 && d < 2 * half) {
      const bool first = a.neox ? d < half : (d & 1) == 0;
      const int64_t j = a.neox ? (first ? d : d - half) : d / 2;
      const int64_t partner = a.neox ? (first ? d + half : d - half) : (d ^ 1);
      const float other = ld(partner), c = ct[j], s = st[j];
      const float x0 = first ? o : other, x1 = first ? other : o;
      o = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)) : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    if (region == 0) {
      a.qbuf[i] = o;
    } else {
      const int64_t e = kv_index(a.kv, a.layer, hh, pos) + d;
      void *dst = region == 1 ? a.kv.k : a.kv.v;
      if (a.kv.f16) ((__half *)dst)[e] = __float2half_rn(o);
      else ((float *)dst)[e] = o;
    }
  }
}

__device__ __forceinline__ float kv_load(const KvView &kv, const void *base, int64_t e) {
  return kv.f16 ? __half2float(((const __half *)base)[e]) : ((const float *)base)[e];
}

// One CTA per query head (gqa_attention_prefill_portable for one token).
__global__ void k_strict_attn(const StrictAttnArgs a) {
  extern __shared__ float sc[];  // scores, then probabilities, of the active positions
  __shared__ float red[2];
  const int64_t HD = a.kv.head_dim, hq = blockIdx.x, G = a.n_heads_q / a.kv.n_kv, hkv = hq / G;
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t vstart = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t active = seq - vstart;
  const float *qh = a.qbuf + hq * HD;
  for (int64_t i = threadIdx.x; i < active; i += blockDim.x) {
    const int64_t e0 = kv_index(a.kv, a.layer, hkv, vstart + i);
    float d = -0.0f;
    for (int64_t e = 0; e < HD; e++) d = __fadd_rn(d, __fmul_rn(qh[e], kv_load(a.kv, a.kv.k, e0 + e)));
    sc[i] = __fmul_rn(d, a.scale);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int64_t i = 0; i < active; i++)
      if (sc[i] > m) m = sc[i];
    red[0] = m;
  }
  __syncthreads();
  const float maxs = red[0];
  for (int64_t i = threadIdx.x; i < active; i += blockDim.x) sc[i] = exp_ref(__fsub_rn(sc[i], maxs));
  __syncthreads();
  if (threadIdx.x == 0) {
    float den = 0.0f;
    for (int64_t i = 0; i < active; i++) den = __fadd_rn(den, sc[i]);
    red[1] = den > 0.0f ? __fdiv_rn(1.0f, den) : 0.0f;
  }
  __syncthreads();
  const float inv = red[1];
  for (int64_t e = threadIdx.x; e < HD; e += blockDim.x) {
    float o = 0.0f;
    for (int64_t i = 0; i < active; i++) {
      const float wgt = __fmul_rn(sc[i], inv);
      o = __fadd_rn(o, __fmul_rn(wgt, kv_load(a.kv, a.kv.v, kv_index(a.kv, a.layer, hkv, vstart + i) + e)));
    }
    a.out[hq * HD + e] = o;
  }
}

__global__ void k_set_token_pos(uint32_t *d_token, uint32_t token, int64_t *d_pos, int64_t pos) {
  *d_token = token;
  *d_pos = pos;
}

}  // namespace

void launch_set_token_pos(uint32_t *d_token, uint32_t token, int64_t *d_pos, int64_t pos, cudaStream_t s) {
  k_set_token_pos<<<1, 1, 0, s>>>(d_token, token, d_pos, pos);
}

void launch_strict_rmsnorm(const float *x, const float *w, int64_t n, float eps, float *out, cudaStream_t s) {
  k_strict_rmsnorm<<<1, 256, 0, s>>>(x, w, n, eps, out);
}

size_t strict_gemv_smem(int64_t cols) { return (size_t)8 * 2 * (size_t)(cols / 32) * sizeof(float); }

void launch_strict_gemv(const DevMat &w, const int8_t *q8, const float *scales, int64_t rows, bool add, float *y,
                        const float *bias, cudaStream_t s) {
  if (rows <= 0) return;
  const size_t smem = strict_gemv_smem(w.cols);
  const int64_t blocks64 = (rows + 7) / 8;
  const unsigned blocks = (unsigned)(blocks64 < 1184 ? blocks64 : 1184);
  if (w.quant == JAL_Q4_0) {
    cudaFuncSetAttribute(k_strict_gemv<JAL_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_strict_gemv<JAL_Q4_0><<<blocks, 256, smem, s>>>(w, q8, scales, rows, add ? 1 : 0, y, bias);
  } else {
    cudaFuncSetAttribute(k_strict_gemv<JAL_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_strict_gemv<JAL_Q8_0><<<blocks, 256, smem, s>>>(w, q8, scales, rows, add ? 1 : 0, y, bias);
  }
}

void launch_strict_swiglu(const float *g, const float *u, int64_t n, float *out, cudaStream_t s) {
  if (n <= 0) return;
  k_strict_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, u, n, out);
}

void launch_strict_qkv_prep(const StrictQkvArgs &a, cudaStream_t s) { k_strict_qkv_prep<<<1, 256, 0, s>>>(a); }

void launch_strict_attn(const StrictAttnArgs &a, int64_t n_ctx, cudaStream_t s) {
  const size_t smem = (size_t)n_ctx * sizeof(float);
  cudaFuncSetAttribute(k_strict_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_strict_attn<<<(unsigned)a.n_heads_q, 128, smem, s>>>(a);
}

}  // namespace jal
