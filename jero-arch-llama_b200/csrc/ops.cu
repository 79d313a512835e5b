// Element-wise and reduction ops: RoPE over rows, SwiGLU, the reference-form
// GQA attention over contiguous f32 planes (op-level entry point), and the
// greedy argmax that closes a decode step on the device.
#include "dev_util.cuh"
#include "device.hpp"
#include "exact.cuh"
#include "jal.h"

namespace jal {

namespace {

// apply_rope_compat (recipe.rs:2775-2834): angle = f32(pos) * inv_freq[i].
__global__ void k_rope_rows(float *qk, int64_t row_len, int64_t head_dim, int64_t rotary_dim, int neox, int64_t pos0,
                            const float *inv_freq) {
  const int64_t t = blockIdx.x, pos = pos0 + t;
  if (pos == 0) return;
  const int64_t half = rotary_dim / 2, heads = row_len / head_dim;
  float *row = qk + t * row_len;
  const float p = (float)pos;
  for (int64_t i = threadIdx.x; i < heads * half; i += blockDim.x) {
    int64_t h = i / half, j = i % half;
    float s, c;
    sincosf(__fmul_rn(p, inv_freq[j]), &s, &c);
    float *hr = row + h * head_dim;
    int64_t i0 = neox ? j : 2 * j, i1 = neox ? j + half : 2 * j + 1;
    float x0 = hr[i0], x1 = hr[i1];
    hr[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    hr[i1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
}

// swiglu_compat (recipe.rs:3037-3047) with the reference's exp.
__device__ __forceinline__ float swiglu1(float g, float u) { return exact::swiglu_ref(g, u); }

__global__ void k_swiglu(const float *g, const float *u, int64_t n, float *out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = swiglu1(g[i], u[i]);
}

// SwiGLU of m rows of gate | up (row stride `stride`) straight into the
// QuantizedActQ8 blocks of the next projection: the element values are
// swiglu1's and the per-block quantization is k_act_quant's (repack_cache.rs:
// 390-422), without an f32 row in between.  One warp per (row, 32-block).
__global__ void k_swiglu_act_quant(const float *__restrict__ gu, int64_t m, int64_t f, int64_t stride,
                                   int8_t *__restrict__ q8, float *__restrict__ scales) {
  const int64_t nb = (f + 31) / 32;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (wid >= m * nb) return;  // whole warps leave together
  const int64_t t = wid / nb, b = wid % nb, c = b * 32 + lane;
  float v = c < f ? swiglu1(gu[t * stride + c], gu[t * stride + f + c]) : 0.0f;
  if (!isfinite(v)) v = 0.0f;
  const float amax = warp_max(fabsf(v));
  const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
  q8[t * nb * 32 + c] = c < f ? act_quant_one(v, inv) : (int8_t)0;
  if (lane == 0) scales[t * nb + b] = scale;
}

// gqa_attention_prefill_portable (recipe.rs:2949-3022) in the reference's f32
// order, one CTA per (token, query head); scores of the visible positions are
// kept in shared memory.  Scores: sequential q.k from -0.0 then * scale; max;
// e = exp(s - max); den = sequential sum (exact::seq_sum_nonneg); output
// chains out[e] = sum over positions of (p * inv) * v in position order.
constexpr int kGqaThreads = 128;
__global__ void __launch_bounds__(kGqaThreads) k_gqa_ref(const float *q, const float *k, const float *v, int64_t nq,
                                                        int64_t nkv, int64_t hd, int64_t total_seq, int64_t start_pos,
                                                        int64_t window, float scale, float *out) {
  extern __shared__ float sc[];
  __shared__ float red[33];
  __shared__ exact::SumSmem<kGqaThreads> ssm;
  const int64_t tok = blockIdx.x, hq = blockIdx.y, group = nq / nkv, hkv = hq / group;
  const int64_t kvs = nkv * hd, qpos = start_pos + tok;
  const int64_t vend = qpos + 1 < total_seq ? qpos + 1 : total_seq;
  const int64_t vstart = window > 0 ? (qpos + 1 > window ? qpos + 1 - window : 0) : 0;
  const int64_t n = vend > vstart ? vend - vstart : 0;
  const float *qh = q + (tok * nq + hq) * hd;
  float mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += kGqaThreads) {
    const float *kh = k + (vstart + i) * kvs + hkv * hd;
    float d = -0.0f;
    for (int64_t e = 0; e < hd; e++) d = __fadd_rn(d, __fmul_rn(qh[e], kh[e]));
    const float s = __fmul_rn(d, scale);
    sc[i] = s;
    if (s > mx) mx = s;
  }
  mx = warp_max(mx);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int i = 0; i < kGqaThreads / 32; i++)
      if (red[i] > m) m = red[i];
    red[32] = m;
  }
  __syncthreads();
  mx = red[32];
  for (int64_t i = threadIdx.x; i < n; i += kGqaThreads) sc[i] = exact::exp_ref(__fsub_rn(sc[i], mx));
  __syncthreads();
  const float denom = exact::seq_sum_nonneg<kGqaThreads>(sc, (int)n, 0.0f, ssm);
  const float inv = denom > 0.0f ? __fdiv_rn(1.0f, denom) : 0.0f;
  float *oh = out + (tok * nq + hq) * hd;
  for (int64_t e = threadIdx.x; e < hd; e += kGqaThreads) {
    float o = 0.0f;
    for (int64_t i = 0; i < n; i++) o = __fadd_rn(o, __fmul_rn(__fmul_rn(sc[i], inv), v[(vstart + i) * kvs + hkv * hd + e]));
    oh[e] = o;
  }
}

// Greedy argmax with lowest-index tie break.  Each CTA reduces a slice; the
// last CTA (atomic counter) reduces the slice winners, stores the token and
// advances the device position.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void k_argmax(const float *logits, int64_t n, float *pv, int *pi, unsigned *cnt, uint32_t *token_out,
                         int64_t *d_pos, uint32_t *hist, int pdl, uint32_t *epoch) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ bool last;
  if (pdl) pdl_wait();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = logits[i];
    if (v != v) v = -INFINITY;
    if (better(v, (int)i, bv, bi)) { bv = v; bi = (int)i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x / 32); k++)
      if (better(sv[k], si[k], bv, bi)) { bv = sv[k]; bi = si[k]; }
    pv[blockIdx.x] = bv;
    pi[blockIdx.x] = bi;
    __threadfence();
    last = atomicAdd(cnt, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) {
    if (pdl) pdl_trigger();
    return;
  }
  // The last CTA reduces the per-CTA winners with all its threads at once.
  __threadfence();
  float fv = -INFINITY;
  int fi = 0x7fffffff;
  for (unsigned k = threadIdx.x; k < gridDim.x; k += blockDim.x) {
    float v = __ldcg(pv + k);
    int i = __ldcg(pi + k);
    if (better(v, i, fv, fi)) { fv = v; fi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, fv, o);
    int oi = __shfl_xor_sync(0xffffffffu, fi, o);
    if (better(ov, oi, fv, fi)) { fv = ov; fi = oi; }
  }
  __syncthreads();
  if (l == 0) { sv[w] = fv; si[w] = fi; }
  __syncthreads();
  if (threadIdx.x != 0) {
    if (pdl) pdl_trigger();
    return;
  }
  for (int k = 1; k < (int)(blockDim.x / 32); k++)
    if (better(sv[k], si[k], fv, fi)) { fv = sv[k]; fi = si[k]; }
  const uint32_t tok = (uint32_t)(fi == 0x7fffffff ? 0 : fi);
  *token_out = tok;
  if (d_pos) {
    if (hist) hist[*d_pos + 1] = tok;  // token of the next position
    *d_pos += 1;
  }
  if (epoch) *epoch += 1u;  // tensor-parallel exchange: the next step's flags
  *cnt = 0u;
  if (pdl) pdl_trigger();
}

}  // namespace

void launch_rope_rows(float *qk, int64_t m, int64_t row_len, int64_t head_dim, int64_t rotary_dim, int neox,
                      int64_t pos0, const float *inv_freq, cudaStream_t s) {
  if (!m) return;
  k_rope_rows<<<(unsigned)m, 256, 0, s>>>(qk, row_len, head_dim, rotary_dim, neox, pos0, inv_freq);
}

void launch_swiglu(const float *g, const float *u, int64_t n, float *out, cudaStream_t s) {
  if (!n) return;
  k_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, u, n, out);
}

void launch_swiglu_act_quant(const float *gu, int64_t m, int64_t f, int64_t stride, int8_t *q8, float *scales,
                             cudaStream_t s) {
  const int64_t warps = m * ((f + 31) / 32);
  if (!warps) return;
  k_swiglu_act_quant<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(gu, m, f, stride, q8, scales);
}

void launch_gqa_attention_ref(const float *q, const float *k, const float *v, int64_t m, int64_t nq, int64_t nkv,
                              int64_t hd, int64_t total_seq, int64_t start_pos, int64_t window, float scale,
                              float *out, cudaStream_t s) {
  if (!m) return;
  size_t smem = ((size_t)total_seq + exact::kSumSlack) * sizeof(float);  // scores + the sum's read slack
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_gqa_ref, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_gqa_ref<<<dim3((unsigned)m, (unsigned)nq), 128, smem, s>>>(q, k, v, nq, nkv, hd, total_seq, start_pos, window,
                                                              scale, out);
}

void launch_argmax(const float *logits, int64_t n, float *part_val, int *part_idx, unsigned *cnt, int n_blocks,
                   uint32_t *token_out, int64_t *d_pos, uint32_t *hist, int pdl, cudaStream_t s, uint32_t *epoch) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_argmax, logits, n, part_val, part_idx, cnt, token_out, d_pos, hist, pdl, epoch);
}

}  // namespace jal
