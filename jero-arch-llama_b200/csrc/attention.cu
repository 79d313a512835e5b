// Attention kernels over the paged KV cache.
//
// Decode (one token): split-K ("flash decoding") over the sequence with one
// thread-block cluster per KV head.  Each CTA of the cluster loads the head
// group's queries from the QKV projection output, adds the optional biases,
// applies RoPE, scores its slice of positions and keeps an online softmax.
// The CTA whose slice holds the current position appends the new K/V.  The
// split partials are merged through distributed shared memory (no global
// round trip); every rank finalises and quantizes a share of the 32-blocks
// of the head outputs for the output projection.
// Math follows gqa_attention_prefill_portable (recipe.rs:2949-3022) up to the
// order of f32 sums: score = (q . k) * scale, exp(s - max), sum, weighted V.
//
// Prefill: RoPE + KV append of m tokens, then a causal flash kernel with f32
// accumulation.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kSub = 128;  // positions per sub-chunk
constexpr int kMaxG = 8;   // query heads per KV head
constexpr int kMaxClusterCtas = 16;  // CTAs per KV head (one cluster)

__device__ __forceinline__ int64_t kv_elem(const KvView &kv, int64_t layer, int64_t h, int64_t pos) {
  int64_t page = kv.page_table[pos / kv.page_size], slot = pos % kv.page_size;
  return (((layer * kv.n_pages + page) * kv.n_kv + h) * kv.page_size + slot) * kv.head_dim;
}

__device__ __forceinline__ void store_kv(void *base, int f16, int64_t e, float v) {
  if (f16) ((__half *)base)[e] = __float2half_rn(v);
  else ((float *)base)[e] = v;
}

// Rotate pair (x0, x1) by (c, s): recipe.rs:2750-2767.
__device__ __forceinline__ void rot(float &x0, float &x1, float c, float s) {
  float a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  float b = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  x0 = a;
  x1 = b;
}

template <int HD, bool F16>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnDecodeArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float q_s[kMaxG][HD];
  __shared__ float kn_s[HD], vn_s[HD];
  __shared__ float p_s[kMaxG][kSub];
  __shared__ float red_s[4][kMaxG];
  __shared__ float alpha_s[kMaxG];
  __shared__ float acc_s[4][kMaxG][HD];  // acc_s[0] holds this CTA's partial after the reduction
  __shared__ float ml_s[2][kMaxG];       // running max / denominator of this CTA
  __shared__ float wgt_s[kMaxClusterCtas][kMaxG];
  __shared__ float den_s[kMaxG];
  const int cs = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
  const int h = blockIdx.x / cs, tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int G = (int)(a.n_heads_q / a.kv.n_kv);
  const int64_t Q = a.n_heads_q * HD, KVD = a.kv.n_kv * HD;

  pdl_wait();
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t span = seq - lo, per = (span + cs - 1) / cs;
  const int64_t s0 = lo + rank * per, s1 = s0 + per < seq ? s0 + per : seq;

  // q / new k / new v of this head group (+ bias), then RoPE.
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    int g = i / HD, d = i % HD;
    int64_t e = (int64_t)(h * G + g) * HD + d;
    q_s[g][d] = a.bq ? __fadd_rn(a.qkv[e], a.bq[e]) : a.qkv[e];
  }
  for (int d = tid; d < HD; d += kAttnThreads) {
    int64_t ek = (int64_t)h * HD + d;
    kn_s[d] = a.bk ? __fadd_rn(a.qkv[Q + ek], a.bk[ek]) : a.qkv[Q + ek];
    vn_s[d] = a.bv ? __fadd_rn(a.qkv[Q + KVD + ek], a.bv[ek]) : a.qkv[Q + KVD + ek];
  }
  __syncthreads();
  if (!a.skip_rope && pos > 0) {
    const int half = (int)(a.rotary_dim / 2);
    const bool use_long = a.long_threshold >= 0 && seq > a.long_threshold;
    const float *ct = (use_long ? a.cos_tab_long : a.cos_tab) + pos * half;
    const float *st = (use_long ? a.sin_tab_long : a.sin_tab) + pos * half;
    for (int i = tid; i < (G + 1) * half; i += kAttnThreads) {
      int g = i / half, j = i % half;
      float *row = g < G ? q_s[g] : kn_s;
      int i0 = a.neox ? j : 2 * j, i1 = a.neox ? j + half : 2 * j + 1;
      float x0 = row[i0], x1 = row[i1];
      rot(x0, x1, ct[j], st[j]);
      row[i0] = x0;
      row[i1] = x1;
    }
    __syncthreads();
  }
  // Append the new K/V (recipe.rs:2319-2326) from the CTA owning `pos`.
  if (pos >= s0 && pos < s1) {
    int64_t e = kv_elem(a.kv, a.layer, h, pos);
    for (int d = tid; d < HD; d += kAttnThreads) {
      store_kv(a.kv.k, a.kv.f16, e + d, kn_s[d]);
      store_kv(a.kv.v, a.kv.f16, e + d, vn_s[d]);
    }
  }

  float m_run[kMaxG], l_run[kMaxG];
  constexpr int DPL = HD / 32;  // dims per lane in the PV phase
  float acc[kMaxG][DPL];
#pragma unroll
  for (int g = 0; g < kMaxG; g++) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; j++) acc[g][j] = 0.0f;
  }

  for (int64_t c0 = s0; c0 < s1; c0 += kSub) {
    const int n = (int)(s1 - c0 < kSub ? s1 - c0 : kSub);
    // Phase 1: scores, one position per thread, K streamed 8 dims at a time.
    if (tid < n) {
      const int64_t s = c0 + tid;
      float dot[kMaxG];
#pragma unroll
      for (int g = 0; g < kMaxG; g++) dot[g] = 0.0f;
      const bool fresh = s == pos;
      const int64_t e = fresh ? 0 : kv_elem(a.kv, a.layer, h, s);
#pragma unroll 4
      for (int j = 0; j < HD / 8; j++) {
        float kr[8];
        if (fresh) {
#pragma unroll
          for (int k = 0; k < 8; k++) kr[k] = kn_s[j * 8 + k];
        } else if (F16) {
          uint4 v = *((const uint4 *)((const __half *)a.kv.k + e) + j);
          const __half2 *hv = (const __half2 *)&v;
#pragma unroll
          for (int k = 0; k < 4; k++) {
            float2 f = __half22float2(hv[k]);
            kr[2 * k] = f.x;
            kr[2 * k + 1] = f.y;
          }
        } else {
          const float4 *fp = (const float4 *)((const float *)a.kv.k + e) + 2 * j;
          float4 v0 = fp[0], v1 = fp[1];
          kr[0] = v0.x; kr[1] = v0.y; kr[2] = v0.z; kr[3] = v0.w;
          kr[4] = v1.x; kr[5] = v1.y; kr[6] = v1.z; kr[7] = v1.w;
        }
#pragma unroll
        for (int g = 0; g < kMaxG; g++) {
          if (g < G) {
#pragma unroll
            for (int k = 0; k < 8; k++) dot[g] = fmaf(q_s[g][j * 8 + k], kr[k], dot[g]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxG; g++)
        if (g < G) p_s[g][tid] = __fmul_rn(dot[g], a.scale);
    }
    __syncthreads();
    // Phase 2: chunk max per head, rescale factors, probabilities.
    float cm[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      float v = (g < G && tid < n) ? p_s[g][tid] : -INFINITY;
      cm[g] = warp_max(v);
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < kMaxG; g++) red_s[warp][g] = cm[g];
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      float mx = fmaxf(fmaxf(red_s[0][g], red_s[1][g]), fmaxf(red_s[2][g], red_s[3][g]));
      float mn = fmaxf(m_run[g], mx);
      float al = (m_run[g] == -INFINITY) ? 0.0f : expf(m_run[g] - mn);
      if (tid == 0 && g < G) alpha_s[g] = al;
      m_run[g] = mn;
      cm[g] = mn;
    }
    __syncthreads();
    float ps[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      float p = 0.0f;
      if (g < G && tid < n) {
        p = expf(p_s[g][tid] - cm[g]);
        p_s[g][tid] = p;
      }
      ps[g] = warp_sum(p);
    }
    __syncthreads();
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < kMaxG; g++) red_s[warp][g] = ps[g];
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kMaxG; g++) {
      if (g < G) {
        float al = alpha_s[g];
        l_run[g] = l_run[g] * al + ((red_s[0][g] + red_s[1][g]) + (red_s[2][g] + red_s[3][g]));
#pragma unroll
        for (int j = 0; j < DPL; j++) acc[g][j] *= al;
      }
    }
    // Phase 3: P.V, warp w takes positions w, w+4, ...; lane owns DPL dims.
    for (int t = warp; t < n; t += 4) {
      const int64_t s = c0 + t;
      float vr[DPL];
      if (s == pos) {
#pragma unroll
        for (int j = 0; j < DPL; j++) vr[j] = vn_s[lane * DPL + j];
      } else {
        int64_t e = kv_elem(a.kv, a.layer, h, s) + lane * DPL;
        if (F16) {
          const __half2 *vp = (const __half2 *)((const __half *)a.kv.v + e);
#pragma unroll
          for (int j = 0; j < DPL / 2; j++) {
            float2 f = __half22float2(vp[j]);
            vr[2 * j] = f.x;
            vr[2 * j + 1] = f.y;
          }
        } else {
          const float2 *vp = (const float2 *)((const float *)a.kv.v + e);
#pragma unroll
          for (int j = 0; j < DPL / 2; j++) {
            float2 f = vp[j];
            vr[2 * j] = f.x;
            vr[2 * j + 1] = f.y;
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxG; g++) {
        if (g < G) {
          float p = p_s[g][t];
#pragma unroll
          for (int j = 0; j < DPL; j++) acc[g][j] = fmaf(p, vr[j], acc[g][j]);
        }
      }
    }
    __syncthreads();
  }

  // Reduce the 4 warps' accumulators into acc_s[0]: this CTA's partial.
#pragma unroll
  for (int g = 0; g < kMaxG; g++)
    if (g < G) {
#pragma unroll
      for (int j = 0; j < DPL; j++) acc_s[warp][g][lane * DPL + j] = acc[g][j];
    }
  if (tid < G) {
    float mg = -INFINITY, lg = 0.0f;
#pragma unroll
    for (int g = 0; g < kMaxG; g++)
      if (g == tid) { mg = m_run[g]; lg = l_run[g]; }
    ml_s[0][tid] = mg;
    ml_s[1][tid] = lg;
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    int g = i / HD, d = i % HD;
    acc_s[0][g][d] = (acc_s[0][g][d] + acc_s[1][g][d]) + (acc_s[2][g][d] + acc_s[3][g][d]);
  }
  cluster.sync();
  // Merge the cluster's partials through distributed shared memory:
  // out = sum_r e^(m_r - M) acc_r / sum_r e^(m_r - M) l_r.  Every remote
  // read of a phase is issued independently (one DSMEM round trip each).
  if (tid < cs * G) {
    const int r = tid / G, g = tid % G;
    wgt_s[r][g] = cluster.map_shared_rank(&ml_s[0][0], r)[g];
    p_s[g][r] = cluster.map_shared_rank(&ml_s[1][0], r)[g];  // l_r, staged in p_s (free now)
  }
  __syncthreads();
  if (tid < G) {
    float M = -INFINITY;
    for (int r = 0; r < cs; r++) M = fmaxf(M, wgt_s[r][tid]);
    float den = 0.0f;
    for (int r = 0; r < cs; r++) {
      const float mr = wgt_s[r][tid];
      const float w = mr == -INFINITY ? 0.0f : expf(mr - M);
      wgt_s[r][tid] = w;
      den = fmaf(w, p_s[tid][r], den);
    }
    den_s[tid] = den;
  }
  __syncthreads();
  // Rank r finalises 32-blocks r, r + cs, ... of this head group and
  // quantizes them (QuantizedActQ8; head boundaries are 32-aligned).
  for (int bi = rank + warp * cs; bi < G * HD / 32; bi += 4 * cs) {
    const int e = bi * 32 + lane, g = e / HD, d = e % HD;
    float part[kMaxClusterCtas];
#pragma unroll
    for (int r = 0; r < kMaxClusterCtas; r++)
      part[r] = r < cs ? cluster.map_shared_rank(&acc_s[0][0][0], r)[g * HD + d] : 0.0f;
    float num = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxClusterCtas; r++)
      if (r < cs) num = fmaf(wgt_s[r][g], part[r], num);
    float o = den_s[g] > 0.0f ? __fdiv_rn(num, den_s[g]) : 0.0f;
    a.out[(int64_t)h * G * HD + e] = o;
    if (!isfinite(o)) o = 0.0f;
    const float amax = warp_max(fabsf(o));
    const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
    const int64_t gb = ((int64_t)h * G * HD) / 32 + bi;
    a.out_q[gb * 32 + lane] = act_quant_one(o, inv);
    if (lane == 0) a.out_s[gb] = scale;
  }
  // Keep this CTA's shared memory alive until every rank has read it.
  cluster.sync();
  pdl_trigger();
}

template <int HD, bool F16>
void launch_decode_t(const AttnDecodeArgs &a, cudaStream_t s) {
  auto kern = k_attn_decode<HD, F16>;
  const int cs = a.n_splits;
  if (cs > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.kv.n_kv * cs));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, a);
}

// ---- prefill: bias + RoPE + KV append -------------------------------------
__global__ void k_rope_append(const RopeAppendArgs a) {
  const int64_t t = blockIdx.x, pos = a.start_pos + t;
  const int64_t HD = a.kv.head_dim, Q = a.n_heads_q * HD, KVD = a.kv.n_kv * HD;
  float *row = a.qkv + t * a.qkv_stride;
  for (int64_t i = threadIdx.x; i < Q; i += blockDim.x)
    if (a.bq) row[i] = __fadd_rn(row[i], a.bq[i]);
  for (int64_t i = threadIdx.x; i < KVD; i += blockDim.x) {
    if (a.bk) row[Q + i] = __fadd_rn(row[Q + i], a.bk[i]);
    if (a.bv) row[Q + KVD + i] = __fadd_rn(row[Q + KVD + i], a.bv[i]);
  }
  __syncthreads();
  if (!a.skip_rope && pos > 0) {
    const int64_t half = a.rotary_dim / 2, heads = a.n_heads_q + a.kv.n_kv;
    const float *ct = a.cos_tab + pos * half, *st = a.sin_tab + pos * half;
    for (int64_t i = threadIdx.x; i < heads * half; i += blockDim.x) {
      int64_t hh = i / half, j = i % half;
      float *hr = row + hh * HD;  // q heads then k heads are contiguous
      int64_t i0 = a.neox ? j : 2 * j, i1 = a.neox ? j + half : 2 * j + 1;
      float x0 = hr[i0], x1 = hr[i1];
      rot(x0, x1, ct[j], st[j]);
      hr[i0] = x0;
      hr[i1] = x1;
    }
    __syncthreads();
  }
  for (int64_t i = threadIdx.x; i < KVD; i += blockDim.x) {
    int64_t hh = i / HD, d = i % HD;
    int64_t e = kv_elem(a.kv, a.layer, hh, pos) + d;
    store_kv(a.kv.k, a.kv.f16, e, row[Q + i]);
    store_kv(a.kv.v, a.kv.f16, e, row[Q + KVD + i]);
  }
}

// ---- prefill: causal flash attention (f32) --------------------------------
// CTA = (query head, 32-query tile), 128 threads.  Thread (qi = tid/4, sub =
// tid%4) scores keys sub, sub+4, ... of each 64-key tile and owns output
// dims sub, sub+4, ... of its query.
constexpr int kPQ = 32, kPK = 64;

template <int HD, bool F16>
__global__ void __launch_bounds__(128) k_attn_prefill(const AttnPrefillArgs a) {
  extern __shared__ float sm[];
  float *q_s = sm;                          // [kPQ][HD]
  float *k_s = q_s + kPQ * HD;              // [kPK][HD + 1]
  float *v_s = k_s + kPK * (HD + 1);        // [kPK][HD]
  float *p_s = v_s + kPK * HD;              // [kPQ][kPK]
  const int hq = blockIdx.x, tid = threadIdx.x, qi = tid / 4, sub = tid % 4;
  const int64_t G = a.n_heads_q / a.kv.n_kv, hkv = hq / G;
  const int64_t q0 = (int64_t)blockIdx.y * kPQ;
  const int64_t nq = a.m - q0 < kPQ ? a.m - q0 : kPQ;
  for (int i = tid; i < kPQ * HD; i += 128) {
    int r = i / HD, d = i % HD;
    q_s[i] = r < nq ? a.qkv[(q0 + r) * a.qkv_stride + (int64_t)hq * HD + d] : 0.0f;
  }
  const int64_t my_pos = a.start_pos + q0 + qi;  // absolute position of this query
  const bool valid_q = qi < nq;
  const int64_t last_pos = a.start_pos + q0 + nq - 1;
  const int64_t first_pos = a.start_pos + q0;
  int64_t kbeg = 0;
  if (a.window > 0 && first_pos + 1 > a.window) kbeg = first_pos + 1 - a.window;
  kbeg = kbeg / kPK * kPK;
  float m_run = -INFINITY, l_run = 0.0f;
  constexpr int DPT = HD / 4;
  float o[DPT];
#pragma unroll
  for (int j = 0; j < DPT; j++) o[j] = 0.0f;
  for (int64_t k0 = kbeg; k0 <= last_pos; k0 += kPK) {
    __syncthreads();
    for (int i = tid; i < kPK * HD; i += 128) {
      int r = i / HD, d = i % HD;
      int64_t s = k0 + r;
      float kv = 0.0f, vv = 0.0f;
      if (s <= last_pos) {
        int64_t e = kv_elem(a.kv, a.layer, hkv, s) + d;
        if (F16) { kv = __half2float(((const __half *)a.kv.k)[e]); vv = __half2float(((const __half *)a.kv.v)[e]); }
        else { kv = ((const float *)a.kv.k)[e]; vv = ((const float *)a.kv.v)[e]; }
      }
      k_s[r * (HD + 1) + d] = kv;
      v_s[r * HD + d] = vv;
    }
    __syncthreads();
    float sc[kPK / 4];
    float cmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPK / 4; j++) {
      int kr = sub + 4 * j;
      int64_t s = k0 + kr;
      bool ok = valid_q && s <= my_pos && (a.window <= 0 || s + a.window > my_pos);
      float dot = 0.0f;
      if (ok) {
#pragma unroll 8
        for (int d = 0; d < HD; d++) dot = fmaf(q_s[qi * HD + d], k_s[kr * (HD + 1) + d], dot);
        dot = __fmul_rn(dot, a.scale);
      }
      sc[j] = ok ? dot : -INFINITY;
      cmax = fmaxf(cmax, sc[j]);
    }
    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
    cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
    float mn = fmaxf(m_run, cmax);
    float al = (m_run == -INFINITY) ? 0.0f : expf(m_run - mn);
    float psum = 0.0f;
#pragma unroll
    for (int j = 0; j < kPK / 4; j++) {
      float p = sc[j] == -INFINITY ? 0.0f : expf(sc[j] - mn);
      p_s[qi * kPK + sub + 4 * j] = p;
      psum += p;
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    m_run = mn;
    l_run = l_run * al + psum;
#pragma unroll
    for (int j = 0; j < DPT; j++) o[j] *= al;
    __syncwarp();
    for (int kr = 0; kr < kPK; kr++) {
      float p = p_s[qi * kPK + kr];
      if (p == 0.0f) continue;
#pragma unroll
      for (int j = 0; j < DPT; j++) o[j] = fmaf(p, v_s[kr * HD + sub + 4 * j], o[j]);
    }
  }
  if (valid_q) {
    float inv = l_run > 0.0f ? __fdiv_rn(1.0f, l_run) : 0.0f;
    float *out = a.out + (q0 + qi) * (a.n_heads_q * HD) + (int64_t)hq * HD;
#pragma unroll
    for (int j = 0; j < DPT; j++) out[sub + 4 * j] = o[j] * inv;
  }
}

}  // namespace

void launch_attn_decode(const AttnDecodeArgs &a, cudaStream_t s) {
  const bool f16 = a.kv.f16;
  if (a.kv.head_dim == 128) {
    if (f16) launch_decode_t<128, true>(a, s);
    else launch_decode_t<128, false>(a, s);
  } else {
    if (f16) launch_decode_t<64, true>(a, s);
    else launch_decode_t<64, false>(a, s);
  }
}

int attn_decode_cluster_size(int head_dim, int f16, int want) {
  for (int cs = want; cs >= 1; cs /= 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs);
    cfg.blockDim = dim3(kAttnThreads);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const void *kern = head_dim == 128 ? (f16 ? (const void *)k_attn_decode<128, true> : (const void *)k_attn_decode<128, false>)
                                       : (f16 ? (const void *)k_attn_decode<64, true> : (const void *)k_attn_decode<64, false>);
    if (cs > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) return cs;
    cudaGetLastError();
  }
  return 1;
}

void launch_rope_append(const RopeAppendArgs &a, cudaStream_t s) {
  if (!a.m) return;
  k_rope_append<<<(unsigned)a.m, 256, 0, s>>>(a);
}

void launch_attn_prefill(const AttnPrefillArgs &a, cudaStream_t s) {
  if (!a.m) return;
  dim3 grid((unsigned)a.n_heads_q, (unsigned)((a.m + kPQ - 1) / kPQ));
  auto go = [&](auto kern, int hd) {
    size_t smem = (size_t)(kPQ * hd + kPK * (hd + 1) + kPK * hd + kPQ * kPK) * sizeof(float);
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 128, smem, s>>>(a);
  };
  if (a.kv.head_dim == 128) {
    if (a.kv.f16) go(k_attn_prefill<128, true>, 128);
    else go(k_attn_prefill<128, false>, 128);
  } else {
    if (a.kv.f16) go(k_attn_prefill<64, true>, 64);
    else go(k_attn_prefill<64, false>, 64);
  }
}

}  // namespace jal
