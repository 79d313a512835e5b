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

#include "attn_dev.cuh"
#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

using namespace adev;

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kMaxClusterCtas = 16;  // CTAs per KV head (one cluster)
constexpr int kErrAttnWait = 2;            // bit set in the context error word

// Decode attention for one token.  Grid: n_kv clusters of cs CTAs; CTA rank r
// of cluster h handles positions [s0, s1) of KV head h, split evenly.
//
// Before griddepcontrol.wait (the cache rows below the current position were
// written by earlier launches) one thread starts bulk copies of the CTA's
// K/V rows into a ring of kStages shared-memory tiles.  After the wait the
// CTA builds q (bias, RoPE) for the head group and the new k/v; the CTA
// holding the current position appends it to the cache and patches its tile.
// Each warp scores its share of a tile (a group of LG lanes per position, q
// held in registers), keeps its own online softmax (max, denominator, P.V
// accumulator with lanes over dims), and the warps are merged at the end.
// Cluster partials are merged through distributed shared memory and every
// rank finalises and quantizes (QuantizedActQ8) a share of the 32-blocks.
template <int HD, bool F16, int GP>
__global__ void __launch_bounds__(kAttnThreads, 2) k_attn_decode(const AttnDecodeArgs a) {
  namespace cg = cooperative_groups;
  using Gm = AttnGeom<HD, F16, kAttnWarps>;
  constexpr int TP = Gm::TP, LG = Gm::LG, PPS = Gm::PPS, DPL = Gm::DPL, TPW = Gm::TPW, VD = Gm::VD;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) char ring[];  // kStages x kStageBytes, reused for the warp merge
  __shared__ __align__(8) uint64_t bars[kStages];
  __shared__ __align__(16) float q_s[GP][HD];
  __shared__ __align__(16) float kn_s[HD], vn_s[HD];
  __shared__ float cs_s[2][HD / 2];  // RoPE cos / sin of this position
  __shared__ __align__(16) float p_w[kAttnWarps][TPW * GP];
  __shared__ __align__(16) float acc_s[GP][HD];  // this CTA's partial (unnormalised)
  __shared__ float ml_s[2][GP];                  // its max / denominator per head
  __shared__ float wgt_s[kMaxClusterCtas][GP];
  __shared__ float lsum_s[kMaxClusterCtas][GP];
  __shared__ float den_s[GP];
  __shared__ float wm_s[kAttnWarps][GP];         // warp merge weights
  const int cs = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
  const int h = blockIdx.x / cs, tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int G = (int)(a.n_heads_q / a.kv.n_kv);
  const int64_t Q = a.n_heads_q * HD, KVD = a.kv.n_kv * HD;

  // Slice of this CTA.  d_pos was written before the previous kernel started.
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t span = seq - lo, per = (span + cs - 1) / cs;
  const int64_t s0 = lo + rank * per;
  const int64_t s1 = s0 + per < seq ? s0 + per : seq;
  const int64_t len = s1 > s0 ? s1 - s0 : 0;
  const int nt = (int)((len + TP - 1) / TP);
  if (tid == 0) {
    for (int s = 0; s < kStages; s++) mbar_init(&bars[s], 1);
    fence_barrier_init();
    fence_proxy_async();
    for (int k = 0; k < nt && k < kStages; k++) {
      const int64_t t0 = s0 + (int64_t)k * TP;
      const int n = (int)(s1 - t0 < TP ? s1 - t0 : TP);
      issue_tile<HD, F16>(a.kv, a.layer, ring + k * kStageBytes, &bars[k], t0, n, h);
    }
  }
  // RoPE rows of this position (static tables) are staged before the wait.
  const bool rope = !a.skip_rope && pos > 0;
  const int half = (int)(a.rotary_dim / 2);
  if (rope) {
    const bool use_long = a.long_threshold >= 0 && seq > a.long_threshold;
    const float *ct = (use_long ? a.cos_tab_long : a.cos_tab) + pos * half;
    const float *st = (use_long ? a.sin_tab_long : a.sin_tab) + pos * half;
    for (int j = tid; j < half; j += kAttnThreads) {
      cs_s[0][j] = ct[j];
      cs_s[1][j] = st[j];
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();

  // q / new k (+ bias, RoPE) and new v (+ bias) in one pass: each thread
  // produces one element, reading its rotation partner directly
  // (recipe.rs:2750-2767 for the rotation).  The stored (possibly
  // f16-rounded) new k/v are what every later step reads, so this step uses
  // the same values; the CTA holding the current position appends them.
  const bool own_pos = pos >= s0 && pos < s1;
  const int64_t app = own_pos ? kv_elem(a.kv, a.layer, h, pos) : 0;
  for (int i = tid; i < (GP + 2) * HD; i += kAttnThreads) {
    const int g = i / HD, d = i % HD;  // g < GP: q head, GP: k, GP + 1: v
    if (g < GP && g >= G) { q_s[g][d] = 0.0f; continue; }
    const int64_t off = g < GP ? (int64_t)(h * G + g) * HD : (g == GP ? Q : Q + KVD) + (int64_t)h * HD;
    const float *bias = g < GP ? a.bq : (g == GP ? a.bk : a.bv);
    auto ld = [&](int dd) {
      const float x = a.qkv[off + dd];
      return bias ? __fadd_rn(x, bias[(g < GP ? (int64_t)(h * G + g) * HD : (int64_t)h * HD) + dd]) : x;
    };
    float o = ld(d);
    if (rope && g <= GP && d < 2 * half) {
      const bool first = a.neox ? d < half : (d & 1) == 0;
      const int j = a.neox ? (first ? d : d - half) : d / 2;
      const int partner = a.neox ? (first ? d + half : d - half) : (d ^ 1);
      const float other = ld(partner);
      const float c = cs_s[0][j], sn = cs_s[1][j];
      const float x0 = first ? o : other, x1 = first ? other : o;
      o = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (g < GP) {
      q_s[g][d] = o;
    } else {
      if (F16) o = __half2float(__float2half_rn(o));
      if (g == GP) kn_s[d] = o;
      else vn_s[d] = o;
      if (own_pos) store_kv(g == GP ? a.kv.k : a.kv.v, a.kv.f16, app + d, o);  // append (recipe.rs:2319-2326)
    }
  }
  __syncthreads();

  // q slice of this lane for scoring: dims c*DPL .. c*DPL + DPL - 1.
  const int c = lane % LG, grp = lane / LG;
  float qr[GP][DPL];
#pragma unroll
  for (int g = 0; g < GP; g++)
#pragma unroll
    for (int k = 0; k < DPL; k++) qr[g][k] = q_s[g][c * DPL + k];

  float m_run[GP], acc[GP][VD];
  float l_lane = 0.0f;  // denominator of head lane % GP
#pragma unroll
  for (int g = 0; g < GP; g++) {
    m_run[g] = -INFINITY;
#pragma unroll
    for (int j = 0; j < VD; j++) acc[g][j] = 0.0f;
  }
  bool ok = true;
  float *pw = p_w[warp];

  for (int k = 0; k < nt; k++) {
    const int st = k % kStages;
    if (!mbar_wait_bounded(&bars[st], (uint32_t)((k / kStages) & 1))) ok = false;
    const int64_t t0 = s0 + (int64_t)k * TP;
    const int n = (int)(s1 - t0 < TP ? s1 - t0 : TP);
    char *Ks = ring + st * kStageBytes;
    char *Vs = Ks + TP * Gm::ROW;
    if (own_pos && pos >= t0 && pos < t0 + n) {
      const int j = (int)(pos - t0);
      for (int d = tid; d < HD; d += kAttnThreads) {
        if (F16) {
          ((__half *)(Ks + j * Gm::ROW))[d] = __float2half_rn(kn_s[d]);
          ((__half *)(Vs + j * Gm::ROW))[d] = __float2half_rn(vn_s[d]);
        } else {
          ((float *)(Ks + j * Gm::ROW))[d] = kn_s[d];
          ((float *)(Vs + j * Gm::ROW))[d] = vn_s[d];
        }
      }
      __syncthreads();
    }
    // Scores of this warp's TPW positions.
    float mt[GP];
#pragma unroll
    for (int g = 0; g < GP; g++) mt[g] = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < TPW / PPS; sp++) {
      const int jl = sp * PPS + grp;  // position within the warp's share
      const int j = warp * TPW + jl;  // position within the tile
      float d[GP];
#pragma unroll
      for (int g = 0; g < GP; g++) d[g] = 0.0f;
      if (j < n) {
        float kv[DPL];
        load_vals<F16, DPL>(Ks + j * Gm::ROW + c * 16, kv);
#pragma unroll
        for (int g = 0; g < GP; g++)
#pragma unroll
          for (int e = 0; e < DPL; e++) d[g] = fmaf(qr[g][e], kv[e], d[g]);
      }
#pragma unroll
      for (int o = 1; o < LG; o <<= 1)
#pragma unroll
        for (int g = 0; g < GP; g++) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
      float mine = -INFINITY;
#pragma unroll
      for (int g = 0; g < GP; g++) {
        const float sc = j < n ? __fmul_rn(d[g], a.scale) : -INFINITY;
        mt[g] = fmaxf(mt[g], sc);
        if (g == c) mine = sc;
      }
      if (c < GP) pw[jl * GP + c] = mine;
    }
#pragma unroll
    for (int o = LG; o < 32; o <<= 1)
#pragma unroll
      for (int g = 0; g < GP; g++) mt[g] = fmaxf(mt[g], __shfl_xor_sync(0xffffffffu, mt[g], o));
    float alpha[GP], mg = -INFINITY, ag = 0.0f;
#pragma unroll
    for (int g = 0; g < GP; g++) {
      const float mn = fmaxf(m_run[g], mt[g]);
      alpha[g] = m_run[g] == -INFINITY ? 0.0f : expf(m_run[g] - mn);
      m_run[g] = mn;
      if (g == lane % GP) { mg = mn; ag = alpha[g]; }
    }
    __syncwarp();
    // Probabilities (entry e = position * GP + head; head = lane % GP).
    float ls = 0.0f;
#pragma unroll
    for (int e = lane; e < TPW * GP; e += 32) {
      const float sv = pw[e];
      const float p = sv == -INFINITY ? 0.0f : expf(sv - mg);
      pw[e] = p;
      ls += p;
    }
#pragma unroll
    for (int o = GP; o < 32; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    l_lane = l_lane * ag + ls;
#pragma unroll
    for (int g = 0; g < GP; g++)
#pragma unroll
      for (int j = 0; j < VD; j++) acc[g][j] *= alpha[g];
    __syncwarp();
    // P.V over this warp's positions; lane owns dims lane*VD ...
#pragma unroll 4
    for (int jl = 0; jl < TPW; jl++) {
      const int j = warp * TPW + jl;
      if (j >= n) break;
      float v[VD];
      load_vals<F16, VD>(Vs + j * Gm::ROW + lane * VD * Gm::ES, v);
      float p[GP];
#pragma unroll
      for (int g = 0; g < GP; g++) p[g] = pw[jl * GP + g];
#pragma unroll
      for (int g = 0; g < GP; g++)
#pragma unroll
        for (int e = 0; e < VD; e++) acc[g][e] = fmaf(p[g], v[e], acc[g][e]);
    }
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && k + kStages < nt) {
      fence_proxy_async();
      const int64_t t1 = s0 + (int64_t)(k + kStages) * TP;
      const int n1 = (int)(s1 - t1 < TP ? s1 - t1 : TP);
      issue_tile<HD, F16>(a.kv, a.layer, Ks, &bars[st], t1, n1, h);
    }
  }
  if (!ok) {
    if (a.err) atomicOr(a.err, kErrAttnWait);
    // Give copies that may still be in flight a bounded chance to land
    // before the ring is reused.
    for (int k = nt > kStages ? nt - kStages : 0; k < nt; k++)
      mbar_wait_bounded(&bars[k % kStages], (uint32_t)((k / kStages) & 1));
  }

  // Merge the warps: partials in the (now idle) ring.
  float *acc_w = (float *)ring;               // [W][GP][HD]
  float *m_w = acc_w + kAttnWarps * GP * HD;  // [W][GP]
  float *l_w = m_w + kAttnWarps * GP;         // [W][GP]
#pragma unroll
  for (int g = 0; g < GP; g++)
#pragma unroll
    for (int j = 0; j < VD; j++) acc_w[(warp * GP + g) * HD + lane * VD + j] = acc[g][j];
  if (lane < GP) {
    float mm = -INFINITY;
#pragma unroll
    for (int g = 0; g < GP; g++)
      if (g == lane) mm = m_run[g];
    m_w[warp * GP + lane] = mm;
    l_w[warp * GP + lane] = l_lane;
  }
  __syncthreads();
  if (tid < GP) {
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, m_w[w * GP + tid]);
    float l = 0.0f;
    for (int w = 0; w < kAttnWarps; w++) {
      const float mw = m_w[w * GP + tid];
      const float wt = mw == -INFINITY ? 0.0f : expf(mw - M);
      wm_s[w][tid] = wt;
      l = fmaf(wt, l_w[w * GP + tid], l);
    }
    ml_s[0][tid] = M;
    ml_s[1][tid] = l;
  }
  __syncthreads();
  for (int i = tid; i < GP * HD; i += kAttnThreads) {
    const int g = i / HD;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) s = fmaf(wm_s[w][g], acc_w[(w * GP) * HD + i], s);
    acc_s[g][i % HD] = s;
  }
  cluster.sync();
  // Merge the cluster's partials through distributed shared memory:
  // out = sum_r e^(m_r - M) acc_r / sum_r e^(m_r - M) l_r.
  if (tid < cs * GP) {
    const int r = tid / GP, g = tid % GP;
    wgt_s[r][g] = cluster.map_shared_rank(&ml_s[0][0], r)[g];
    lsum_s[r][g] = cluster.map_shared_rank(&ml_s[1][0], r)[g];
  }
  __syncthreads();
  if (tid < GP) {
    float M = -INFINITY;
    for (int r = 0; r < cs; r++) M = fmaxf(M, wgt_s[r][tid]);
    float den = 0.0f;
    for (int r = 0; r < cs; r++) {
      const float mr = wgt_s[r][tid];
      const float w = mr == -INFINITY ? 0.0f : expf(mr - M);
      wgt_s[r][tid] = w;
      den = fmaf(w, lsum_s[r][tid], den);
    }
    den_s[tid] = den;
  }
  __syncthreads();
  // Rank r finalises 32-blocks r, r + cs, ... of this head group and
  // quantizes them (QuantizedActQ8; head boundaries are 32-aligned).
  for (int bi = rank + warp * cs; bi < G * HD / 32; bi += kAttnWarps * cs) {
    const int e = bi * 32 + lane, g = e / HD, d = e % HD;
    float part[kMaxClusterCtas];
#pragma unroll
    for (int r = 0; r < kMaxClusterCtas; r++)
      part[r] = r < cs ? cluster.map_shared_rank(&acc_s[0][0], r)[g * HD + d] : 0.0f;
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
}

template <int HD, bool F16, int GP>
const void *decode_fn() {
  return (const void *)k_attn_decode<HD, F16, GP>;
}

const void *pick_decode(int hd, int f16, int G) {
  const int gp = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
#define JAL_PICK(HDV, F, GPV) \
  if (hd == HDV && (f16 != 0) == F && gp == GPV) return decode_fn<HDV, F, GPV>();
  JAL_PICK(128, true, 1) JAL_PICK(128, true, 2) JAL_PICK(128, true, 4) JAL_PICK(128, true, 8)
  JAL_PICK(128, false, 1) JAL_PICK(128, false, 2) JAL_PICK(128, false, 4) JAL_PICK(128, false, 8)
  JAL_PICK(64, true, 1) JAL_PICK(64, true, 2) JAL_PICK(64, true, 4) JAL_PICK(64, true, 8)
  JAL_PICK(64, false, 1) JAL_PICK(64, false, 2) JAL_PICK(64, false, 4) JAL_PICK(64, false, 8)
#undef JAL_PICK
  return nullptr;
}

constexpr size_t kDecodeSmem = (size_t)kStages * kStageBytes;

void prepare_decode_fn(const void *fn, int cs) {
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmem);
  cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (cs > 8) cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
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

// ---- prefill: causal flash attention on the tensor cores (f16 KV) --------
// CTA = (query head, 64-query tile), 4 warps of 16 queries.  Per 64-key tile
// K (row-major) and V (transposed) are staged in shared memory as f16; S =
// Q K^T and O += P V run as mma.sync m16n8k16 f16 x f16 -> f32, with Q and
// P rounded to f16 (K and V already are, in an f16 cache) and the online
// softmax, scale and masks in f32.  Fragments (g = lane / 4, q = lane % 4):
// A regs (row g, k 2q..2q+1), (g + 8, 2q..), (g, 2q + 8..), (g + 8, 2q + 8..);
// B regs (k 2q..2q+1, col g), (2q + 8.., g); C (row g, cols 2q, 2q + 1),
// (g + 8, ...).  The S accumulator of key tiles 2t, 2t + 1 is the P operand
// of k-step t as it lies in registers.
constexpr int kFQ = 64, kFK = 64;

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int HD>
__global__ void __launch_bounds__(128) k_attn_prefill_mma(const AttnPrefillArgs a) {
  constexpr int KS = HD / 16, NO = HD / 8, NK = kFK / 8;
  constexpr int KSTR = HD + 8, VSTR = kFK + 8;  // padded rows (halves): conflict-free fragment loads
  __shared__ __align__(16) __half k_s[kFK * KSTR];
  __shared__ __align__(16) __half vt_s[HD * VSTR];
  const int hq = blockIdx.x, tid = threadIdx.x, warp = tid / 32, lane = tid % 32, g = lane / 4, q = lane % 4;
  const int64_t G = a.n_heads_q / a.kv.n_kv, hkv = hq / G;
  const int64_t q0 = (int64_t)blockIdx.y * kFQ;
  const int64_t nq = a.m - q0 < kFQ ? a.m - q0 : kFQ;
  const int r0 = warp * 16 + g, r1 = r0 + 8;  // this lane's two query rows in the tile
  const bool v0 = r0 < nq, v1 = r1 < nq;
  const int64_t p0 = a.start_pos + q0 + r0, p1 = p0 + 8;
  uint32_t qf[KS][4];
  {
    const float *q0p = a.qkv + (q0 + (v0 ? r0 : 0)) * a.qkv_stride + (int64_t)hq * HD;
    const float *q1p = a.qkv + (q0 + (v1 ? r1 : 0)) * a.qkv_stride + (int64_t)hq * HD;
#pragma unroll
    for (int s = 0; s < KS; s++) {
      const int d = 16 * s + 2 * q;
      qf[s][0] = v0 ? pack_h2(q0p[d], q0p[d + 1]) : 0u;
      qf[s][1] = v1 ? pack_h2(q1p[d], q1p[d + 1]) : 0u;
      qf[s][2] = v0 ? pack_h2(q0p[d + 8], q0p[d + 9]) : 0u;
      qf[s][3] = v1 ? pack_h2(q1p[d + 8], q1p[d + 9]) : 0u;
    }
  }
  const int64_t last_pos = a.start_pos + q0 + nq - 1, first_pos = a.start_pos + q0;
  int64_t kbeg = 0;
  if (a.window > 0 && first_pos + 1 > a.window) kbeg = first_pos + 1 - a.window;
  kbeg = kbeg / kFK * kFK;
  float o[NO][4];
#pragma unroll
  for (int n = 0; n < NO; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  for (int64_t k0 = kbeg; k0 <= last_pos; k0 += kFK) {
    __syncthreads();
    for (int i = tid; i < kFK * HD / 8; i += 128) {
      const int r = i / (HD / 8), c8 = i % (HD / 8);
      const int64_t pos = k0 + r;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (pos <= last_pos) {
        const int64_t e = kv_elem(a.kv, a.layer, hkv, pos) + c8 * 8;
        kv = *(const uint4 *)((const __half *)a.kv.k + e);
        vv = *(const uint4 *)((const __half *)a.kv.v + e);
      }
      *(uint4 *)&k_s[r * KSTR + c8 * 8] = kv;
      const __half *vh = reinterpret_cast<const __half *>(&vv);
#pragma unroll
      for (int j = 0; j < 8; j++) vt_s[(c8 * 8 + j) * VSTR + r] = vh[j];
    }
    __syncthreads();
    // Skip the tile only when it is masked for every lane: mma.sync needs the
    // whole warp, so the decision must be warp-uniform.
    if (__all_sync(0xffffffffu, k0 > p1 || (!v0 && !v1))) continue;
    float sc[NK][4];
#pragma unroll
    for (int j = 0; j < NK; j++) {
      sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
      const __half *kr = k_s + (8 * j + g) * KSTR + 2 * q;
#pragma unroll
      for (int s = 0; s < KS; s++)
        mma_f16_16816(sc[j], qf[s], *(const uint32_t *)(kr + 16 * s), *(const uint32_t *)(kr + 16 * s + 8));
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < NK; j++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int64_t key = k0 + 8 * j + 2 * q + (i & 1);
        const int64_t qp = i < 2 ? p0 : p1;
        const bool ok = (i < 2 ? v0 : v1) && key <= qp && (a.window <= 0 || key + a.window > qp);
        const float v = ok ? __fmul_rn(sc[j][i], a.scale) : -INFINITY;
        sc[j][i] = v;
        if (i < 2) mx0 = fmaxf(mx0, v);
        else mx1 = fmaxf(mx1, v);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float al0 = m0 == -INFINITY ? 0.0f : expf(m0 - n0), al1 = m1 == -INFINITY ? 0.0f : expf(m1 - n1);
    m0 = n0;
    m1 = n1;
    float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
    for (int j = 0; j < NK; j++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float p = sc[j][i] == -INFINITY ? 0.0f : expf(sc[j][i] - (i < 2 ? n0 : n1));
        sc[j][i] = p;
        if (i < 2) ps0 += p;
        else ps1 += p;
      }
    l0 = l0 * al0 + ps0;  // this lane's keys; the quad is summed at the end
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int n = 0; n < NO; n++) {
      o[n][0] *= al0; o[n][1] *= al0;
      o[n][2] *= al1; o[n][3] *= al1;
    }
#pragma unroll
    for (int t = 0; t < kFK / 16; t++) {
      const uint32_t pa[4] = {pack_h2(sc[2 * t][0], sc[2 * t][1]), pack_h2(sc[2 * t][2], sc[2 * t][3]),
                              pack_h2(sc[2 * t + 1][0], sc[2 * t + 1][1]), pack_h2(sc[2 * t + 1][2], sc[2 * t + 1][3])};
#pragma unroll
      for (int n = 0; n < NO; n++) {
        const __half *vr = vt_s + (8 * n + g) * VSTR + 16 * t + 2 * q;
        mma_f16_16816(o[n], pa, *(const uint32_t *)vr, *(const uint32_t *)(vr + 8));
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = l0 > 0.0f ? __fdiv_rn(1.0f, l0) : 0.0f, i1 = l1 > 0.0f ? __fdiv_rn(1.0f, l1) : 0.0f;
  const int64_t ostride = a.n_heads_q * HD;
  float *out0 = a.out + (q0 + r0) * ostride + (int64_t)hq * HD + 2 * q;
  float *out1 = a.out + (q0 + r1) * ostride + (int64_t)hq * HD + 2 * q;
#pragma unroll
  for (int n = 0; n < NO; n++) {
    if (v0) { out0[8 * n] = o[n][0] * i0; out0[8 * n + 1] = o[n][1] * i0; }
    if (v1) { out1[8 * n] = o[n][2] * i1; out1[8 * n + 1] = o[n][3] * i1; }
  }
}

}  // namespace

void launch_attn_decode(const AttnDecodeArgs &a, cudaStream_t s) {
  const int G = (int)(a.n_heads_q / a.kv.n_kv);
  const void *fn = pick_decode((int)a.kv.head_dim, a.kv.f16, G);
  if (!fn) return;
  const int cs = a.n_splits;
  prepare_decode_fn(fn, cs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.kv.n_kv * cs));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = kDecodeSmem;
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
  void *args[] = {(void *)&a};
  cudaLaunchKernelExC(&cfg, fn, args);
}

int attn_decode_cluster_size(int head_dim, int f16, int G, int want) {
  const void *fn = pick_decode(head_dim, f16, G);
  if (!fn) return 0;
  for (int cs = want; cs >= 1; cs /= 2) {
    prepare_decode_fn(fn, cs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kDecodeSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess && n > 0) return cs;
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
  if (a.kv.f16 && (a.kv.head_dim == 128 || a.kv.head_dim == 64)) {  // tensor cores
    dim3 g2((unsigned)a.n_heads_q, (unsigned)((a.m + kFQ - 1) / kFQ));
    if (a.kv.head_dim == 128) k_attn_prefill_mma<128><<<g2, 128, 0, s>>>(a);
    else k_attn_prefill_mma<64><<<g2, 128, 0, s>>>(a);
    return;
  }
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
