// Decode attention in the reference's f32 order (gqa_attention_prefill_portable,
// recipe.rs:2949-3022, for one token over the paged KV cache).
//
// Per query head the reference computes, over the active positions t:
//   score_t = (sum_d q_d * k_td, left to right from -0.0) * scale
//   max over t; e_t = exp(score_t - max); den = sum_t e_t (from +0.0)
//   inv = den > 0 ? 1 / den : 0
//   out_d = sum_t (e_t * inv) * v_td, left to right over t from +0.0
// Every product and sum is one f32 rounding, no fused multiply-add.
//
// This kernel stops at the weights w_t = e_t * inv, which it writes per
// query head and position; xattn_v.cu runs the output chains.
//
// Grid: one thread-block cluster of CS CTAs per KV head (CS >= G, the query
// heads per KV head).  Every CTA builds q (bias, RoPE) for the G heads and
// the new k / v (the CTA holding the current position appends them; with an
// f16 cache the rounded values are what every step reads), then scores its
// contiguous share of the positions: a thread per position loads its K row
// (prefetched into L2 before griddepcontrol.wait) into registers, 256 bytes
// at a time as independent 16-byte loads, and runs the G score chains over
// the dims in order.  The cluster agrees on each head's max through
// distributed shared memory (all ranks' maxima read at once), and every CTA
// writes its e_t straight into the position-ordered array of the CTA that
// owns the head.  CTA g < G then forms head g's exact sequential denominator
// (exact::seq_sum_nonneg) and writes w_t.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "attn_dev.cuh"
#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "exact.cuh"
#include "jal.h"

namespace jal {

namespace {

constexpr int kXT = 384, kXW = kXT / 32;  // one thread per position: 8 x 384 positions in one round

template <int HD, bool F16>
struct XA {
  static constexpr int ES = F16 ? 2 : 4;
  static constexpr int ROW = HD * ES;
  static constexpr int NCH = ROW / 16;  // 16-byte chunks per row
  static constexpr int CH = 16 / ES;    // elements per chunk
  static constexpr int GRP = NCH < 16 ? NCH : 16;  // chunks loaded at once (256 bytes)
};

struct XAttnLayout {
  size_t sc, E, sum, total;
};

__host__ __device__ inline XAttnLayout xattn_layout(int per_cap, int n_ctx) {
  XAttnLayout L;
  size_t o = 0;
  L.sc = o; o += ((size_t)8 * per_cap * 4 + 15) / 16 * 16;
  L.E = o; o += ((size_t)n_ctx * 4 + 16 + 15) / 16 * 16;  // E[i] at lo % 4 + i
  L.sum = o; o += (sizeof(exact::SumSmem<kXT>) + 15) / 16 * 16;  // also E's read slack
  L.total = o;  // every piece starts 16-byte aligned (the sum's 16-byte entries)
  return L;
}

// Stage k of positions [A, B): [max(A, (A/R + k) R), min(B, (A/R + k + 1) R)).
struct StageRange {
  int64_t t0;
  int n;
};
__device__ __forceinline__ StageRange stage_of(int64_t A, int64_t B, int R, int k) {
  const int64_t base = (A / R + k) * R;
  const int64_t t0 = base > A ? base : A, t1 = base + R < B ? base + R : B;
  return {t0, (int)(t1 - t0)};
}
__device__ __forceinline__ int stage_count(int64_t A, int64_t B, int R) {
  return B > A ? (int)((B + R - 1) / R - A / R) : 0;
}

// Dims [c * CH, c * CH + CH) of a row chunk as floats.
template <bool F16, int CH>
__device__ __forceinline__ void chunk_vals(uint4 raw, float (&o)[CH]) {
  if (F16) {
    const __half2 *h = (const __half2 *)&raw;
#pragma unroll
    for (int k = 0; k < CH / 2; k++) {
      const float2 f = __half22float2(h[k]);
      o[2 * k] = f.x;
      o[2 * k + 1] = f.y;
    }
  } else {
    o[0] = __uint_as_float(raw.x);
    o[1] = __uint_as_float(raw.y);
    o[2] = __uint_as_float(raw.z);
    o[3] = __uint_as_float(raw.w);
  }
}

template <int HD, bool F16, int GP>
__global__ void __launch_bounds__(kXT, 1) k_xattn(const AttnDecodeArgs a, int per_cap, int n_ctx, int R) {
  const KernelTrace trace(a.trace);
  namespace cg = cooperative_groups;
  using A = XA<HD, F16>;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) char smem[];
  __shared__ __align__(16) float q_s[GP][HD];
  __shared__ __align__(16) float kn_s[HD];
  __shared__ float cs_s[2][HD / 2];
  __shared__ float mx_s[8], red_s[kXW][GP];
  __shared__ float gmax_s[8], xr_s[16][8];
  const XAttnLayout L = xattn_layout(per_cap, n_ctx);
  float *sc = (float *)(smem + L.sc);  // [8][per_cap]: scores

  const int cs = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
  const int h = blockIdx.x / cs, tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = (int)(a.n_heads_q / a.kv.n_kv);
  const int64_t Q = a.n_heads_q * HD, KVD = a.kv.n_kv * HD;
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t span = seq - lo, per = (span + cs - 1) / cs;
  const int64_t s0 = lo + rank * per, s1 = s0 + per < seq ? s0 + per : seq;
  const int len = s1 > s0 ? (int)(s1 - s0) : 0;
  float *E = (float *)(smem + L.E) + (lo & 3);  // E[i]: position lo + i
  const bool vsum = rank < G;

  // Rows below the current position were written by earlier launches (the
  // current row is taken from shared memory below): thread k looks up stage k
  // of this CTA's share (all lookups in parallel) and prefetches it to L2.
  {
    const int nks = stage_count(s0, s1, R);
    for (int k = tid; k < nks; k += kXT) {
      const StageRange st = stage_of(s0, s1, R, k);
      l2_prefetch_bulk((const char *)a.kv.k + adev::kv_elem(a.kv, a.layer, h, st.t0) * A::ES,
                       (uint64_t)st.n * A::ROW);
    }
  }
  const bool rope = !a.skip_rope && pos > 0;
  const int half = (int)(a.rotary_dim / 2);
  if (rope) {
    const bool use_long = a.long_threshold >= 0 && seq > a.long_threshold;
    const float *ct = (use_long ? a.cos_tab_long : a.cos_tab) + pos * half;
    const float *st = (use_long ? a.sin_tab_long : a.sin_tab) + pos * half;
    for (int j = tid; j < half; j += kXT) {
      cs_s[0][j] = ct[j];
      cs_s[1][j] = st[j];
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (tid == 0) trace.mark(0);  // the grid dependency resolved

  // q (G heads) and the new k / v: bias, then RoPE (recipe.rs:2490-2518,
  // 2717-2773); the appended row is the stored (f16-rounded) value.
  const bool own_pos = pos >= s0 && pos < s1;
  const int64_t app = own_pos ? adev::kv_elem(a.kv, a.layer, h, pos) : 0;
  for (int i = tid; i < (G + 2) * HD; i += kXT) {
    const int g = i / HD, d = i % HD;  // g < G: q head, G: k, G + 1: v
    const int64_t off = g < G ? (int64_t)(h * G + g) * HD : (g == G ? Q : Q + KVD) + (int64_t)h * HD;
    const float *bias = g < G ? a.bq : (g == G ? a.bk : a.bv);
    const int64_t boff = g < G ? (int64_t)(h * G + g) * HD : (int64_t)h * HD;
    auto ld = [&](int dd) {
      const float x = a.qkv[off + dd];
      return bias ? __fadd_rn(x, bias[boff + dd]) : x;
    };
    float o = ld(d);
    if (rope && g <= G && d < 2 * half) {
      const bool first = a.neox ? d < half : (d & 1) == 0;
      const int j = a.neox ? (first ? d : d - half) : d / 2;
      const int partner = a.neox ? (first ? d + half : d - half) : (d ^ 1);
      const float other = ld(partner), c = cs_s[0][j], sn = cs_s[1][j];
      const float x0 = first ? o : other, x1 = first ? other : o;
      o = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (g < G) {
      q_s[g][d] = o;
    } else {
      if (F16) o = __half2float(__float2half_rn(o));
      if (g == G) kn_s[d] = o;
      if (own_pos) adev::store_kv(g == G ? a.kv.k : a.kv.v, a.kv.f16, app + d, o);  // recipe.rs:2319-2326
    }
  }
  for (int i = tid; i < (GP - G) * HD; i += kXT) q_s[G + i / HD][i % HD] = 0.0f;
  __syncthreads();

  // Phase A: scores, one thread per position of this CTA's share.
  float lmax[GP];
#pragma unroll
  for (int g = 0; g < GP; g++) lmax[g] = -INFINITY;
  for (int j = tid; j < len; j += kXT) {
    const int64_t t = s0 + j;
    float d[GP];
#pragma unroll
    for (int g = 0; g < GP; g++) d[g] = -0.0f;
    if (t == pos) {  // the current row: from the values just built
      for (int e = 0; e < HD; e++)
#pragma unroll
        for (int g = 0; g < GP; g++) d[g] = __fadd_rn(d[g], __fmul_rn(q_s[g][e], kn_s[e]));
    } else {
      const uint4 *row = (const uint4 *)((const char *)a.kv.k + adev::kv_elem(a.kv, a.layer, h, t) * A::ES);
#pragma unroll
      for (int grp = 0; grp < A::NCH / A::GRP; grp++) {
        uint4 raw[A::GRP];
#pragma unroll
        for (int c = 0; c < A::GRP; c++) raw[c] = row[grp * A::GRP + c];
#pragma unroll
        for (int c = 0; c < A::GRP; c++) {
          float kv[A::CH];
          chunk_vals<F16, A::CH>(raw[c], kv);
          const int e0 = (grp * A::GRP + c) * A::CH;
#pragma unroll
          for (int e4 = 0; e4 < A::CH; e4 += 4) {
            float4 qv[GP];
#pragma unroll
            for (int g = 0; g < GP; g++) qv[g] = *(const float4 *)&q_s[g][e0 + e4];
#pragma unroll
            for (int g = 0; g < GP; g++) {
              d[g] = __fadd_rn(d[g], __fmul_rn(qv[g].x, kv[e4]));
              d[g] = __fadd_rn(d[g], __fmul_rn(qv[g].y, kv[e4 + 1]));
              d[g] = __fadd_rn(d[g], __fmul_rn(qv[g].z, kv[e4 + 2]));
              d[g] = __fadd_rn(d[g], __fmul_rn(qv[g].w, kv[e4 + 3]));
            }
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < GP; g++) {
      if (g < G) {
        const float sv = __fmul_rn(d[g], a.scale);
        sc[g * per_cap + j] = sv;
        if (sv > lmax[g]) lmax[g] = sv;
      }
    }
  }
  if (lane == 0) trace.mark(1);  // scores done (the latest warp of any CTA)
  // Per-head max of this CTA (order-independent; NaN never wins, as with
  // `if score > max_score`).
#pragma unroll
  for (int g = 0; g < GP; g++) {
    float m = warp_max(lmax[g]);
    if (lane == 0) red_s[warp][g] = m;
  }
  __syncthreads();
  if (tid < 8) {
    float m = -INFINITY;
    if (tid < GP)
      for (int w = 0; w < kXW; w++)
        if (red_s[w][tid] > m) m = red_s[w][tid];
    mx_s[tid] = m;
  }
  cluster.sync();
  if (tid == 0) trace.mark(2);  // maxima exchanged
  // Every rank's per-head maxima, read in parallel: thread r * G + g reads
  // rank r's head g.
  if (tid < cs * G) xr_s[tid / G][tid % G] = cluster.map_shared_rank(mx_s, tid / G)[tid % G];
  __syncthreads();
  if (tid < G) {
    float m = -INFINITY;
    for (int r = 0; r < cs; r++)
      if (xr_s[r][tid] > m) m = xr_s[r][tid];
    gmax_s[tid] = m;
  }
  __syncthreads();
  // e_t = exp(score - max) goes straight into E of the CTA that sums head g
  // (rank g), at the position's place.
  for (int g = 0; g < G; g++) {
    float *dst = cluster.map_shared_rank(E, g) + (s0 - lo);
    for (int j = tid; j < len; j += kXT) dst[j] = exact::exp_ref(__fsub_rn(sc[g * per_cap + j], gmax_s[g]));
  }
  cluster.sync();  // every e_t has landed; no remote access after this point
  if (tid == 0) trace.mark(3);  // exp terms in place
  if (!vsum) return;
  const int g = rank;
  const float den = exact::seq_sum_nonneg<kXT>(E, (int)span, 0.0f, *(exact::SumSmem<kXT> *)(smem + L.sum));
  if (tid == 0) trace.mark(4);  // denominator
  const float inv = den > 0.0f ? __fdiv_rn(1.0f, den) : 0.0f;
  float *wg = a.w_out + (int64_t)(h * G + g) * a.w_stride + lo;  // this head's weights, by position
  for (int64_t i = tid; i < span; i += kXT) wg[i] = __fmul_rn(E[i], inv);
}

template <int HD, bool F16>
const void *xattn_fn(int G) {
  if (G <= 1) return (const void *)k_xattn<HD, F16, 1>;
  if (G <= 2) return (const void *)k_xattn<HD, F16, 2>;
  if (G <= 4) return (const void *)k_xattn<HD, F16, 4>;
  return (const void *)k_xattn<HD, F16, 8>;
}

const void *pick_x(int hd, int f16, int G) {
  if (G > 8) return nullptr;
  if (hd == 128) return f16 ? xattn_fn<128, true>(G) : xattn_fn<128, false>(G);
  if (hd == 64) return f16 ? xattn_fn<64, true>(G) : xattn_fn<64, false>(G);
  return nullptr;
}

// Positions per K prefetch: the largest power of two <= 64 dividing the
// page size.
int stage_rows(int64_t page_size) {
  int R = 1;
  while (R * 2 <= 64 && page_size % (R * 2) == 0) R *= 2;
  return R;
}

constexpr size_t kSmemCap = 220 * 1024;

}  // namespace

int xattn_cluster_size(int head_dim, int f16, int G, int n_kv, int64_t n_ctx) {
  const void *fn = pick_x(head_dim, f16, G);
  if (!fn || G > 16) return 0;
  // The largest cluster (<= 16, >= G) for which every KV head's cluster is
  // resident at once: a second wave would double the kernel's latency.
  int best = 0;
  for (int cs = 16; cs >= G && cs >= 1; cs /= 2) {
    const int per_cap = (int)((n_ctx + cs - 1) / cs);
    const size_t smem = xattn_layout(per_cap, (int)n_ctx).total;
    if (smem + 8 * 1024 > kSmemCap) continue;  // + static shared memory
    {  // only ever raise the limit: contexts created earlier may launch larger shares
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess || (size_t)fa.maxDynamicSharedSizeBytes < smem)
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    if (cs > 8) cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cs);
    cfg.blockDim = dim3(kXT);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (n >= n_kv) return cs;
    if (n > 0 && !best) best = cs;
  }
  return best;
}

int xattn_batch_cluster_size(int head_dim, int f16, int G, int64_t n_ctx) {
  const void *fn = pick_x(head_dim, f16, G);
  if (!fn || G > 16) return 0;
  // The smallest cluster (>= G) whose shares fit: several sequences' score
  // kernels then run side by side.
  for (int cs = 1; cs <= 16; cs *= 2) {
    if (cs < G) continue;
    const int per_cap = (int)((n_ctx + cs - 1) / cs);
    const size_t smem = xattn_layout(per_cap, (int)n_ctx).total;
    if (smem + 8 * 1024 > kSmemCap) continue;
    if (cs > 8) cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return cs;
  }
  return 0;
}

void launch_xattn_decode(const AttnDecodeArgs &a, int64_t n_ctx, cudaStream_t s) {
  const int G = (int)(a.n_heads_q / a.kv.n_kv);
  const void *fn = pick_x((int)a.kv.head_dim, a.kv.f16, G);
  const int cs = a.n_splits;
  if (!fn || cs < G) fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention: unsupported shape");
  int per_cap = (int)((n_ctx + cs - 1) / cs), nc = (int)n_ctx, R = stage_rows(a.kv.page_size);
  const size_t smem = xattn_layout(per_cap, nc).total;
  if (smem + 8 * 1024 > kSmemCap)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention: n_ctx %lld does not fit", (long long)n_ctx);
  if (R < 8) fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention: page size %lld not a multiple of 8",
                  (long long)a.kv.page_size);
  {  // raise the kernel's shared-memory limit when this share needs more
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, fn) == cudaSuccess && (size_t)fa.maxDynamicSharedSizeBytes < smem)
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.kv.n_kv * cs));
  cfg.blockDim = dim3(kXT);
  cfg.dynamicSmemBytes = smem;
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
  void *args[] = {(void *)&a, (void *)&per_cap, (void *)&nc, (void *)&R};
  cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace jal
