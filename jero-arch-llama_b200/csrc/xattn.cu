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
// Grid: one thread-block cluster of CS CTAs per KV head (CS >= G, the query
// heads per KV head).  Phase A: every CTA builds q (bias, RoPE) for the G
// heads and the new k / v (the CTA holding the current position appends
// them; with an f16 cache the rounded values are what every step reads), then
// scores its contiguous share of the positions from K rows that arrive by
// bulk copies into a pitched shared-memory ring (one copy per position row,
// pitch row + 16 bytes so a warp reading 32 rows at one offset stays
// conflict-free), one sequential chain per (head, position).  The cluster
// agrees on each head's max through distributed shared memory and every CTA
// turns its scores into e_t.  Phase B: CTA g < G gathers head g's e_t in
// position order, forms the exact sequential denominator
// (exact::seq_sum_nonneg), and runs the HD output chains (thread d) over all
// positions in order with V rows streamed through a second bulk-copy ring;
// a producer warp refills a ring slot once every chain has passed it.  The
// output row and its QuantizedActQ8 blocks (the O projection's input) are
// written by that CTA.  Waits on copies are bounded: a wait that gives up
// sets bit 2 of the context's error word and the kernel runs to its end.
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

constexpr int kXT = 256, kXW = kXT / 32;
constexpr int kTK = 32, kNSK = 4;  // K ring: positions per stage, stages
constexpr int kTV = 32;            // V ring: positions per stage
constexpr int kErrCopyWait = 4;

template <int HD, bool F16>
struct XA {
  static constexpr int ES = F16 ? 2 : 4;
  static constexpr int ROW = HD * ES;
  static constexpr int KP = ROW + 16;
  static constexpr int CH = 16 / ES;  // elements per 16-byte chunk
  static constexpr int NSV = F16 ? 6 : 3;  // V ring stages
};

struct XAttnLayout {
  size_t kring, vring, sc, E, sum, total;
};

template <int HD, bool F16>
__host__ __device__ inline XAttnLayout xattn_layout(int per_cap, int n_ctx) {
  using A = XA<HD, F16>;
  XAttnLayout L;
  size_t o = 0;
  L.kring = o; o += (size_t)kNSK * kTK * A::KP;
  L.vring = o; o += (size_t)A::NSV * kTV * A::ROW;
  L.sc = o; o += ((size_t)8 * per_cap * 4 + 15) / 16 * 16;
  L.E = o; o += ((size_t)n_ctx * 4 + 15) / 16 * 16;
  L.sum = o; o += (sizeof(exact::SumSmem<kXT>) + 15) / 16 * 16;
  L.total = o;
  return L;
}

// Bulk copies of K (pitched) or V (dense) rows [t0, t0 + n) of KV head h.
template <int HD, bool F16, bool PITCHED>
__device__ void issue_rows(const KvView &kv, int64_t layer, int h, const void *base, char *dst, uint64_t *bar,
                           int64_t t0, int n) {
  using A = XA<HD, F16>;
  mbar_expect_tx(bar, (uint32_t)(n * A::ROW));
  if (PITCHED) {
    for (int j = 0; j < n; j++) {
      const int64_t e = adev::kv_elem(kv, layer, h, t0 + j);
      bulk_g2s(dst + j * A::KP, (const char *)base + e * A::ES, (uint32_t)A::ROW, bar);
    }
  } else {
    int done = 0;
    while (done < n) {  // one copy per page run
      const int64_t p = t0 + done, slot = p % kv.page_size;
      const int run = (int)(kv.page_size - slot < n - done ? kv.page_size - slot : n - done);
      const int64_t e = adev::kv_elem(kv, layer, h, p);
      bulk_g2s(dst + done * A::ROW, (const char *)base + e * A::ES, (uint32_t)(run * A::ROW), bar);
      done += run;
    }
  }
}

template <int HD, bool F16>
__global__ void __launch_bounds__(kXT, 1) k_xattn(const AttnDecodeArgs a, int per_cap, int n_ctx) {
  namespace cg = cooperative_groups;
  using A = XA<HD, F16>;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) char smem[];
  __shared__ __align__(8) uint64_t kbar[kNSK], vfull[A::NSV], vempty[A::NSV];
  __shared__ __align__(16) float q_s[8][HD];
  __shared__ __align__(16) float kn_s[HD], vn_s[HD];
  __shared__ float cs_s[2][HD / 2];
  __shared__ float mx_s[8], red_s[kXW][8];
  __shared__ float gmax_s[8];
  __shared__ int bad_s;
  const XAttnLayout L = xattn_layout<HD, F16>(per_cap, n_ctx);
  char *kring = smem + L.kring, *vring = smem + L.vring;
  float *sc = (float *)(smem + L.sc);  // [8][per_cap]: scores, then e_t
  float *E = (float *)(smem + L.E);

  const int cs = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
  const int h = blockIdx.x / cs, tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = (int)(a.n_heads_q / a.kv.n_kv);
  const int64_t Q = a.n_heads_q * HD, KVD = a.kv.n_kv * HD;
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t span = seq - lo, per = (span + cs - 1) / cs;
  const int64_t s0 = lo + rank * per, s1 = s0 + per < seq ? s0 + per : seq;
  const int len = s1 > s0 ? (int)(s1 - s0) : 0;
  const int nk = (len + kTK - 1) / kTK;
  const bool vsum = rank < G;
  const int nv = vsum ? (int)((span + kTV - 1) / kTV) : 0;

  if (tid == 0) {
    for (int s = 0; s < kNSK; s++) mbar_init(&kbar[s], 1);
    for (int s = 0; s < A::NSV; s++) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], HD);
    }
    bad_s = 0;
    fence_barrier_init();
    fence_proxy_async();
    // Rows below the current position were written by earlier launches; the
    // current row is patched from registers / shared memory below.
    for (int k = 0; k < nk && k < kNSK; k++) {
      const int64_t t0 = s0 + (int64_t)k * kTK;
      issue_rows<HD, F16, true>(a.kv, a.layer, h, a.kv.k, kring + k * kTK * A::KP, &kbar[k], t0,
                                (int)(s1 - t0 < kTK ? s1 - t0 : kTK));
    }
    for (int k = 0; k < nv && k < A::NSV; k++) {
      const int64_t t0 = lo + (int64_t)k * kTV;
      issue_rows<HD, F16, false>(a.kv, a.layer, h, a.kv.v, vring + k * kTV * A::ROW, &vfull[k], t0,
                                 (int)(seq - t0 < kTV ? seq - t0 : kTV));
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
      else vn_s[d] = o;
      if (own_pos) adev::store_kv(g == G ? a.kv.k : a.kv.v, a.kv.f16, app + d, o);  // recipe.rs:2319-2326
    }
  }
  __syncthreads();

  // Phase A: scores.  Warp w takes head w % GP of stage (round * R + w / GP).
  const int GP = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
  const int R = kXW / GP < kNSK ? kXW / GP : kNSK;  // stages per round (each in its own ring slot)
  bool ok = true;
  float lmax = -INFINITY;  // this thread's head: warp % GP
  for (int k0 = 0; k0 < nk; k0 += R) {
    const int k = k0 + warp / GP, g = warp % GP;
    if (warp / GP < R && k < nk && g < G) {
      const int slot = k % kNSK;
      if (!mbar_wait_bounded(&kbar[slot], (uint32_t)((k / kNSK) & 1))) ok = false;
      const int64_t t0 = s0 + (int64_t)k * kTK;
      const int n = (int)(s1 - t0 < kTK ? s1 - t0 : kTK);
      if (lane < n) {
        const int64_t t = t0 + lane;
        const char *row = kring + slot * kTK * A::KP + lane * A::KP;
        const float *qg = q_s[g];
        float d = -0.0f;
        if (t == pos) {  // the current row: from the values just built
          for (int e = 0; e < HD; e++) d = __fadd_rn(d, __fmul_rn(qg[e], kn_s[e]));
        } else {
#pragma unroll 4
          for (int c = 0; c < HD / A::CH; c++) {
            float kv[A::CH];
            adev::load_vals<F16, A::CH>(row + c * 16, kv);
#pragma unroll
            for (int e = 0; e < A::CH; e++) d = __fadd_rn(d, __fmul_rn(qg[c * A::CH + e], kv[e]));
          }
        }
        const float s = __fmul_rn(d, a.scale);
        sc[g * per_cap + (int)(t - s0)] = s;
        if (s > lmax) lmax = s;
      }
    }
    __syncthreads();  // the round's stages are consumed
    if (tid == 0) {
      fence_proxy_async();
      for (int kk = k0; kk < k0 + R && kk < nk; kk++) {
        const int kn = kk + kNSK;
        if (kn < nk) {
          const int64_t t0 = s0 + (int64_t)kn * kTK;
          issue_rows<HD, F16, true>(a.kv, a.layer, h, a.kv.k, kring + (kn % kNSK) * kTK * A::KP, &kbar[kn % kNSK], t0,
                                    (int)(s1 - t0 < kTK ? s1 - t0 : kTK));
        }
      }
    }
  }
  // Per-head max of this CTA (max is order-independent; NaN never wins, as
  // with `if score > max_score`).
  lmax = warp_max(lmax);
  if (lane == 0) red_s[warp][warp % GP] = lmax;
  __syncthreads();
  if (tid < 8) {
    float m = -INFINITY;
    for (int w = tid; w < kXW; w += GP)
      if (tid < GP && red_s[w][tid] > m) m = red_s[w][tid];
    mx_s[tid] = m;
  }
  if (!ok) bad_s = 1;
  cluster.sync();
  if (tid < G) {
    float m = -INFINITY;
    for (int r = 0; r < cs; r++) {
      const float v = cluster.map_shared_rank(mx_s, r)[tid];
      if (v > m) m = v;
    }
    gmax_s[tid] = m;
  }
  __syncthreads();
  for (int i = tid; len > 0 && i < G * len; i += kXT) {
    const int g = i / len, j = i % len;
    sc[g * per_cap + j] = exact::exp_ref(__fsub_rn(sc[g * per_cap + j], gmax_s[g]));
  }
  cluster.sync();  // every rank's e_t is ready

  // Phase B: CTA g gathers head g's e_t in position order.
  const int g = rank;
  if (vsum)
    for (int64_t i = tid; i < span; i += kXT) {
      const int rr = (int)(i / per), j = (int)(i % per);
      E[i] = cluster.map_shared_rank(sc, rr)[g * per_cap + j];
    }
  cluster.sync();  // no remote reads after this point
  if (!vsum) {
    if (bad_s && tid == 0 && a.err) atomicOr(a.err, kErrCopyWait);
    return;
  }
  const float den = exact::seq_sum_nonneg<kXT>(E, (int)span, 0.0f, *(exact::SumSmem<kXT> *)(smem + L.sum));
  const float inv = den > 0.0f ? __fdiv_rn(1.0f, den) : 0.0f;
  for (int64_t i = tid; i < span; i += kXT) E[i] = __fmul_rn(E[i], inv);
  __syncthreads();

  float o = 0.0f;
  if (tid < HD) {  // output chain d = tid over all positions
    const int d = tid;
    for (int k = 0; k < nv; k++) {
      const int slot = k % A::NSV;
      if (!mbar_wait_bounded(&vfull[slot], (uint32_t)((k / A::NSV) & 1))) ok = false;
      const int64_t t0 = lo + (int64_t)k * kTV;
      const int n = (int)(seq - t0 < kTV ? seq - t0 : kTV);
      const char *vs = vring + slot * kTV * A::ROW;
      const float *w = E + (t0 - lo);
#pragma unroll 8
      for (int j = 0; j < n; j++) {
        float v = F16 ? __half2float(((const __half *)(vs + j * A::ROW))[d]) : ((const float *)(vs + j * A::ROW))[d];
        if (t0 + j == pos) v = vn_s[d];
        o = __fadd_rn(o, __fmul_rn(w[j], v));
      }
      mbar_arrive(&vempty[slot]);
    }
  } else if (tid == HD) {  // producer: refill a slot once every chain passed it
    for (int k = A::NSV; k < nv; k++) {
      const int slot = k % A::NSV;
      if (!mbar_wait_bounded(&vempty[slot], (uint32_t)(((k - A::NSV) / A::NSV) & 1))) ok = false;
      fence_proxy_async();
      const int64_t t0 = lo + (int64_t)k * kTV;
      issue_rows<HD, F16, false>(a.kv, a.layer, h, a.kv.v, vring + slot * kTV * A::ROW, &vfull[slot], t0,
                                 (int)(seq - t0 < kTV ? seq - t0 : kTV));
    }
  }
  if (tid < HD) {
    const int64_t e = (int64_t)(h * G + g) * HD + tid;
    a.out[e] = o;
    float v = isfinite(o) ? o : 0.0f;
    const float amax = warp_max(fabsf(v));
    const float scale = act_scale_from_amax(amax), is = act_inv_from_scale(scale);
    a.out_q[e] = act_quant_one(v, is);
    if (lane == 0) a.out_s[e / 32] = scale;
  }
  if (!ok) atomicOr(&bad_s, 1);
  __syncthreads();
  if (bad_s && tid == 0 && a.err) atomicOr(a.err, kErrCopyWait);
}

template <int HD, bool F16>
const void *xattn_fn() {
  return (const void *)k_xattn<HD, F16>;
}

const void *pick_x(int hd, int f16) {
  if (hd == 128) return f16 ? xattn_fn<128, true>() : xattn_fn<128, false>();
  if (hd == 64) return f16 ? xattn_fn<64, true>() : xattn_fn<64, false>();
  return nullptr;
}

size_t x_smem(int hd, int f16, int per_cap, int n_ctx) {
  if (hd == 128) return f16 ? xattn_layout<128, true>(per_cap, n_ctx).total : xattn_layout<128, false>(per_cap, n_ctx).total;
  return f16 ? xattn_layout<64, true>(per_cap, n_ctx).total : xattn_layout<64, false>(per_cap, n_ctx).total;
}

}  // namespace

int xattn_cluster_size(int head_dim, int f16, int G, int64_t n_ctx) {
  const void *fn = pick_x(head_dim, f16);
  if (!fn || G > 16) return 0;
  const int want = n_ctx >= 1024 ? 16 : 8;
  for (int cs = want; cs >= G && cs >= 1; cs /= 2) {
    const int per_cap = (int)((n_ctx + cs - 1) / cs);
    const size_t smem = x_smem(head_dim, f16, per_cap, (int)n_ctx);
    if (smem > 227 * 1024) continue;
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess && n > 0) return cs;
    cudaGetLastError();
  }
  return 0;
}

void launch_xattn_decode(const AttnDecodeArgs &a, int64_t n_ctx, cudaStream_t s) {
  const void *fn = pick_x((int)a.kv.head_dim, a.kv.f16);
  const int cs = a.n_splits;
  if (!fn || cs < 1) fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention: unsupported shape");
  const int per_cap = (int)((n_ctx + cs - 1) / cs);
  const size_t smem = x_smem((int)a.kv.head_dim, a.kv.f16, per_cap, (int)n_ctx);
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
  int nc = (int)n_ctx;
  void *args[] = {(void *)&a, (void *)&per_cap, (void *)&nc};
  cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace jal
