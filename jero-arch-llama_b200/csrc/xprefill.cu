// Prefill attention in the reference's f32 order (gqa_attention_prefill_portable,
// recipe.rs:2949-3022) over the paged KV cache, for m queries at
// start_pos..start_pos + m - 1 (causal, optional sliding window).
//
// Per (query, head): score_t = (sum_d q_d * k_td from -0.0, left to right) *
// scale over the valid keys t in [lo, pos]; e_t = exp(score_t - max); den =
// sequential sum of e_t from +0.0; w_t = e_t * (1 / den); out_d = sequential
// sum over t of w_t * v_td from +0.0.  One rounding per operation, no fused
// multiply-add, so the result equals the reference bit for bit (exp is the
// correctly rounded value; see exact::exp_ref).
//
// CTA = (query head, block of QB = 4 queries), 256 threads.  Keys of the
// block's range stream through a shared-memory tile (K pitched by 16 bytes so
// a warp scoring 32 keys at one offset stays conflict-free), loaded with
// cp.async one tile ahead.  Scores of the QB queries over the whole key range
// stay in shared memory (QB x keys floats).  Warp w scores query w % 4 over
// keys (w / 4) * 32 + lane of the tile, one sequential chain over d per
// score.  The four denominators are exact sequential sums computed at once
// by four 64-thread groups (exact::seq_sum_nonneg on named barriers).  The
// output chains (query, d) then run over the keys in order, two per thread,
// V streaming through the same tile buffers.
#include <cuda_fp16.h>

#include "attn_dev.cuh"
#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "exact.cuh"
#include "jal.h"

namespace jal {

namespace {

constexpr int kPT = 256, kQB = 4, kKT = 64;  // threads, queries per CTA, keys per tile

template <int HD, bool F16>
struct XP {
  static constexpr int ES = F16 ? 2 : 4;
  static constexpr int ROW = HD * ES;
  static constexpr int KP = ROW + 16;
  static constexpr int CH = 16 / ES;
  static constexpr int TILE = kKT * KP;  // bytes of one K (pitched) or V tile buffer
};

__device__ __forceinline__ void cpa16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Rows [k0, k0 + n) of KV head h of `base` into a tile with row pitch `pitch`.
template <int HD, bool F16>
__device__ void load_tile(const KvView &kv, int64_t layer, int h, const void *base, char *tile, int pitch, int64_t k0,
                          int n) {
  using A = XP<HD, F16>;
  constexpr int PR = A::ROW / 16;  // 16-byte pieces per row
  for (int i = threadIdx.x; i < n * PR; i += kPT) {
    const int j = i / PR, p = i % PR;
    const int64_t e = adev::kv_elem(kv, layer, h, k0 + j);
    cpa16(tile + j * pitch + p * 16, (const char *)base + e * A::ES + p * 16);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int HD, bool F16>
__global__ void __launch_bounds__(kPT, 1) k_xattn_prefill(const AttnPrefillArgs a, int smax) {
  using A = XP<HD, F16>;
  extern __shared__ __align__(16) char smem[];
  char *tiles = smem;                                  // 2 x TILE
  float *S = (float *)(smem + 2 * A::TILE);            // [kQB][smax]
  __shared__ exact::SumSmem<64> ssm[kQB];
  __shared__ __align__(16) float q_s[kQB][HD];
  __shared__ float red_s[8];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int hq = blockIdx.x, G = (int)(a.n_heads_q / a.kv.n_kv), h = hq / G;
  const int64_t q0 = (int64_t)blockIdx.y * kQB;
  const int nq = (int)(a.m - q0 < kQB ? a.m - q0 : kQB);
  // Key range of the block and of each query.
  int64_t qlo[kQB], qhi[kQB];
#pragma unroll
  for (int j = 0; j < kQB; j++) {
    const int64_t p = a.start_pos + q0 + (j < nq ? j : nq - 1);
    qhi[j] = p;
    qlo[j] = (a.window > 0 && p + 1 > a.window) ? p + 1 - a.window : 0;
  }
  const int64_t klo = qlo[0], khi = qhi[nq - 1];
  const int nk = (int)(khi - klo + 1), ntile = (nk + kKT - 1) / kKT;
  for (int i = tid; i < kQB * HD; i += kPT) {
    const int j = i / HD, d = i % HD;
    q_s[j][d] = j < nq ? a.qkv[(q0 + j) * a.qkv_stride + (int64_t)hq * HD + d] : 0.0f;
  }

  // Scores.
  load_tile<HD, F16>(a.kv, a.layer, h, a.kv.k, tiles, A::KP, klo, min(kKT, nk));
  const int jq = warp % kQB, ko = (warp / kQB) * 32 + lane;  // query and key slot of this thread
  float lmax = -INFINITY;
  for (int k = 0; k < ntile; k++) {
    if (k + 1 < ntile) {
      const int64_t k1 = klo + (int64_t)(k + 1) * kKT;
      load_tile<HD, F16>(a.kv, a.layer, h, a.kv.k, tiles + ((k + 1) & 1) * A::TILE, A::KP, k1,
                         (int)(khi + 1 - k1 < kKT ? khi + 1 - k1 : kKT));
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int64_t t = klo + (int64_t)k * kKT + ko;
    if (jq < nq && t >= qlo[jq] && t <= qhi[jq]) {
      const char *row = tiles + (k & 1) * A::TILE + ko * A::KP;
      float d = -0.0f;
#pragma unroll 4
      for (int c = 0; c < HD / A::CH; c++) {
        float kv[A::CH];
        adev::load_vals<F16, A::CH>(row + c * 16, kv);
#pragma unroll
        for (int e = 0; e < A::CH; e++) d = __fadd_rn(d, __fmul_rn(q_s[jq][c * A::CH + e], kv[e]));
      }
      const float s = __fmul_rn(d, a.scale);
      S[jq * smax + (int)(t - klo)] = s;
      if (s > lmax) lmax = s;
    }
    __syncthreads();  // the tile is consumed before it is refilled
  }
  // Per-query max: warps w and w + 4 score query w % 4.
  lmax = warp_max(lmax);
  if (lane == 0) red_s[warp] = lmax;
  // V tile 0 goes out while the softmax runs.
  load_tile<HD, F16>(a.kv, a.layer, h, a.kv.v, tiles, A::ROW, klo, min(kKT, nk));
  __syncthreads();
  // Group j (threads 64j .. 64j + 63) finishes query j's softmax terms.
  {
    const int j = tid / 64, gt = tid % 64;
    if (j < nq) {
      const float m = red_s[j] > red_s[j + 4] ? red_s[j] : red_s[j + 4];
      float *Sj = S + j * smax + (int)(qlo[j] - klo);
      const int n = (int)(qhi[j] - qlo[j] + 1);
      for (int i = gt; i < n; i += 64) Sj[i] = exact::exp_ref(__fsub_rn(Sj[i], m));
      exact::group_sync<64>(1 + j);
      const float den = exact::seq_sum_nonneg<64>(Sj, n, 0.0f, ssm[j], gt, 1 + j);
      const float inv = den > 0.0f ? __fdiv_rn(1.0f, den) : 0.0f;
      for (int i = gt; i < n; i += 64) Sj[i] = __fmul_rn(Sj[i], inv);
    }
  }
  __syncthreads();
  // Output chains: thread (pair jp, dim d) runs queries 2 jp and 2 jp + 1.
  const int d = tid % HD, jp = tid / HD;  // HD = 128: jp in {0, 1}; HD = 64: jp in {0..3}
  float o[2] = {0.0f, 0.0f};
  for (int k = 0; k < ntile; k++) {
    if (k + 1 < ntile) {
      const int64_t k1 = klo + (int64_t)(k + 1) * kKT;
      load_tile<HD, F16>(a.kv, a.layer, h, a.kv.v, tiles + ((k + 1) & 1) * A::TILE, A::ROW, k1,
                         (int)(khi + 1 - k1 < kKT ? khi + 1 - k1 : kKT));
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const char *vt = tiles + (k & 1) * A::TILE;
    const int64_t t0 = klo + (int64_t)k * kKT;
    const int n = (int)(khi + 1 - t0 < kKT ? khi + 1 - t0 : kKT);
    if (HD == 128 || jp < 2) {
      // Both chains of the thread walk the tile's keys together: keys in
      // [a0, b0) belong to both queries, the rest to one of them.  Each
      // chain still adds its terms in key order.
      const int j0 = 2 * jp, j1 = 2 * jp + 1;
      const bool v0 = j0 < nq, v1 = j1 < nq;
      auto lo_of = [&](int j) { return (int)((qlo[j] > t0 ? qlo[j] : t0) - t0); };
      auto hi_of = [&](int j) { return (int)((qhi[j] < t0 + n - 1 ? qhi[j] : t0 + n - 1) - t0); };  // inclusive
      const int l0 = v0 ? lo_of(j0) : n, h0 = v0 ? hi_of(j0) : -1, l1 = v1 ? lo_of(j1) : n, h1 = v1 ? hi_of(j1) : -1;
      const float *W0 = S + j0 * smax + (int)(t0 - klo), *W1 = S + j1 * smax + (int)(t0 - klo);
      auto val = [&](int i) {
        const char *row = vt + i * A::ROW;
        return F16 ? __half2float(((const __half *)row)[d]) : ((const float *)row)[d];
      };
      // Each chain's keys [l, h] of this tile split into the part below the
      // shared range [slo, shi], the shared range (one V load for both
      // terms) and the part above it, taken in that order.
      const int slo = l0 > l1 ? l0 : l1, shi = h0 < h1 ? h0 : h1;
      if (slo > shi) {
        for (int i = l0; i <= h0; i++) o[0] = __fadd_rn(o[0], __fmul_rn(W0[i], val(i)));
        for (int i = l1; i <= h1; i++) o[1] = __fadd_rn(o[1], __fmul_rn(W1[i], val(i)));
      } else {
        for (int i = l0; i < slo; i++) o[0] = __fadd_rn(o[0], __fmul_rn(W0[i], val(i)));
        for (int i = l1; i < slo; i++) o[1] = __fadd_rn(o[1], __fmul_rn(W1[i], val(i)));
#pragma unroll 4
        for (int i = slo; i <= shi; i++) {
          const float v = val(i);
          o[0] = __fadd_rn(o[0], __fmul_rn(W0[i], v));
          o[1] = __fadd_rn(o[1], __fmul_rn(W1[i], v));
        }
        for (int i = shi + 1; i <= h0; i++) o[0] = __fadd_rn(o[0], __fmul_rn(W0[i], val(i)));
        for (int i = shi + 1; i <= h1; i++) o[1] = __fadd_rn(o[1], __fmul_rn(W1[i], val(i)));
      }
    }
    __syncthreads();
  }
  if (HD == 128 || jp < 2) {
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int j = 2 * jp + u;
      if (j < nq) a.out[(q0 + j) * (a.n_heads_q * HD) + (int64_t)hq * HD + d] = o[u];
    }
  }
}

template <int HD, bool F16>
void launch_p(const AttnPrefillArgs &a, int smax, cudaStream_t s) {
  const size_t smem = 2 * (size_t)XP<HD, F16>::TILE + ((size_t)kQB * smax + exact::kSumSlack) * 4;  // + the sum's read slack
  cudaFuncSetAttribute(k_xattn_prefill<HD, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)a.n_heads_q, (unsigned)((a.m + kQB - 1) / kQB));
  k_xattn_prefill<HD, F16><<<grid, kPT, smem, s>>>(a, smax);
}

}  // namespace

// Keys one CTA may score: the block's range is at most (window or start + m).
bool xattn_prefill_supported(int64_t head_dim, int64_t max_keys) {
  if (head_dim != 64 && head_dim != 128) return false;
  const size_t smem = 2 * (size_t)(kKT * (head_dim * 4 + 16)) + ((size_t)kQB * (max_keys + kQB) + exact::kSumSlack) * 4;
  return smem <= 220 * 1024;
}

void launch_xattn_prefill(const AttnPrefillArgs &a, cudaStream_t s) {
  if (a.m <= 0) return;
  const int64_t end = a.start_pos + a.m;
  const int smax = (int)((a.window > 0 && a.window < end ? a.window : end) + kQB);
  if (!xattn_prefill_supported(a.kv.head_dim, smax))
    fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order prefill attention: %lld keys do not fit", (long long)smax);
  if (a.kv.head_dim == 128) {
    if (a.kv.f16) launch_p<128, true>(a, smax, s);
    else launch_p<128, false>(a, smax, s);
  } else {
    if (a.kv.f16) launch_p<64, true>(a, smax, s);
    else launch_p<64, false>(a, smax, s);
  }
}

}  // namespace jal
