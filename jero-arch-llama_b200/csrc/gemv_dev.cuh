// Device building blocks of the decode GEMVs, shared by the per-projection
// kernels (gemv.cu) and the persistent decode kernel (decode_mega.cu):
// the activation prologue (RMSNorm / f32 -> QuantizedActQ8 in shared
// memory), the SwiGLU epilogue and the segmented fast path's per-lane
// loads and block dots.
#pragma once

#include <cuda_fp16.h>

#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {
namespace gdev {

// Shared-memory activation layout for token t (nbp = nb rounded up to 32,
// the padding blocks zero):
//   [lo: nbp x 16 B][hi: nbp x 16 B][scale, sum32: nbp x 8 B]
// followed, for RMSNorm inputs, by the norm weights (K floats).
__host__ __device__ inline size_t act_bytes(int nbp) { return (size_t)nbp * 40; }
__host__ __device__ inline size_t smem_bytes(int in_mode, int M, int nb) {
  const int nbp = (nb + 31) & ~31;
  size_t b = act_bytes(nbp) * M;
  if (in_mode == GEMV_IN_NORM) b += (size_t)nb * 32 * 4;
  return b;
}

// Barrier over the first NT threads: __syncthreads for BAR 0, else the named
// barrier BAR (for kernels where some warps skip the activation prologue).
template <int BAR, int NT>
__device__ __forceinline__ void group_sync() {
  if constexpr (BAR == 0) __syncthreads();
  else asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
}

template <int WARPS, int BAR = 0>
__device__ float block_reduce_sum(float v, float *red) {
  v = warp_sum(v);
  int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  group_sync<BAR, WARPS * 32>();
  if (w == 0) {
    float t = l < WARPS ? red[l] : 0.0f;
    t = warp_sum(t);
    if (l == 0) red[32] = t;
  }
  group_sync<BAR, WARPS * 32>();
  float r = red[32];
  group_sync<BAR, WARPS * 32>();
  return r;
}

__device__ __forceinline__ void put_scale_sum(char *base, int nbp, int b, float scale, int sum32) {
  ((float2 *)(base + nbp * 32))[b] = make_float2(scale, __int_as_float(sum32));
}

// Activation prologue (QuantizedActQ8 per 32-block: amax over the block,
// scale = amax / 127, q = clamp(round(v * (1 / scale)))), written to shared
// memory with the block's int sum; one barrier at the end (plus one block
// reduction for RMSNorm).  Inputs are read straight from global memory; norm
// weights were staged in shared memory before griddepcontrol.wait.
template <int M, int WARPS, int BAR = 0>
__device__ void gemv_prologue(const GemvArgs &a, char *smem, int nb, int nbp, float *red) {
  constexpr int T = WARPS * 32;
  const int K = nb * 32, tid = threadIdx.x;
  if (nbp > nb) {  // padding blocks: zero quants, zero scale and sum
    for (int i = tid; i < M * (nbp - nb); i += T) {
      const int t = i / (nbp - nb), b = nb + i % (nbp - nb);
      char *base = smem + t * act_bytes(nbp);
      ((uint4 *)base)[b] = make_uint4(0, 0, 0, 0);
      ((uint4 *)(base + nbp * 16))[b] = make_uint4(0, 0, 0, 0);
      put_scale_sum(base, nbp, b, 0.0f, 0);
    }
  }
  if (a.in_mode == GEMV_IN_Q8) {
    for (int i = tid; i < M * nb; i += T) {
      const int t = i / nb, b = i % nb;
      char *base = smem + t * act_bytes(nbp);
      int4 lo = make_int4(0, 0, 0, 0), hi = lo;
      float sc = 0.0f;
      if (t < a.m) {
        const int4 *p = (const int4 *)(a.xq + t * a.xq_stride + b * 32);
        lo = p[0];
        hi = p[1];
        sc = a.xs[t * (a.xq_stride / 32) + b];
      }
      int s = dp4a_ss(lo.x, 0x01010101, 0);
      s = dp4a_ss(lo.y, 0x01010101, s);
      s = dp4a_ss(lo.z, 0x01010101, s);
      s = dp4a_ss(lo.w, 0x01010101, s);
      s = dp4a_ss(hi.x, 0x01010101, s);
      s = dp4a_ss(hi.y, 0x01010101, s);
      s = dp4a_ss(hi.z, 0x01010101, s);
      s = dp4a_ss(hi.w, 0x01010101, s);
      ((int4 *)base)[b] = lo;
      ((int4 *)(base + nbp * 16))[b] = hi;
      put_scale_sum(base, nbp, b, sc, s);
    }
    group_sync<BAR, WARPS * 32>();
    return;
  }
  // f32 inputs: four lanes per 32-block (8 consecutive elements each; the
  // block max and int sum combine over the 4-lane group with two shuffles).
  const bool norm = a.in_mode == GEMV_IN_NORM;
  const float *normw = (const float *)(smem + act_bytes(nbp) * M);
  const int jobs = M * nb * 4, jobs_r = (jobs + 31) & ~31;  // whole warps per iteration
  float inv_norm[M];
#pragma unroll
  for (int t = 0; t < M; t++) inv_norm[t] = 1.0f;
  if (norm) {
    float ss[M];
#pragma unroll
    for (int t = 0; t < M; t++) ss[t] = 0.0f;
    for (int i = tid; i < nb * 4; i += T) {
#pragma unroll
      for (int t = 0; t < M; t++) {
        if (t < a.m) {
          const float4 *xp = (const float4 *)(a.x + t * a.x_stride + i * 8);
#pragma unroll
          for (int j = 0; j < 2; j++) {
            const float4 v = xp[j];
            ss[t] = fmaf(v.x, v.x, ss[t]);
            ss[t] = fmaf(v.y, v.y, ss[t]);
            ss[t] = fmaf(v.z, v.z, ss[t]);
            ss[t] = fmaf(v.w, v.w, ss[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < M; t++) {
      if (t < a.m) {
        const float tot = block_reduce_sum<WARPS, BAR>(ss[t], red);
        inv_norm[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
      }
    }
  }
  for (int i = tid; i < jobs_r; i += T) {
    const bool valid = i < jobs;
    const int blk = i >> 2, sub = i & 3;
    const int t = valid ? blk / nb : 0, b = valid ? blk % nb : 0;
    const bool live = valid && t < a.m;
    float invn = inv_norm[0];
#pragma unroll
    for (int tt = 1; tt < M; tt++)
      if (tt == t) invn = inv_norm[tt];
    float v[8];
    if (live) {
      const float4 *xp = (const float4 *)(a.x + t * a.x_stride + b * 32 + sub * 8);
      const float4 x0 = xp[0], x1 = xp[1];
      v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
      v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
      if (norm) {
        const float4 *wp = (const float4 *)(normw + b * 32 + sub * 8);
        const float4 w0 = wp[0], w1 = wp[1];
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fmul_rn(v[e], invn), w[e]);
      }
#pragma unroll
      for (int e = 0; e < 8; e++)
        if (!isfinite(v[e])) v[e] = 0.0f;
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = 0.0f;
    }
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(v[e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
    int q[8], s = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      q[e] = act_quant_one(v[e], inv);
      s += q[e];
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (valid) {
      char *base = smem + t * act_bytes(nbp);
      const uint32_t p0 = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
                          ((uint32_t)(q[3] & 0xff) << 24);
      const uint32_t p1 = (uint32_t)(q[4] & 0xff) | ((uint32_t)(q[5] & 0xff) << 8) | ((uint32_t)(q[6] & 0xff) << 16) |
                          ((uint32_t)(q[7] & 0xff) << 24);
      // elements sub*8 .. sub*8+7: sub 0, 1 in the low 16 bytes, 2, 3 in the high
      char *half = sub < 2 ? base + b * 16 : base + nbp * 16 + b * 16;
      *(uint2 *)(half + (sub & 1) * 8) = make_uint2(p0, p1);
      if (sub == 0) put_scale_sum(base, nbp, b, live ? scale : 0.0f, live ? s : 0);
    }
  }
  group_sync<BAR, WARPS * 32>();
}

// Norm weights are static, so they are staged before griddepcontrol.wait.
template <int M, int WARPS>
__device__ void gemv_prologue_pre(const GemvArgs &a, char *smem, int nb, int nbp) {
  if (a.in_mode != GEMV_IN_NORM) return;
  const int K = nb * 32;
  float *normw = (float *)(smem + act_bytes(nbp) * M);
  for (int i = threadIdx.x; i < K / 4; i += WARPS * 32) ((float4 *)normw)[i] = ((const float4 *)a.norm_w)[i];
}

// M = 1 prologue for f32 / RMSNorm inputs with every global load issued
// before any use: each thread reads its JMAX jobs of 8 consecutive elements
// (and their norm weights) into registers at once, so the prologue costs one
// memory round trip plus the norm reduction.  Same quantization as
// gemv_prologue; padding blocks [nb, nbp) are zeroed.
template <int WARPS, int JMAX, bool NORM, bool PEER = false>
__device__ __forceinline__ void prologue_m1_impl(const GemvArgs &a, char *smem, int nb, int nbp, float *red) {
  constexpr int T = WARPS * 32;
  const int tid = threadIdx.x, jobs = nb * 4;
  for (int b = nb + tid; b < nbp; b += T) {
    ((uint4 *)smem)[b] = make_uint4(0, 0, 0, 0);
    ((uint4 *)(smem + nbp * 16))[b] = make_uint4(0, 0, 0, 0);
    put_scale_sum(smem, nbp, b, 0.0f, 0);
  }
  // Tensor-parallel exchange: each thread waits for the flagged words of its
  // own elements from every rank.
  constexpr bool peer = NORM && PEER;
  const uint32_t flag = peer ? ld_relaxed_gpu_u32(a.peer_epoch) * 256u + (uint32_t)a.peer_phase + 1u : 0u;
  bool peer_ok = true;
  float v[JMAX][8], w[NORM ? JMAX : 1][8];
#pragma unroll
  for (int j = 0; j < JMAX; j++) {
    const int i = tid + j * T;
    if (i < jobs) {
      const float4 *xp = (const float4 *)(a.x + i * 8);
      const float4 x0 = xp[0], x1 = xp[1];
      v[j][0] = x0.x; v[j][1] = x0.y; v[j][2] = x0.z; v[j][3] = x0.w;
      v[j][4] = x1.x; v[j][5] = x1.y; v[j][6] = x1.z; v[j][7] = x1.w;
      if (peer) {  // residual + partials in rank order
        for (int r = 0; r < a.peer_world; r++)
          peer_ok = peer_take8(a.peer_in + (size_t)r * a.x_stride + i * 8, flag, v[j], a.peer_wait_ns) && peer_ok;
        if (blockIdx.x == 0 && a.x_out) {
          float4 *op = (float4 *)(a.x_out + i * 8);
          op[0] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
          op[1] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
        }
      }
      if (NORM) {
        const float4 *wp = (const float4 *)(a.norm_w + i * 8);
        const float4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
        w[NORM ? j : 0][0] = w0.x; w[NORM ? j : 0][1] = w0.y; w[NORM ? j : 0][2] = w0.z; w[NORM ? j : 0][3] = w0.w;
        w[NORM ? j : 0][4] = w1.x; w[NORM ? j : 0][5] = w1.y; w[NORM ? j : 0][6] = w1.z; w[NORM ? j : 0][7] = w1.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) v[j][e] = 0.0f;
    }
  }
  if (peer && !peer_ok && a.err) atomicOr(a.err, kErrPeerWait);
  float invn = 1.0f;
  if (NORM) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < JMAX; j++)
#pragma unroll
      for (int e = 0; e < 8; e++) ss = fmaf(v[j][e], v[j][e], ss);
    const float tot = block_reduce_sum<WARPS>(ss, red);
    invn = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)(nb * 32)), a.eps)));
  }
  const int jobs_r = (jobs + 31) & ~31;  // whole warps take part in the shuffles
#pragma unroll
  for (int j = 0; j < JMAX; j++) {
    const int i = tid + j * T;
    if (j * T >= jobs_r) break;
    if (i >= jobs_r) continue;
    const bool valid = i < jobs;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      float t = v[j][e];
      if (NORM && valid) t = __fmul_rn(__fmul_rn(t, invn), w[NORM ? j : 0][e]);
      x[e] = isfinite(t) ? t : 0.0f;
    }
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(x[e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
    int q[8], s = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      q[e] = act_quant_one(x[e], inv);
      s += q[e];
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (valid) {
      const int b = i >> 2, sub = i & 3;
      const uint32_t p0 = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
                          ((uint32_t)(q[3] & 0xff) << 24);
      const uint32_t p1 = (uint32_t)(q[4] & 0xff) | ((uint32_t)(q[5] & 0xff) << 8) | ((uint32_t)(q[6] & 0xff) << 16) |
                          ((uint32_t)(q[7] & 0xff) << 24);
      char *half = sub < 2 ? smem + b * 16 : smem + nbp * 16 + b * 16;
      *(uint2 *)(half + (sub & 1) * 8) = make_uint2(p0, p1);
      if (sub == 0) put_scale_sum(smem, nbp, b, scale, s);
    }
  }
  __syncthreads();
}

// M = 1 prologue: the one-round-trip form when the row fits (RMSNorm rows up
// to 8192 elements, f32 rows up to 16384), else gemv_prologue.  Q8 inputs
// are already one round trip in gemv_prologue.
// PEER: the tensor-parallel exchange input (RMSNorm rows only; the host
// checks the shape).
template <int WARPS, bool PEER = false>
__device__ __forceinline__ void gemv_prologue_m1(const GemvArgs &a, char *smem, int nb, int nbp, float *red) {
  constexpr int T = WARPS * 32, JN = 1024 / T, JF = 2048 / T;
  if (PEER) {
    prologue_m1_impl<WARPS, JN, true, true>(a, smem, nb, nbp, red);
  } else if (a.in_mode == GEMV_IN_NORM && nb * 4 <= JN * T) {
    prologue_m1_impl<WARPS, JN, true>(a, smem, nb, nbp, red);
  } else if (a.in_mode == GEMV_IN_F32 && nb * 4 <= JF * T) {
    prologue_m1_impl<WARPS, JF, false>(a, smem, nb, nbp, red);
  } else {
    gemv_prologue_pre<1, WARPS>(a, smem, nb, nbp);
    gemv_prologue<1, WARPS>(a, smem, nb, nbp, red);
  }
}

__device__ __forceinline__ float swiglu_one(float g, float u) {
  // swiglu_compat (recipe.rs:3037-3047)
  float sig = g <= -20.0f ? 0.0f : (g >= 20.0f ? 1.0f : __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

constexpr int kSegBlocks = 128;

template <int QUANT>
struct W4Row {
  static constexpr int NQ = QUANT == JAL_Q4_0 ? 16 : 32;  // u32 of quants per lane
  uint32_t q[NQ];
  uint2 d;  // four f16 scales
};

// Segment `seg` of `row`; lanes past the row end (ragged last segment) load
// zeros.
// WIDE selects 32-byte loads; the 16-byte form is for code that ptxas
// compiles as a separate (non-inlined) function, where the 32-byte form is
// rejected.
template <int QUANT, bool WIDE = true>
__device__ __forceinline__ void w4_load(const DevMat &w, int64_t row, int seg, int nb, int lane, W4Row<QUANT> &r) {
  constexpr int NQ = W4Row<QUANT>::NQ;
  const int b0 = seg * kSegBlocks + 4 * lane;
  if (b0 < nb) {
    const uint8_t *q = w.qs + row * w.qs_stride + (size_t)b0 * (NQ / 4) * 4;
    if constexpr (WIDE) {
#pragma unroll
      for (int j = 0; j < NQ / 8; j++) ldg_stream32(q + 32 * j, &r.q[8 * j]);
    } else {
#pragma unroll
      for (int j = 0; j < NQ / 4; j++) {
        const uint4 v = ldg_stream16(q + 16 * j);
        r.q[4 * j] = v.x;
        r.q[4 * j + 1] = v.y;
        r.q[4 * j + 2] = v.z;
        r.q[4 * j + 3] = v.w;
      }
    }
    r.d = ldg_stream8(w.d + row * w.d_stride + b0);
  } else {
#pragma unroll
    for (int j = 0; j < NQ; j++) r.q[j] = 0u;
    r.d = make_uint2(0u, 0u);
  }
}

struct W4Act {
  int4 lo[4], hi[4];
  float sc[4];
  int sum[4];
};

template <int QUANT>
__device__ __forceinline__ float w4_dot(const W4Row<QUANT> &r, const W4Act &x) {
  const __half2 d01 = *reinterpret_cast<const __half2 *>(&r.d.x);
  const __half2 d23 = *reinterpret_cast<const __half2 *>(&r.d.y);
  const float ws[4] = {__low2float(d01), __high2float(d01), __low2float(d23), __high2float(d23)};
  float acc = 0.0f;
#pragma unroll
  for (int v = 0; v < 4; v++) {
    int dot;
    if constexpr (QUANT == JAL_Q4_0) {
      const uint32_t *w = &r.q[4 * v];
      int d0 = dp4a_us(w[0] & 0x0F0F0F0Fu, x.lo[v].x, 0);
      int d1 = dp4a_us(w[0] & 0xF0F0F0F0u, x.hi[v].x, 0);
      d0 = dp4a_us(w[1] & 0x0F0F0F0Fu, x.lo[v].y, d0);
      d1 = dp4a_us(w[1] & 0xF0F0F0F0u, x.hi[v].y, d1);
      d0 = dp4a_us(w[2] & 0x0F0F0F0Fu, x.lo[v].z, d0);
      d1 = dp4a_us(w[2] & 0xF0F0F0F0u, x.hi[v].z, d1);
      d0 = dp4a_us(w[3] & 0x0F0F0F0Fu, x.lo[v].w, d0);
      d1 = dp4a_us(w[3] & 0xF0F0F0F0u, x.hi[v].w, d1);
      dot = d0 + (d1 >> 4) - 8 * x.sum[v];  // nibble n encodes n - 8
    } else {
      const uint32_t *w = &r.q[8 * v];
      int d0 = dp4a_ss((int)w[0], x.lo[v].x, 0);
      int d1 = dp4a_ss((int)w[4], x.hi[v].x, 0);
      d0 = dp4a_ss((int)w[1], x.lo[v].y, d0);
      d1 = dp4a_ss((int)w[5], x.hi[v].y, d1);
      d0 = dp4a_ss((int)w[2], x.lo[v].z, d0);
      d1 = dp4a_ss((int)w[6], x.hi[v].z, d1);
      d0 = dp4a_ss((int)w[3], x.lo[v].w, d0);
      d1 = dp4a_ss((int)w[7], x.hi[v].w, d1);
      dot = d0 + d1;
    }
    acc = fmaf(__int2float_rn(dot), x.sc[v] * ws[v], acc);
  }
  return acc;
}

// Row segment of one weight row in shared memory (same layout as in HBM:
// quants, then the f16 scales): blocks bq[v] = seg * 128 + lane + 32 v, v < 4.
// Blocks past the row end (ragged last segment) read block 0 and are zeroed
// by mask bit v, without branches.
template <int QUANT>
__device__ __forceinline__ void w4s_load(const char *row, int nb, const int (&bq)[4], unsigned vmask,
                                         W4Row<QUANT> &r) {
  constexpr int BQ = QUANT == JAL_Q4_0 ? 16 : 32;  // quant bytes per block
  const uint16_t *d = (const uint16_t *)(row + (size_t)nb * BQ);
  uint32_t h[4];
#pragma unroll
  for (int v = 0; v < 4; v++) {
    const bool ok = (vmask >> v) & 1u;
    const uint4 q0 = *(const uint4 *)(row + (size_t)bq[v] * BQ);
    r.q[(BQ / 4) * v + 0] = ok ? q0.x : 0u; r.q[(BQ / 4) * v + 1] = ok ? q0.y : 0u;
    r.q[(BQ / 4) * v + 2] = ok ? q0.z : 0u; r.q[(BQ / 4) * v + 3] = ok ? q0.w : 0u;
    if (BQ == 32) {
      const uint4 q1 = *(const uint4 *)(row + (size_t)bq[v] * BQ + 16);
      r.q[(BQ / 4) * v + 4] = ok ? q1.x : 0u; r.q[(BQ / 4) * v + 5] = ok ? q1.y : 0u;
      r.q[(BQ / 4) * v + 6] = ok ? q1.z : 0u; r.q[(BQ / 4) * v + 7] = ok ? q1.w : 0u;
    }
    h[v] = ok ? (uint32_t)d[bq[v]] : 0u;
  }
  r.d = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

__host__ __device__ inline int seg_count(int64_t cols) { return (int)((cols / 32 + kSegBlocks - 1) / kSegBlocks); }
// Activation area of the segmented path: blocks padded to nseg * 128 (the
// padding zero), then the norm weights for RMSNorm inputs.
__host__ __device__ inline size_t w4_act_region(int in_mode, int nb, int nseg) {
  size_t b = act_bytes(nseg * kSegBlocks);
  if (in_mode == GEMV_IN_NORM) b += (size_t)nb * 32 * 4;
  return (b + 15) / 16 * 16;
}
__host__ __device__ inline size_t w4_smem(int in_mode, int nb, int nseg, int64_t max_rows) {
  const size_t act = w4_act_region(in_mode, nb, nseg);
  return nseg > 1 ? act + (size_t)max_rows * nseg * 4 : act;
}

}  // namespace gdev
}  // namespace jal
