// Decode GEMV in the reference's f32 order (M = 1), for the repacked Q4_0 /
// Q8_0 B200 layout.
//
// Semantics (repack_cache.rs:739-783): for each output row the 16-element
// integer chunk dots are exact; each chunk gives the term
// (f32(dot16) * a_sc) * w_sc, and the row value is the left-to-right f32 sum
// of the terms from +0.0 in chunk order.  Bias and residual are added after
// the fold (recipe.rs:2490-2518, 1004-1032); SwiGLU pairs gate row i with up
// row i (recipe.rs:3024-3050).
//
// Structure: one CTA of 16 warps per SM owns a contiguous, balanced range of
// output rows, taken in chunks of up to 32 physical rows (gate / up rows
// alternate for SwiGLU).  Warp 0 folds: lane r adds row r's terms in chunk
// order, a 16-byte read of four terms at a time, so a row costs ~1.25
// instructions per term whatever the number of rows.  Warps 1..15 produce
// the terms: a unit is one row segment of 128 blocks (4096 columns), read
// with non-allocating 16-byte loads that cover 512 consecutive bytes per warp
// instruction (Q4_0: lane l takes blocks 32v + l, two terms each; Q8_0: lane
// l takes the 16-element chunks 32j + l, one term each), DEPTH units ahead in
// registers; the lane stores its eight chunk terms in place in the chunk's
// term buffer ([rows][2 x columns / 32] floats); each unit arrives on its
// segment's mbarrier, on which the fold warp waits.  Two term buffers
// alternate when they fit, so producers fill chunk c + 1 while chunk c is
// folded.  Before griddepcontrol.wait each CTA starts a bulk L2 prefetch of
// its rows, so the weights stream from HBM while the activation prologue
// runs.
//
// The activation prologue (optional RMSNorm, then QuantizedActQ8 per
// 32-block) is computed by every CTA into shared memory after the wait: the
// 16 quants of each block half in two arrays indexed by block (the second
// shifted by 64 bytes, so Q8_0's alternating lo / hi reads use all 32
// banks); the RMSNorm sum of squares is the reference's sequential sum,
// computed with exact::seq_sum_nonneg.
#include <cuda_fp16.h>

#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "exact.cuh"
#include "jal.h"

namespace jal {

namespace {

constexpr int kNT = 512, kNW = kNT / 32;
constexpr int kSeg = 128;     // blocks per segment (4096 columns)
constexpr int kProdW = kNW - 1;  // term-producing warps (warp 0 folds)
constexpr int kMaxSeg = 8;    // columns <= 32768
constexpr size_t kTermCap = 160 * 1024;  // term buffers + activation
// L2 prefetch per CTA at launch: 148 CTAs x 512 KB stays well inside the
// 126 MB L2 while covering whole projections up to ~75 MB.
constexpr uint64_t kL2PrefetchBytes = 512 * 1024;

template <int QUANT>
struct XCfg {
  static constexpr int NQ4 = QUANT == JAL_Q4_0 ? 4 : 8;  // 16-byte quant loads per lane per unit
  static constexpr int DEPTH = QUANT == JAL_Q4_0 ? 3 : 2;
};

// Shared memory carve-up (bytes, 16-aligned pieces).  The prologue's
// scratch (the f32 input row, the norm weights, the squares and the exact
// sum's workspace) lives in the fold buffers' space, which the main loop
// uses only after the prologue.
struct XLayout {
  int nb, nseg, nbp;
  int cr, nbuf, pitch;  // rows per chunk (fold lanes), term buffers, buffer row pitch (floats)
  size_t act_lo, act_hi, act_m, buf, xin, nw, xsq, sum, total;
};

__host__ __device__ inline XLayout x_layout(int64_t cols, int in_mode) {
  XLayout L;
  L.nb = (int)(cols / 32);
  L.nseg = (L.nb + kSeg - 1) / kSeg;
  L.nbp = L.nseg * kSeg;
  size_t o = 0;
  L.act_lo = o; o += (size_t)L.nbp * 16 + 64;
  L.act_hi = o; o += (size_t)L.nbp * 16;
  L.act_m = o; o += (size_t)L.nbp * 16;
  L.buf = o;
  // A chunk's terms: [cr rows][2 nbp terms], pitch 2 nbp + 4 floats (an odd
  // number of 16-byte units: the fold lanes' 16-byte reads do not conflict).
  L.pitch = 2 * L.nbp + 4;
  L.cr = 32;
  while (L.cr > 8 && (size_t)L.cr * L.pitch * 4 + o > kTermCap) L.cr /= 2;
  L.nbuf = 2 * (size_t)L.cr * L.pitch * 4 + o <= kTermCap ? 2 : 1;
  const size_t fold = (size_t)L.nbuf * L.cr * L.pitch * 4;
  const size_t row = ((size_t)L.nb * 32 * 4 + 15) / 16 * 16;
  size_t p = o;
  L.xin = p; if (in_mode != GEMV_IN_Q8) p += row;
  L.nw = p; if (in_mode == GEMV_IN_NORM) p += row;
  L.xsq = p; if (in_mode == GEMV_IN_NORM) p += row;
  L.sum = p; if (in_mode == GEMV_IN_NORM) p += (sizeof(exact::SumSmem<kNT>) + 15) / 16 * 16;  // also the squares' read slack
  L.total = o + (fold > p - o ? fold : p - o);
  return L;
}

// Activation prologue: QuantizedActQ8 of the (optionally RMSNorm'd) input,
// one warp per 32-block, lane = element.  Per block slot: quants 0..15 in
// act_lo, 16..31 in act_hi, {scale, sum of quants 0..15, sum of 16..31, 0}
// in act_m.  Padding blocks are zero.
template <typename SumSM>
__device__ void x_prologue(const GemvArgs &a, const XLayout &L, char *smem, SumSM *ssm) {
  const int tid = threadIdx.x;
  int8_t *alo = (int8_t *)(smem + L.act_lo), *ahi = (int8_t *)(smem + L.act_hi);
  float4 *am = (float4 *)(smem + L.act_m);
  const int K = L.nb * 32;
  for (int b = L.nb + tid; b < L.nbp; b += kNT) {  // padding blocks
    const int sl = b;
    ((uint4 *)alo)[sl] = make_uint4(0u, 0u, 0u, 0u);
    ((uint4 *)ahi)[sl] = make_uint4(0u, 0u, 0u, 0u);
    am[sl] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // Four lanes per 32-block (lane sub = 0..3 holds elements 8 sub .. 8 sub +
  // 7): the block max and the chunk sums combine over the four lanes.
  const int jobs = L.nb * 4, jobs_r = (jobs + 31) & ~31;
  auto store = [&](int i, bool valid, const int (&q)[8], float scale) {
    const int b = i >> 2, sub = i & 3;
    int s = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) s += q[e];
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // sub 0, 1: elements 0..15; sub 2, 3: 16..31
    const int s_hi = __shfl_down_sync(0xffffffffu, s, 2);
    if (valid) {
      const int sl = b;
      const uint32_t p0 = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
                          ((uint32_t)(q[3] & 0xff) << 24);
      const uint32_t p1 = (uint32_t)(q[4] & 0xff) | ((uint32_t)(q[5] & 0xff) << 8) | ((uint32_t)(q[6] & 0xff) << 16) |
                          ((uint32_t)(q[7] & 0xff) << 24);
      int8_t *half = sub < 2 ? alo : ahi;
      *(uint2 *)(half + sl * 16 + (sub & 1) * 8) = make_uint2(p0, p1);
      if (sub == 0) am[sl] = make_float4(scale, __int_as_float(s), __int_as_float(s_hi), 0.f);
    }
  };
  if (a.in_mode == GEMV_IN_Q8) {
    for (int i = tid; i < jobs_r; i += kNT) {
      const bool valid = i < jobs;
      int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      float scale = 0.0f;
      if (valid) {
        const uint2 raw = *(const uint2 *)(a.xq + (int64_t)i * 8);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          q[e] = (int)(int8_t)((raw.x >> (8 * e)) & 0xff);
          q[4 + e] = (int)(int8_t)((raw.y >> (8 * e)) & 0xff);
        }
        scale = a.xs[i >> 2];
      }
      store(i, valid, q, scale);
    }
    __syncthreads();
    return;
  }
  // One pass of 16-byte loads, all issued before any use, stages the row
  // (and the norm weights, and the squares) in shared memory.
  float *xin = (float *)(smem + L.xin), *nw = (float *)(smem + L.nw), *xsq = (float *)(smem + L.xsq);
  const bool norm = a.in_mode == GEMV_IN_NORM;
  {
    constexpr int U = 8;
    const int n4 = K / 4;
    for (int i0 = 0; i0 < n4; i0 += U * kNT) {
      float4 xv[U], wv[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int i = i0 + u * kNT + tid;
        if (i < n4) {
          xv[u] = ((const float4 *)a.x)[i];
          if (norm) wv[u] = ((const float4 *)a.norm_w)[i];
        }
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int i = i0 + u * kNT + tid;
        if (i < n4) {
          ((float4 *)xin)[i] = xv[u];
          if (norm) {
            ((float4 *)nw)[i] = wv[u];
            ((float4 *)xsq)[i] = make_float4(__fmul_rn(xv[u].x, xv[u].x), __fmul_rn(xv[u].y, xv[u].y),
                                             __fmul_rn(xv[u].z, xv[u].z), __fmul_rn(xv[u].w, xv[u].w));
          }
        }
      }
    }
  }
  __syncthreads();
  float inv = 1.0f;
  if (norm) {
    const float ss = exact::seq_sum_nonneg<kNT>(xsq, K, -0.0f, *ssm);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
  }
  for (int i = tid; i < jobs_r; i += kNT) {
    const bool valid = i < jobs;
    float v[8];
    if (valid) {
      const float4 x0 = ((const float4 *)xin)[2 * i], x1 = ((const float4 *)xin)[2 * i + 1];
      v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w; v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
      if (norm) {
        const float4 w0 = ((const float4 *)nw)[2 * i], w1 = ((const float4 *)nw)[2 * i + 1];
        const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fmul_rn(v[e], inv), w[e]);
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
    const float scale = act_scale_from_amax(amax), is = act_inv_from_scale(scale);
    int q[8];
#pragma unroll
    for (int e = 0; e < 8; e++) q[e] = act_quant_one(v[e], is);
    store(i, valid, q, scale);
  }
  __syncthreads();
}

// f32 of an integer |d| < 2^22 without the conversion unit: 1.5 * 2^23 + d
// is exact in f32 (its bits are those of 1.5 * 2^23 plus d), and so is the
// difference.  Chunk dots stay below 16 * 128 * 127 < 2^22.
__device__ __forceinline__ float exact_i2f(int d) { return __fsub_rn(__int_as_float(0x4B400000 + d), 12582912.0f); }

// Quants and scales of one lane for one (row, segment) unit: four blocks
// (Q4_0) or eight 16-element chunks (Q8_0), and their blocks' f16 scales.
template <int QUANT>
struct XUnit {
  uint4 q[XCfg<QUANT>::NQ4];
  uint16_t d[XCfg<QUANT>::NQ4];
};

template <int QUANT>
__device__ __forceinline__ void x_load(const DevMat &w, int64_t row, int seg, int nb, int lane, XUnit<QUANT> &u) {
  const uint8_t *qp = w.qs + row * w.qs_stride;
  const uint16_t *dp = w.d + row * w.d_stride;
  if (QUANT == JAL_Q4_0) {
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const int b = seg * kSeg + 32 * v + lane;
      u.q[v] = b < nb ? ldg_stream16(qp + (int64_t)b * 16) : make_uint4(0u, 0u, 0u, 0u);
      u.d[v] = b < nb ? ldg_stream2(dp + b) : (uint16_t)0;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int t = 32 * j + lane, b = seg * kSeg + (t >> 1);
      u.q[j] = b < nb ? ldg_stream16(qp + (int64_t)seg * kSeg * 32 + 16 * t) : make_uint4(0u, 0u, 0u, 0u);
      u.d[j] = b < nb ? ldg_stream2(dp + b) : (uint16_t)0;
    }
  }
}

// The lane's chunk terms of a unit, stored at their chunk positions of the
// row's term array (dst = the segment's first term).  Blocks past the row's
// end carry zero quants and scales and store zero terms, which the fold
// does not read.
template <int QUANT>
__device__ __forceinline__ void x_terms(const XUnit<QUANT> &u, const int4 *alo, const int4 *ahi, const float4 *am,
                                        int seg, int lane, float *dst) {
  if (QUANT == JAL_Q4_0) {
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const int bi = 32 * v + lane, b = seg * kSeg + bi;
      const int4 xl = alo[b], xh = ahi[b];
      const float4 m = am[b];
      const uint4 q = u.q[v];
      int d0 = dp4a_us(q.x & 0x0F0F0F0Fu, xl.x, 0);
      d0 = dp4a_us(q.y & 0x0F0F0F0Fu, xl.y, d0);
      d0 = dp4a_us(q.z & 0x0F0F0F0Fu, xl.z, d0);
      d0 = dp4a_us(q.w & 0x0F0F0F0Fu, xl.w, d0);
      int d1 = dp4a_us(q.x & 0xF0F0F0F0u, xh.x, 0);
      d1 = dp4a_us(q.y & 0xF0F0F0F0u, xh.y, d1);
      d1 = dp4a_us(q.z & 0xF0F0F0F0u, xh.z, d1);
      d1 = dp4a_us(q.w & 0xF0F0F0F0u, xh.w, d1);
      d0 -= 8 * __float_as_int(m.y);             // nibble n encodes n - 8
      d1 = (d1 >> 4) - 8 * __float_as_int(m.z);  // high nibbles were multiplied by 16 in place
      const float ws = __half2float(__ushort_as_half(u.d[v]));
      *(float2 *)(dst + 2 * bi) = make_float2(__fmul_rn(__fmul_rn(exact_i2f(d0), m.x), ws),
                                              __fmul_rn(__fmul_rn(exact_i2f(d1), m.x), ws));
    }
  } else {
    const int4 *half = (lane & 1) ? ahi : alo;  // odd chunks are their blocks' second halves
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int t = 32 * j + lane, b = seg * kSeg + (t >> 1);
      const int4 x = half[b];
      const float4 m = am[b];
      const uint4 q = u.q[j];
      int d = dp4a_ss((int)q.x, x.x, 0);
      d = dp4a_ss((int)q.y, x.y, d);
      d = dp4a_ss((int)q.z, x.z, d);
      d = dp4a_ss((int)q.w, x.w, d);
      dst[t] = __fmul_rn(__fmul_rn(exact_i2f(d), m.x), __half2float(__ushort_as_half(u.d[j])));
    }
  }
}

template <int QUANT, int OUT>
__global__ void __launch_bounds__(kNT, 1) k_xgemv(const GemvArgs a) {
  const KernelTrace trace(a.trace);
  constexpr int DEPTH = XCfg<QUANT>::DEPTH;
  constexpr int PAIR = OUT == GEMV_OUT_SWIGLU ? 2 : 1;  // physical rows per logical row
  extern __shared__ __align__(16) char smem[];
  __shared__ __align__(8) uint64_t seg_full[2][kMaxSeg], buf_empty[2];
  const XLayout L = x_layout(a.w.cols, a.in_mode);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = a.rows / gridDim.x, rem = a.rows % gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * base + ((int64_t)blockIdx.x < rem ? blockIdx.x : rem);
  const int cnt = (int)(base + ((int64_t)blockIdx.x < rem ? 1 : 0));
  const int nseg = L.nseg, cr = L.cr, nbuf = L.nbuf, pitch = L.pitch;
  const int nphys = cnt * PAIR, nchunk = (nphys + cr - 1) / cr;
  auto prow = [&](int p) -> int64_t {  // physical row p of this CTA: gate / up alternate for SwiGLU
    const int64_t lr = r0 + p / PAIR;
    return (PAIR == 2 && (p & 1)) ? a.up_offset + lr : lr;
  };
  if (tid == 0) {
    for (int b = 0; b < 2; b++) {
      for (int sg = 0; sg < kMaxSeg; sg++) mbar_init(&seg_full[b][sg], cr);  // one arrival per row of the chunk
      mbar_init(&buf_empty[b], 1);
    }
    fence_barrier_init();
  }
  // This CTA's rows are one contiguous run of row records (two for SwiGLU):
  // start streaming them into L2 before waiting on the previous kernel, so
  // HBM works while the activation prologue runs.
  if (tid == 0 && cnt > 0) {
    const uint64_t rec = (uint64_t)a.w.qs_stride, cap = kL2PrefetchBytes / PAIR;
    const uint64_t bytes = (uint64_t)cnt * rec < cap ? (uint64_t)cnt * rec : cap;
    l2_prefetch_bulk(a.w.qs + r0 * a.w.qs_stride, bytes);
    if (PAIR == 2) l2_prefetch_bulk(a.w.qs + (a.up_offset + r0) * a.w.qs_stride, bytes);
  }
  pdl_wait();
  pdl_trigger();
  x_prologue(a, L, smem, (exact::SumSmem<kNT> *)(smem + L.sum));  // ends with a CTA barrier
  const int4 *alo = (const int4 *)(smem + L.act_lo), *ahi = (const int4 *)(smem + L.act_hi);
  const float4 *am = (const float4 *)(smem + L.act_m);
  float *terms = (float *)(smem + L.buf);  // [nbuf][cr][pitch]

  if (warp == 0) {
    // Fold warp: lane = physical row of the chunk; each row's terms are
    // added in chunk order, segment by segment as the producers finish them.
    for (int c = 0; c < nchunk; c++) {
      const int b = c % nbuf;
      const uint32_t par = (uint32_t)((c / nbuf) & 1);
      const int p = c * cr + lane;
      const bool valid = lane < cr && p < nphys;
      const float *src = terms + ((size_t)b * cr + (lane < cr ? lane : 0)) * pitch;
      float acc = 0.0f;
      for (int sg = 0; sg < nseg; sg++) {
        mbar_wait_bounded(&seg_full[b][sg], par);
        const int blk = L.nb - sg * kSeg < kSeg ? L.nb - sg * kSeg : kSeg;
        const float *t = src + sg * 2 * kSeg;
        if (valid) {
          int i = 0;
          for (; i + 16 <= 2 * blk; i += 16) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = *(const float4 *)(t + i + 4 * u);
#pragma unroll
            for (int u = 0; u < 4; u++)
              acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v[u].x), v[u].y), v[u].z), v[u].w);
          }
          for (; i < 2 * blk; i++) acc = __fadd_rn(acc, t[i]);
        }
      }
      const float other = __shfl_down_sync(0xffffffffu, acc, 1);
      if (valid && (PAIR == 1 || (lane & 1) == 0)) {
        const int64_t lr = r0 + p / PAIR;
        float *yp = a.y + lr;
        if (OUT == GEMV_OUT_STORE) {
          *yp = a.bias ? __fadd_rn(acc, a.bias[lr]) : acc;
        } else if (OUT == GEMV_OUT_ADD) {
          const float pv = a.bias ? __fadd_rn(acc, a.bias[lr]) : acc;
          *yp = __fadd_rn(*yp, pv);
        } else {
          *yp = exact::swiglu_ref(acc, other);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&buf_empty[b]);
    }
    return;
  }

  // Producer warps: units (chunk, segment, row) in that order, unit g of
  // the CTA to warp g % kProdW.  A unit is one row segment: each lane
  // computes eight of its chunk terms and stores them in place; the unit's
  // warp then arrives on the segment's barrier (rows past the
  // CTA's end arrive without work, so every barrier counts cr arrivals).
  const int pw = warp - 1, upc = nseg * cr;
  const int crs = 31 - __clz(cr);  // cr is a power of two
  struct Cursor {
    int c, u;  // chunk, unit in the chunk (segment-major)
  };
  auto advance = [&](Cursor &q) {
    q.u += kProdW;
    while (q.u >= upc) {
      q.u -= upc;
      q.c++;
    }
  };
  XUnit<QUANT> ring[DEPTH];
  Cursor cur = {0, pw}, ahead = cur;
  while (ahead.u >= upc && upc > 0) {
    ahead.u -= upc;
    ahead.c++;
  }
  cur = ahead;
#pragma unroll
  for (int j = 0; j < DEPTH; j++) {
    const int p = ahead.c * cr + (ahead.u & (cr - 1));
    if (ahead.c < nchunk && p < nphys) x_load<QUANT>(a.w, prow(p), ahead.u >> crs, L.nb, lane, ring[j]);
    advance(ahead);
  }
  int waited = -1;  // last chunk whose buffer this warp has waited for

  for (int k0 = 0; cur.c < nchunk; k0 += DEPTH) {
#pragma unroll
    for (int j = 0; j < DEPTH; j++) {
      if (cur.c < nchunk) {
        const int c = cur.c, sg = cur.u >> crs, rr = cur.u & (cr - 1), p = c * cr + rr, b = c % nbuf;
        advance(cur);
        if (c >= nbuf && c != waited) {  // the fold warp has released this buffer
          mbar_wait_bounded(&buf_empty[b], (uint32_t)(((c / nbuf) - 1) & 1));
          waited = c;
        }
        if (p < nphys) x_terms<QUANT>(ring[j], alo, ahi, am, sg, lane, terms + ((size_t)b * cr + rr) * pitch + sg * 2 * kSeg);
        const int pa = ahead.c * cr + (ahead.u & (cr - 1));
        if (ahead.c < nchunk && pa < nphys) x_load<QUANT>(a.w, prow(pa), ahead.u >> crs, L.nb, lane, ring[j]);
        advance(ahead);
        __syncwarp();
        if (lane == 0) mbar_arrive(&seg_full[b][sg]);
      }
    }
  }
}

template <int QUANT, int OUT>
void launch_x(const GemvArgs &a, int grid, cudaStream_t s) {
  const XLayout L = x_layout(a.w.cols, a.in_mode);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_xgemv<QUANT, OUT>, a);
}

template <int QUANT>
void set_x_attrs() {
  cudaFuncSetAttribute(k_xgemv<QUANT, GEMV_OUT_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
  cudaFuncSetAttribute(k_xgemv<QUANT, GEMV_OUT_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
  cudaFuncSetAttribute(k_xgemv<QUANT, GEMV_OUT_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
}

}  // namespace

size_t xgemv_smem_bytes(int quant, int64_t cols, int in_mode) {
  (void)quant;
  return x_layout(cols, in_mode).total;
}

bool xgemv_supported(const GemvArgs &a) {
  if (a.m != 1 || (a.w.quant != JAL_Q4_0 && a.w.quant != JAL_Q8_0)) return false;
  if (x_layout(a.w.cols, a.in_mode).nseg > kMaxSeg) return false;
  if (a.w.cols % 32 != 0 || a.w.qs_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(a.w.qs) & 15) != 0) return false;
  if (a.out_mode != GEMV_OUT_STORE && a.out_mode != GEMV_OUT_ADD && a.out_mode != GEMV_OUT_SWIGLU) return false;
  if (a.peer_in || a.in_mode == GEMV_IN_PREQ) return false;
  return xgemv_smem_bytes(a.w.quant, a.w.cols, a.in_mode) <= 220 * 1024;
}

void xgemv_init() {
  static bool done = false;
  if (done) return;
  set_x_attrs<JAL_Q4_0>();
  set_x_attrs<JAL_Q8_0>();
  done = true;
}

void project_q8(const DevMat &w, const int8_t *xq, const float *xs, int64_t m, float *y, cudaStream_t s) {
  if (m <= 0 || w.rows <= 0) return;
  GemvArgs a;
  a.w = w; a.rows = w.rows; a.m = 1; a.in_mode = GEMV_IN_Q8; a.xq = xq; a.xs = xs; a.xq_stride = w.cols;
  a.out_mode = GEMV_OUT_STORE; a.y = y; a.y_stride = w.rows;
  if (m == 1 && xgemv_supported(a)) {
    launch_xgemv(a, s);
    return;
  }
  GemmArgs g;
  g.w = w; g.m = m; g.rows = w.rows; g.xq = xq; g.xs = xs; g.y = y; g.y_stride = w.rows;
  launch_gemm(g, s);
}

void launch_xgemv(const GemvArgs &a, cudaStream_t s) {
  if (a.rows <= 0) return;
  if (!xgemv_supported(a)) fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order GEMV: unsupported shape or mode");
  xgemv_init();
  int grid = a.grid;
  if (grid <= 0) {
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    grid = (int)(a.rows < sms ? a.rows : sms);
  }
  if (a.w.quant == JAL_Q4_0) {
    if (a.out_mode == GEMV_OUT_STORE) launch_x<JAL_Q4_0, GEMV_OUT_STORE>(a, grid, s);
    else if (a.out_mode == GEMV_OUT_ADD) launch_x<JAL_Q4_0, GEMV_OUT_ADD>(a, grid, s);
    else launch_x<JAL_Q4_0, GEMV_OUT_SWIGLU>(a, grid, s);
  } else {
    if (a.out_mode == GEMV_OUT_STORE) launch_x<JAL_Q8_0, GEMV_OUT_STORE>(a, grid, s);
    else if (a.out_mode == GEMV_OUT_ADD) launch_x<JAL_Q8_0, GEMV_OUT_ADD>(a, grid, s);
    else launch_x<JAL_Q8_0, GEMV_OUT_SWIGLU>(a, grid, s);
  }
}

}  // namespace jal
