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
// output rows; warp w takes rows w, w + 16, ... of it, eight physical rows
// (four gate / up pairs for SwiGLU) at a time.  A row is streamed in
// segments of 128 blocks (4096 columns): lane l owns blocks 4l .. 4l + 3 of
// the segment, loads their quants (64 bytes for Q4_0, 128 for Q8_0) and four
// f16 scales with non-allocating vector loads, DEPTH units (row, segment)
// ahead in registers, and writes its eight chunk terms, in chunk order, into
// the warp's buffer row for that physical row.  When the eight rows' segment is in the buffer, lanes 0 .. 7
// each add one row's terms in order onto that row's accumulator.  No CTA
// barrier is involved after the prologue; the serial adds (256 per segment)
// of one batch run while the next batch's loads are in flight.  Before
// griddepcontrol.wait each CTA starts a bulk L2 prefetch of its rows, so
// the weights stream from HBM while the activation prologue runs.
//
// The activation prologue (optional RMSNorm, then QuantizedActQ8 per
// 32-block) is computed by every CTA into shared memory after the wait, in a
// lane-interleaved layout (block 4l + v of a segment at slot 32v + l) so the
// main loop's reads are conflict-free; the RMSNorm sum of squares is the
// reference's sequential sum, computed with exact::seq_sum_nonneg.
#include <cuda_fp16.h>

#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "exact.cuh"
#include "jal.h"

namespace jal {

namespace {

constexpr int kNT = 512, kNW = kNT / 32;
constexpr int kSeg = 128;   // blocks per segment (4096 columns)
constexpr int kBR = 8;      // physical rows per warp batch (fold lanes)
constexpr int kBP = 260;    // buffer row pitch (floats): 256 terms + 4 (conflict-free fold reads)
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
  size_t act_lo, act_hi, act_m, buf, xin, nw, xsq, sum, total;
};

__host__ __device__ inline XLayout x_layout(int64_t cols, int in_mode) {
  XLayout L;
  L.nb = (int)(cols / 32);
  L.nseg = (L.nb + kSeg - 1) / kSeg;
  L.nbp = L.nseg * kSeg;
  size_t o = 0;
  L.act_lo = o; o += (size_t)L.nbp * 16;
  L.act_hi = o; o += (size_t)L.nbp * 16;
  L.act_m = o; o += (size_t)L.nbp * 16;
  L.buf = o;
  const size_t fold = (size_t)kNW * kBR * kBP * 4;
  const size_t row = ((size_t)L.nb * 32 * 4 + 15) / 16 * 16;
  size_t p = o;
  L.xin = p; if (in_mode != GEMV_IN_Q8) p += row;
  L.nw = p; if (in_mode == GEMV_IN_NORM) p += row;
  L.xsq = p; if (in_mode == GEMV_IN_NORM) p += row;
  L.sum = p; if (in_mode == GEMV_IN_NORM) p += (sizeof(exact::SumSmem<kNT>) + 15) / 16 * 16;  // also the squares' read slack
  L.total = o + (fold > p - o ? fold : p - o);
  return L;
}

// Slot of block b in the lane-interleaved activation layout.
__device__ __forceinline__ int act_slot(int b) {
  const int s = b / kSeg, i = b % kSeg;
  return s * kSeg + (i & 3) * 32 + (i >> 2);
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
    const int sl = act_slot(b);
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
      const int sl = act_slot(b);
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

// Quants and scales of one lane for one (row, segment) unit.
template <int QUANT>
struct XUnit {
  uint4 q[XCfg<QUANT>::NQ4];
  uint2 d;
};

template <int QUANT>
__device__ __forceinline__ void x_load(const DevMat &w, int64_t row, int seg, int nb, int lane, XUnit<QUANT> &u) {
  constexpr int NQ4 = XCfg<QUANT>::NQ4, BQ4 = NQ4 / 4;  // 16-byte pieces per block
  const int b0 = seg * kSeg + 4 * lane;
  const uint8_t *qp = w.qs + row * w.qs_stride + (int64_t)b0 * BQ4 * 16;
#pragma unroll
  for (int j = 0; j < NQ4; j++)
    u.q[j] = (b0 + j / BQ4 < nb) ? ldg_stream16(qp + 16 * j) : make_uint4(0u, 0u, 0u, 0u);
  u.d = b0 < nb ? ldg_stream8(w.d + row * w.d_stride + b0) : make_uint2(0u, 0u);
}

// The lane's eight chunk terms of a unit, in chunk order.
template <int QUANT>
__device__ __forceinline__ void x_terms(const XUnit<QUANT> &u, const int4 *alo, const int4 *ahi, const float4 *am,
                                        int seg, int lane, float (&t)[8]) {
  constexpr int BQ4 = XCfg<QUANT>::NQ4 / 4;
  const __half2 d01 = *reinterpret_cast<const __half2 *>(&u.d.x);
  const __half2 d23 = *reinterpret_cast<const __half2 *>(&u.d.y);
  const float ws[4] = {__low2float(d01), __high2float(d01), __low2float(d23), __high2float(d23)};
#pragma unroll
  for (int v = 0; v < 4; v++) {
    const int sl = seg * kSeg + v * 32 + lane;
    const int4 xl = alo[sl], xh = ahi[sl];
    const float4 m = am[sl];
    int d0, d1;
    if (QUANT == JAL_Q4_0) {
      const uint4 q = u.q[v];
      d0 = dp4a_us(q.x & 0x0F0F0F0Fu, xl.x, 0);
      d0 = dp4a_us(q.y & 0x0F0F0F0Fu, xl.y, d0);
      d0 = dp4a_us(q.z & 0x0F0F0F0Fu, xl.z, d0);
      d0 = dp4a_us(q.w & 0x0F0F0F0Fu, xl.w, d0);
      d1 = dp4a_us(q.x & 0xF0F0F0F0u, xh.x, 0);
      d1 = dp4a_us(q.y & 0xF0F0F0F0u, xh.y, d1);
      d1 = dp4a_us(q.z & 0xF0F0F0F0u, xh.z, d1);
      d1 = dp4a_us(q.w & 0xF0F0F0F0u, xh.w, d1);
      d0 -= 8 * __float_as_int(m.y);             // nibble n encodes n - 8
      d1 = (d1 >> 4) - 8 * __float_as_int(m.z);  // high nibbles were multiplied by 16 in place
    } else {
      const uint4 q0 = u.q[BQ4 * v], q1 = u.q[BQ4 * v + 1];
      d0 = dp4a_ss((int)q0.x, xl.x, 0);
      d0 = dp4a_ss((int)q0.y, xl.y, d0);
      d0 = dp4a_ss((int)q0.z, xl.z, d0);
      d0 = dp4a_ss((int)q0.w, xl.w, d0);
      d1 = dp4a_ss((int)q1.x, xh.x, 0);
      d1 = dp4a_ss((int)q1.y, xh.y, d1);
      d1 = dp4a_ss((int)q1.z, xh.z, d1);
      d1 = dp4a_ss((int)q1.w, xh.w, d1);
    }
    t[2 * v] = __fmul_rn(__fmul_rn(exact_i2f(d0), m.x), ws[v]);
    t[2 * v + 1] = __fmul_rn(__fmul_rn(exact_i2f(d1), m.x), ws[v]);
  }
}

template <int QUANT, int OUT>
__global__ void __launch_bounds__(kNT, 1) k_xgemv(const GemvArgs a) {
  constexpr int DEPTH = XCfg<QUANT>::DEPTH;
  constexpr int PAIR = OUT == GEMV_OUT_SWIGLU ? 2 : 1;  // physical rows per logical row
  constexpr int LPB = kBR / PAIR;                       // logical rows per batch
  extern __shared__ __align__(16) char smem[];
  const XLayout L = x_layout(a.w.cols, a.in_mode);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = a.rows / gridDim.x, rem = a.rows % gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * base + ((int64_t)blockIdx.x < rem ? blockIdx.x : rem);
  const int cnt = (int)(base + ((int64_t)blockIdx.x < rem ? 1 : 0));
  // This warp's logical rows: r0 + warp + 16 i, i < nl.
  const int nl = cnt > warp ? (cnt - 1 - warp) / kNW + 1 : 0;
  const int nbatch = (nl + LPB - 1) / LPB;
  const int nseg = L.nseg;
  float *buf = (float *)(smem + L.buf) + (size_t)warp * kBR * kBP;
  // Units of the warp in order: batch by batch; within a batch segment-major
  // over its physical rows (gate, up, gate, up, ... for SwiGLU).  A cursor
  // walks them without divisions.
  auto batch_rows = [&](int b) { return (nl - b * LPB < LPB ? nl - b * LPB : LPB) * PAIR; };
  struct Cursor {
    int b, sg, p, np;
  };
  auto advance = [&](Cursor &c) {
    if (++c.p == c.np) {
      c.p = 0;
      if (++c.sg == nseg) {
        c.sg = 0;
        c.np = batch_rows(++c.b);
      }
    }
  };
  const int total = nbatch ? (nbatch - 1) * kBR * nseg + batch_rows(nbatch - 1) * nseg : 0;
  auto prow = [&](int b, int p) -> int64_t {
    const int64_t lr = r0 + warp + (int64_t)(b * LPB + p / PAIR) * kNW;
    return (PAIR == 2 && (p & 1)) ? a.up_offset + lr : lr;
  };

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
  x_prologue(a, L, smem, (exact::SumSmem<kNT> *)(smem + L.sum));
  XUnit<QUANT> ring[DEPTH];
  Cursor cur = {0, 0, 0, nbatch ? batch_rows(0) : 0}, ahead = cur;
#pragma unroll
  for (int j = 0; j < DEPTH; j++)
    if (j < total) {
      x_load<QUANT>(a.w, prow(ahead.b, ahead.p), ahead.sg, L.nb, lane, ring[j]);
      advance(ahead);
    }
  const int4 *alo = (const int4 *)(smem + L.act_lo), *ahi = (const int4 *)(smem + L.act_hi);
  const float4 *am = (const float4 *)(smem + L.act_m);

  float acc = 0.0f;  // lane p < kBR: physical row p of the current batch
  for (int k0 = 0; k0 < total; k0 += DEPTH) {
#pragma unroll
    for (int j = 0; j < DEPTH; j++) {
      const int k = k0 + j;
      if (k < total) {
        const int b = cur.b, sg = cur.sg, p = cur.p, np = cur.np;
        advance(cur);
        float t[8];
        x_terms<QUANT>(ring[j], alo, ahi, am, sg, lane, t);
        if (k + DEPTH < total) {
          x_load<QUANT>(a.w, prow(ahead.b, ahead.p), ahead.sg, L.nb, lane, ring[j]);
          advance(ahead);
        }
        float *dst = buf + p * kBP + 8 * lane;
        *(float4 *)dst = make_float4(t[0], t[1], t[2], t[3]);
        *(float4 *)(dst + 4) = make_float4(t[4], t[5], t[6], t[7]);
        if (p == np - 1) {  // the batch's segment is complete: fold it
          __syncwarp();
          const int blk = L.nb - sg * kSeg < kSeg ? L.nb - sg * kSeg : kSeg;
          const int nt = 2 * blk;
          if (lane < np) {
            const float *src = buf + lane * kBP;
            int i = 0;
            for (; i + 4 <= nt; i += 4) {
              const float4 v = *(const float4 *)(src + i);
              acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v.x), v.y), v.z), v.w);
            }
            for (; i < nt; i++) acc = __fadd_rn(acc, src[i]);
          }
          __syncwarp();
          if (sg == nseg - 1) {  // rows of the batch are done
            const float other = __shfl_down_sync(0xffffffffu, acc, 1);
            if (lane < np && (PAIR == 1 || (lane & 1) == 0)) {
              const int64_t lr = r0 + warp + (int64_t)(b * LPB + lane / PAIR) * kNW;
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
            acc = 0.0f;
          }
        }
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
  cudaFuncSetAttribute(k_xgemv<QUANT, GEMV_OUT_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(k_xgemv<QUANT, GEMV_OUT_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(k_xgemv<QUANT, GEMV_OUT_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

}  // namespace

size_t xgemv_smem_bytes(int quant, int64_t cols, int in_mode) {
  (void)quant;
  return x_layout(cols, in_mode).total;
}

bool xgemv_supported(const GemvArgs &a) {
  if (a.m != 1 || (a.w.quant != JAL_Q4_0 && a.w.quant != JAL_Q8_0)) return false;
  if (a.w.cols % 32 != 0 || a.w.qs_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(a.w.qs) & 15) != 0) return false;
  if (a.w.d_stride % 4 != 0) return false;  // 8-byte scale loads
  if (a.out_mode != GEMV_OUT_STORE && a.out_mode != GEMV_OUT_ADD && a.out_mode != GEMV_OUT_SWIGLU) return false;
  if (a.peer_in || a.in_mode == GEMV_IN_PREQ) return false;
  return xgemv_smem_bytes(a.w.quant, a.w.cols, a.in_mode) <= 227 * 1024;
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
