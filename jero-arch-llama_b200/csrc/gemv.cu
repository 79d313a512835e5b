// Decode GEMV for the repacked Q4_0 / Q8_0 B200 layout (M <= 8 tokens).
//
// Semantics (repack_cache.rs:739-783): the integer block dot of the int8
// activation with the weight quants is exact (int32), and the row value is
// the f32 sum over blocks of f32(dot) * a_sc * w_sc.  The two 16-element
// chunks of a 32-block share both scales, so they are summed in int32 first
// (exactly the sum of the reference's two dot16 partials); the f32 order of
// the accumulation differs from the reference's sequential loop.
//
// Structure: one persistent CTA of WARPS warps per SM owns a contiguous
// range of rows (balanced to within one row); warp w of the CTA takes rows
// r0 + w, r0 + w + WARPS, ...  A row is streamed in chunks of 32*U blocks
// (lane l loads blocks l, l+32, ... with 16-byte loads that do not allocate
// in L1), DEPTH chunks in flight per warp.  Before griddepcontrol.wait the
// CTA asks the copy engine to prefetch the first pf_bytes of its rows into
// L2 (cp.async.bulk.prefetch.L2) and loads its first DEPTH chunks, so weight
// traffic starts while the previous kernel drains; afterwards each warp keeps
// its own L2 prefetch a fixed number of rows ahead.  The
// activation prologue (optionally RMSNorm, then the QuantizedActQ8
// quantizer) writes per-block int8 halves, the f32 scale and the 32-element
// int sum into shared memory.
//
// Per block and token the inner loop is 3 shared loads, 8 LOP3, 8 IDP4A,
// a shift and two integer adds, one half->float, one I2F, FMUL and FFMA:
// the high nibbles are masked in place (w & 0xF0F0F0F0) and the product,
// a multiple of 16, is shifted back; the -8 nibble offset is applied with
// the activation block sum.  The f16 scales were sanitized at repack time
// (Inf/NaN -> +-0.0625, the reference's f16_to_f32_finite), so a plain
// conversion is exact here.
#include <cuda_fp16.h>

#include <cstdlib>

#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "gemv_dev.cuh"
#include "jal.h"

namespace jal {

namespace {

using namespace gdev;

template <int QUANT>
struct ChunkRegs;
template <>
struct ChunkRegs<JAL_Q4_0> {
  static constexpr int U = 4;  // blocks per lane per chunk (64 B / lane)
  uint4 w[U];
  unsigned short d[U];
};
template <>
struct ChunkRegs<JAL_Q8_0> {
  static constexpr int U = 2;  // blocks per lane per chunk (64 B / lane)
  uint4 w[2 * U];
  unsigned short d[U];
};

template <int QUANT>
__device__ __forceinline__ void load_chunk(const DevMat &w, int64_t row, int part, int nb, int lane,
                                           ChunkRegs<QUANT> &r) {
  constexpr int U = ChunkRegs<QUANT>::U;
  const uint8_t *qrow = w.qs + row * w.qs_stride;
  const uint16_t *drow = w.d + row * w.d_stride;
#pragma unroll
  for (int v = 0; v < U; v++) {
    int b = part * 32 * U + v * 32 + lane;
    if (b < nb) {
      if (QUANT == JAL_Q4_0) {
        r.w[v] = ldg_stream16(qrow + (int64_t)b * 16);
      } else {
        r.w[2 * v] = ldg_stream16(qrow + (int64_t)b * 32);
        r.w[2 * v + 1] = ldg_stream16(qrow + (int64_t)b * 32 + 16);
      }
      r.d[v] = ldg_stream2(drow + b);
    }
  }
}

// acc + f32(int dot of block b) * (a_sc * w_sc) for one token.
template <int QUANT>
__device__ __forceinline__ float block_fma(const ChunkRegs<QUANT> &r, int v, const char *base, int nbp, int b,
                                           float ws, float acc) {
  const int4 alo = ((const int4 *)base)[b];
  const int4 ahi = ((const int4 *)(base + nbp * 16))[b];
  const float2 ss = ((const float2 *)(base + nbp * 32))[b];
  int dot;
  if (QUANT == JAL_Q4_0) {
    const uint4 w = r.w[v];
    int d0 = dp4a_us(w.x & 0x0F0F0F0Fu, alo.x, 0);
    int d1 = dp4a_us(w.x & 0xF0F0F0F0u, ahi.x, 0);
    d0 = dp4a_us(w.y & 0x0F0F0F0Fu, alo.y, d0);
    d1 = dp4a_us(w.y & 0xF0F0F0F0u, ahi.y, d1);
    d0 = dp4a_us(w.z & 0x0F0F0F0Fu, alo.z, d0);
    d1 = dp4a_us(w.z & 0xF0F0F0F0u, ahi.z, d1);
    d0 = dp4a_us(w.w & 0x0F0F0F0Fu, alo.w, d0);
    d1 = dp4a_us(w.w & 0xF0F0F0F0u, ahi.w, d1);
    dot = d0 + (d1 >> 4) - 8 * __float_as_int(ss.y);  // nibble n encodes n - 8
  } else {
    const uint4 w0 = r.w[2 * v], w1 = r.w[2 * v + 1];
    int d0 = dp4a_ss((int)w0.x, alo.x, 0);
    int d1 = dp4a_ss((int)w1.x, ahi.x, 0);
    d0 = dp4a_ss((int)w0.y, alo.y, d0);
    d1 = dp4a_ss((int)w1.y, ahi.y, d1);
    d0 = dp4a_ss((int)w0.z, alo.z, d0);
    d1 = dp4a_ss((int)w1.z, ahi.z, d1);
    d0 = dp4a_ss((int)w0.w, alo.w, d0);
    d1 = dp4a_ss((int)w1.w, ahi.w, d1);
    dot = d0 + d1;
  }
  return fmaf(__int2float_rn(dot), ss.x * ws, acc);
}

// Position in a warp's chunk sequence: logical row index i (row gw + i*WARPS),
// unit (0 = the row itself or the gate half, 1 = the up half) and part (the
// chunk of 32*U blocks within the row).  Advanced by increments only.
struct Cursor {
  int i = 0, unit = 0, part = 0;
  __device__ __forceinline__ void next(int parts, int units) {
    if (++part == parts) {
      part = 0;
      if (++unit == units) { unit = 0; ++i; }
    }
  }
};

template <int QUANT, int M, int OUT, int WARPS, int DEPTH>
__global__ void __launch_bounds__(WARPS * 32, 16 / WARPS) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) char smem[];
  __shared__ float red[33];
  constexpr int U = ChunkRegs<QUANT>::U;
  constexpr int UNITS = OUT == GEMV_OUT_SWIGLU ? 2 : 1;
  const int nb = (int)(a.w.cols / 32), nbp = (nb + 31) & ~31;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int parts = (nb + 32 * U - 1) / (32 * U);
  // Contiguous, balanced row range [r0, r0 + cnt) of this CTA.
  const int64_t base = a.rows / gridDim.x, rem = a.rows % gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * base + ((int64_t)blockIdx.x < rem ? blockIdx.x : rem);
  const int64_t cnt = base + ((int64_t)blockIdx.x < rem ? 1 : 0);
  const int my_rows = cnt > warp ? (int)((cnt - 1 - warp) / WARPS + 1) : 0;
  const int64_t gw = r0 + warp;  // row of logical index i is gw + i * WARPS
  const int64_t qrow = a.w.qs_stride, drow = a.w.d_stride * 2;
  // L2 prefetch distance in rows per warp, from the per-CTA prefetch budget.
  int pd = (int)(a.pf_bytes / (UNITS * (qrow + drow) * WARPS));
  if (pd < 1) pd = 1;
  if (threadIdx.x == 0 && a.pf_bytes > 0) {
    const int64_t pr = cnt < (int64_t)pd * WARPS ? cnt : (int64_t)pd * WARPS;
#pragma unroll
    for (int u = 0; u < UNITS; u++) {
      const int64_t rr = r0 + (u ? a.up_offset : 0);
      l2_prefetch_bulk(a.w.qs + rr * qrow, (uint64_t)(pr * qrow));
      l2_prefetch_bulk((const char *)a.w.d + rr * drow, (uint64_t)(pr * drow));
    }
  }

  Cursor ld, cp;  // next chunk to load / to compute
  ChunkRegs<QUANT> buf[DEPTH];
#pragma unroll
  for (int k = 0; k < DEPTH; k++) {
    if (ld.i < my_rows) {
      load_chunk<QUANT>(a.w, gw + ld.i * WARPS + (ld.unit ? a.up_offset : 0), ld.part, nb, lane, buf[k]);
      ld.next(parts, UNITS);
    }
  }
  gemv_prologue_pre<M, WARPS>(a, smem, nb, nbp);
  pdl_wait();
  pdl_trigger();
  gemv_prologue<M, WARPS>(a, smem, nb, nbp, red);

  float acc0[M], acc1[M];
#pragma unroll
  for (int t = 0; t < M; t++) acc0[t] = acc1[t] = 0.0f;

  while (cp.i < my_rows) {
#pragma unroll
    for (int k = 0; k < DEPTH; k++) {
      if (cp.i < my_rows) {
#pragma unroll
        for (int v = 0; v < U; v++) {
          const int b = cp.part * 32 * U + v * 32 + lane;
          if (b < nb) {
            const float ws = __half2float(__ushort_as_half(buf[k].d[v]));
#pragma unroll
            for (int t = 0; t < M; t++) {
              if (cp.unit == 0) acc0[t] = block_fma<QUANT>(buf[k], v, smem + t * act_bytes(nbp), nbp, b, ws, acc0[t]);
              else acc1[t] = block_fma<QUANT>(buf[k], v, smem + t * act_bytes(nbp), nbp, b, ws, acc1[t]);
            }
          }
        }
        if (ld.i < my_rows) {
          load_chunk<QUANT>(a.w, gw + ld.i * WARPS + (ld.unit ? a.up_offset : 0), ld.part, nb, lane, buf[k]);
          ld.next(parts, UNITS);
        }
        if (cp.part == 0 && cp.unit == 0 && lane == 0 && a.pf_bytes > 0 && cp.i + pd < my_rows) {
          const int64_t pr = gw + (int64_t)(cp.i + pd) * WARPS;
#pragma unroll
          for (int u = 0; u < UNITS; u++) {
            const int64_t rr = pr + (u ? a.up_offset : 0);
            l2_prefetch_bulk(a.w.qs + rr * qrow, (uint64_t)qrow);
            l2_prefetch_bulk((const char *)a.w.d + rr * drow, (uint64_t)drow);
          }
        }
        if (cp.part == parts - 1 && cp.unit == UNITS - 1) {
          const int64_t lr = gw + (int64_t)cp.i * WARPS;
          float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
          for (int t = 0; t < M; t++) {
            const float r0 = warp_sum(acc0[t]);
            const float r1 = UNITS == 2 ? warp_sum(acc1[t]) : 0.0f;
            if (lane == t) { s0 = r0; s1 = r1; }
            acc0[t] = acc1[t] = 0.0f;
          }
          if (lane < a.m) {
            float *yp = a.y + lane * a.y_stride + lr;
            if (OUT == GEMV_OUT_STORE) {
              *yp = a.bias ? s0 + a.bias[lr] : s0;
            } else if (OUT == GEMV_OUT_ADD) {
              const float p = a.bias ? s0 + a.bias[lr] : s0;
              *yp = *yp + p;
            } else {
              *yp = swiglu_one(s0, s1);
            }
          }
        }
        cp.next(parts, UNITS);
      }
    }
  }
}

// ---- segmented fast path (M = 1) ------------------------------------------
//
// A row is split into nseg segments of 128 blocks (nseg = 1 for 4096
// columns, 4 for the 14336-column down projection, whose last segment holds
// 64 blocks).  Warp w owns segment w % nseg of rows r0 + w / nseg,
// r0 + w / nseg + WARPS / nseg, ...  Within a segment lane l owns blocks
// 4l .. 4l+3: its quants are one contiguous 64-byte (Q4_0) / 128-byte (Q8_0)
// piece read with 32-byte loads, its four scales one 8-byte load, and its
// four blocks of the quantized activation stay in registers for the whole
// kernel.  A segment costs the loads, 4 block dots and one warp reduction;
// DEPTH segments are in flight per warp.  With nseg > 1 the per-segment sums
// of a row are added in segment order at the end of the kernel.
// OUTX = output mode | kPeerIn when the input is the tensor-parallel exchange.
constexpr int kPeerIn = 4;
template <int QUANT, int OUTX, int WARPS, int DEPTH>
__global__ void __launch_bounds__(WARPS * 32, 16 / WARPS) k_gemv_w4(const GemvArgs a) {
  constexpr int OUT = OUTX & 3;
  constexpr bool PEER_IN = (OUTX & kPeerIn) != 0;
  extern __shared__ __align__(16) char smem[];
  __shared__ float red[33];
  constexpr int UNITS = OUT == GEMV_OUT_SWIGLU ? 2 : 1;
  const int nb = (int)(a.w.cols / 32), nseg = seg_count(a.w.cols), nbp = nseg * kSegBlocks;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int seg = warp % nseg, phase = warp / nseg, nph = WARPS / nseg;
  const int64_t base = a.rows / gridDim.x, rem = a.rows % gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * base + ((int64_t)blockIdx.x < rem ? blockIdx.x : rem);
  const int64_t cnt = base + ((int64_t)blockIdx.x < rem ? 1 : 0);
  const int my_rows = cnt > phase ? (int)((cnt - 1 - phase) / nph + 1) : 0;
  const int64_t gw = r0 + phase;
  const int total = my_rows * UNITS;  // unit k: row index k / UNITS, half k % UNITS
  float *part = (float *)(smem + w4_act_region(a.in_mode, nb, nseg));  // [cnt][nseg]
  auto unit_row = [&](int k) -> int64_t {
    return gw + (int64_t)(k / UNITS) * nph + ((UNITS == 2 && (k & 1)) ? a.up_offset : 0);
  };

  // Before griddepcontrol.wait: either the copy engine prefetches the
  // CTA's first pf_bytes into L2 (no load slots held, so the activation
  // loads after the wait are not queued behind weight traffic), or, with
  // pf_bytes == 0, the warps load their first DEPTH segments into registers.
  W4Row<QUANT> buf[DEPTH];
  const bool l2_first = a.pf_bytes > 0;
  if (l2_first) {
    if (threadIdx.x == 0 && cnt > 0) {
      int64_t pr = a.pf_bytes / (UNITS * a.w.qs_stride);
      if (pr < 1) pr = 1;
      if (pr > cnt) pr = cnt;
#pragma unroll
      for (int u = 0; u < UNITS; u++)
        l2_prefetch_bulk(a.w.qs + (r0 + (u ? a.up_offset : 0)) * a.w.qs_stride, (uint64_t)(pr * a.w.qs_stride));
    }
  } else {
#pragma unroll
    for (int j = 0; j < DEPTH; j++)
      if (j < total) w4_load<QUANT>(a.w, unit_row(j), seg, nb, lane, buf[j]);
  }
  pdl_wait();
  pdl_trigger();
  // GEMV_OUT_PEER: flag of this step's words (the epoch advanced before the wait)
  const unsigned long long xflag =
      OUT == GEMV_OUT_PEER ? (unsigned long long)(ld_relaxed_gpu_u32(a.peer_epoch) * 256u + (uint32_t)a.peer_phase + 1u) << 32
                           : 0ull;
  if (l2_first) {  // weight loads first: they overlap the prologue's round trip
#pragma unroll
    for (int j = 0; j < DEPTH; j++)
      if (j < total) w4_load<QUANT>(a.w, unit_row(j), seg, nb, lane, buf[j]);
  }
  gemv_prologue_m1<WARPS, PEER_IN>(a, smem, nb, nbp, red);
  W4Act x;
#pragma unroll
  for (int v = 0; v < 4; v++) {
    const int b = seg * kSegBlocks + 4 * lane + v;  // < nbp; padding blocks are zero
    x.lo[v] = ((const int4 *)smem)[b];
    x.hi[v] = ((const int4 *)(smem + nbp * 16))[b];
    const float2 ss = ((const float2 *)(smem + nbp * 32))[b];
    x.sc[v] = ss.x;
    x.sum[v] = __float_as_int(ss.y);
  }

  float gate = 0.0f;
  for (int k0 = 0; k0 < total; k0 += DEPTH) {
#pragma unroll
    for (int j = 0; j < DEPTH; j++) {
      const int k = k0 + j;
      if (k < total) {
        float s = w4_dot<QUANT>(buf[j], x);
        if (k + DEPTH < total) w4_load<QUANT>(a.w, unit_row(k + DEPTH), seg, nb, lane, buf[j]);
        s = warp_sum(s);
        const int li = phase + (k / UNITS) * nph;  // row within the CTA
        if (UNITS == 2 && (k & 1) == 0) {
          gate = s;
        } else if (nseg > 1) {
          if (lane == 0) part[li * nseg + seg] = s;
        } else if (lane == 0) {
          const int64_t lr = r0 + li;
          float *yp = a.y + lr;
          if (OUT == GEMV_OUT_PEER) {
            const unsigned long long word = xflag | __float_as_uint(a.bias ? s + a.bias[lr] : s);
            for (int r = 0; r < a.peer_world; r++) st_relaxed_sys_u64(a.peer_out[r] + lr, word);
          } else if (OUT == GEMV_OUT_STORE) *yp = a.bias ? s + a.bias[lr] : s;
          else if (OUT == GEMV_OUT_ADD) *yp = *yp + (a.bias ? s + a.bias[lr] : s);
          else *yp = swiglu_one(gate, s);
        }
      }
    }
  }
  if (nseg > 1 && OUT != GEMV_OUT_SWIGLU) {
    __syncthreads();
    for (int li = threadIdx.x; li < cnt; li += WARPS * 32) {
      float s = 0.0f;
      for (int q = 0; q < nseg; q++) s += part[li * nseg + q];
      const int64_t lr = r0 + li;
      float *yp = a.y + lr;
      if (OUT == GEMV_OUT_PEER) {
        const unsigned long long word = xflag | __float_as_uint(a.bias ? s + a.bias[lr] : s);
        for (int r = 0; r < a.peer_world; r++) st_relaxed_sys_u64(a.peer_out[r] + lr, word);
      } else if (OUT == GEMV_OUT_STORE) *yp = a.bias ? s + a.bias[lr] : s;
      else *yp = *yp + (a.bias ? s + a.bias[lr] : s);
    }
  }
}

int g_w4_warps = -1;
int w4_warps() {
  if (g_w4_warps < 0) {
    const char *e = getenv("JAL_W4_WARPS");
    g_w4_warps = (e && atoi(e) == 8) ? 8 : 16;
  }
  return g_w4_warps;
}

int64_t g_w4_pf = -1;
int64_t w4_prefetch_bytes() {
  if (g_w4_pf < 0) {
    // Default 0: register loads before the wait.  Llama-3-8B Q4_0 decode
    // at position 2048: 1.81 ms per step, against 1.88 ms with a 64 KB L2
    // prefetch per CTA instead.
    const char *e = getenv("JAL_W4_PF_KB");
    g_w4_pf = e ? (int64_t)atoll(e) * 1024 : 0;
  }
  return g_w4_pf;
}

template <int QUANT, int OUT, int WARPS>
void launch_w4_w(GemvArgs a, int grid, cudaStream_t s) {
  constexpr int DEPTH = QUANT == JAL_Q4_0 ? 3 : 2;
  a.pf_bytes = w4_prefetch_bytes();
  const int nb = (int)(a.w.cols / 32), nseg = seg_count(a.w.cols);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = w4_smem(a.in_mode, nb, nseg, (a.rows + grid - 1) / grid);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_gemv_w4<QUANT, OUT, WARPS, DEPTH>, a);
}

template <int QUANT, int OUT>
void launch_w4_t(const GemvArgs &a, int grid, cudaStream_t s) {
  if (w4_warps() == 8) launch_w4_w<QUANT, OUT, 8>(a, grid, s);
  else launch_w4_w<QUANT, OUT, 16>(a, grid, s);
}

template <int QUANT, int OUT>
void set_w4_attrs() {
  constexpr int DEPTH = QUANT == JAL_Q4_0 ? 3 : 2;
  const void *fns[2] = {(const void *)k_gemv_w4<QUANT, OUT, 16, DEPTH>, (const void *)k_gemv_w4<QUANT, OUT, 8, DEPTH>};
  for (const void *f : fns) cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
}

// Shapes the segmented path takes: M = 1, 1, 2 or 4 segments (cols up to
// 16384, a multiple of 128), SwiGLU only with one segment, and per-CTA
// partials that fit in shared memory.
bool w4_fits(const GemvArgs &a, int grid) {
  const int64_t nb = a.w.cols / 32;
  if (a.m != 1 || nb % 4 != 0) return false;
  // 32-byte loads: every row must start 32-byte aligned.
  if (a.w.qs_stride % 32 != 0 || (reinterpret_cast<uintptr_t>(a.w.qs) & 31) != 0) return false;
  const int nseg = seg_count(a.w.cols);
  if (nseg != 1 && nseg != 2 && nseg != 4) return false;
  if (nseg > 1 && a.out_mode == GEMV_OUT_SWIGLU) return false;
  if (nseg > w4_warps()) return false;
  return w4_smem(a.in_mode, (int)nb, nseg, (a.rows + grid - 1) / grid) <= (size_t)kGemvMaxSmem;
}

int g_use_w4 = -1;
bool use_w4() {
  if (g_use_w4 < 0) {
    const char *e = getenv("JAL_GEMV_KERNEL");
    g_use_w4 = (e && e[0] == 'c') ? 0 : 1;
  }
  return g_use_w4 != 0;
}

// Launch shapes: (warps per CTA, chunks in flight per warp).  The default
// is one 16-warp CTA per SM; JAL_GEMV_SHAPE=B selects 8-warp CTAs (<= 128
// registers) that leave room on each SM for a CTA of the next kernel, which
// measured slower on B200 for the Llama-3-8B decode shapes.
constexpr int kWarpsA = 16, kDepthA = 3;
constexpr int kWarpsB = 8, kDepthB = 3;
constexpr int64_t kDefaultPrefetchBytes = 96 * 1024;

int g_shape = -1;  // 0 = A, 1 = B
int g_sm_count = 0;
int64_t g_pf_bytes = -1;

int shape() {
  if (g_shape < 0) {
    const char *e = getenv("JAL_GEMV_SHAPE");
    g_shape = (e && *e == 'B') ? 1 : 0;
  }
  return g_shape;
}

int64_t prefetch_bytes() {
  if (g_pf_bytes < 0) {
    const char *e = getenv("JAL_GEMV_PF_KB");
    g_pf_bytes = e ? (int64_t)atoll(e) * 1024 : kDefaultPrefetchBytes;
  }
  return g_pf_bytes;
}

template <int QUANT, int M, int OUT, int WARPS, int DEPTH>
void launch_t(const GemvArgs &a, int grid, cudaStream_t s) {
  const int nb = (int)(a.w.cols / 32);
  size_t smem = smem_bytes(a.in_mode, M, nb);
  auto kern = k_gemv<QUANT, M, OUT, WARPS, DEPTH>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, a);
}

template <int QUANT, int OUT, int WARPS, int DEPTH>
void launch_m(const GemvArgs &a, int grid, cudaStream_t s) {
  switch (a.m) {
    case 1: launch_t<QUANT, 1, OUT, WARPS, DEPTH>(a, grid, s); break;
    case 2: launch_t<QUANT, 2, OUT, WARPS, DEPTH>(a, grid, s); break;
    case 3: case 4: launch_t<QUANT, 4, OUT, WARPS, DEPTH>(a, grid, s); break;
    default: launch_t<QUANT, 8, OUT, WARPS, DEPTH>(a, grid, s); break;
  }
}

template <int QUANT, int OUT>
void launch_q(const GemvArgs &a, int grid, cudaStream_t s) {
  if (shape() == 1) launch_m<QUANT, OUT, kWarpsB, kDepthB>(a, grid, s);
  else launch_m<QUANT, OUT, kWarpsA, kDepthA>(a, grid, s);
}

template <int QUANT, int OUT, int WARPS, int DEPTH>
void set_attrs() {
  const int lim = kGemvMaxSmem;
  const void *fns[4] = {(const void *)k_gemv<QUANT, 1, OUT, WARPS, DEPTH>, (const void *)k_gemv<QUANT, 2, OUT, WARPS, DEPTH>,
                        (const void *)k_gemv<QUANT, 4, OUT, WARPS, DEPTH>, (const void *)k_gemv<QUANT, 8, OUT, WARPS, DEPTH>};
  for (const void *f : fns) {
    cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  }
}

template <int WARPS, int DEPTH>
void set_attrs_all() {
  set_attrs<JAL_Q4_0, GEMV_OUT_STORE, WARPS, DEPTH>();
  set_attrs<JAL_Q4_0, GEMV_OUT_ADD, WARPS, DEPTH>();
  set_attrs<JAL_Q4_0, GEMV_OUT_SWIGLU, WARPS, DEPTH>();
  set_attrs<JAL_Q8_0, GEMV_OUT_STORE, WARPS, DEPTH>();
  set_attrs<JAL_Q8_0, GEMV_OUT_ADD, WARPS, DEPTH>();
  set_attrs<JAL_Q8_0, GEMV_OUT_SWIGLU, WARPS, DEPTH>();
}

}  // namespace

bool w4_matrix_ok(const DevMat &w) {
  if (w.quant != JAL_Q4_0 && w.quant != JAL_Q8_0) return false;
  const int64_t nb = w.cols / 32;
  if (w.cols % 32 || nb % 4 != 0) return false;
  if (w.qs_stride % 32 != 0 || (reinterpret_cast<uintptr_t>(w.qs) & 31) != 0) return false;
  const int nseg = seg_count(w.cols);
  return nseg >= 1 && nseg <= 16;
}

void gemv_init() {
  static bool done = false;
  if (done) return;
  set_attrs_all<kWarpsA, kDepthA>();
  set_attrs_all<kWarpsB, kDepthB>();
  set_w4_attrs<JAL_Q4_0, GEMV_OUT_STORE>();
  set_w4_attrs<JAL_Q4_0, GEMV_OUT_ADD>();
  set_w4_attrs<JAL_Q4_0, GEMV_OUT_SWIGLU>();
  set_w4_attrs<JAL_Q8_0, GEMV_OUT_STORE>();
  set_w4_attrs<JAL_Q8_0, GEMV_OUT_ADD>();
  set_w4_attrs<JAL_Q8_0, GEMV_OUT_SWIGLU>();
  set_w4_attrs<JAL_Q4_0, GEMV_OUT_PEER>();
  set_w4_attrs<JAL_Q8_0, GEMV_OUT_PEER>();
  set_w4_attrs<JAL_Q4_0, GEMV_OUT_STORE | kPeerIn>();
  set_w4_attrs<JAL_Q4_0, GEMV_OUT_SWIGLU | kPeerIn>();
  set_w4_attrs<JAL_Q8_0, GEMV_OUT_STORE | kPeerIn>();
  set_w4_attrs<JAL_Q8_0, GEMV_OUT_SWIGLU | kPeerIn>();
  done = true;
}

size_t gemv_smem_bytes(int in_mode, int m, int64_t cols) {
  int M = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
  return smem_bytes(in_mode, M, (int)(cols / 32));
}

int gemv_default_grid(const GemvArgs &a) {
  if (!g_sm_count) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  const int warps = shape() == 1 ? kWarpsB : kWarpsA;
  int64_t need = (a.rows + warps - 1) / warps;
  int64_t cap = (int64_t)g_sm_count;
  return (int)(need < cap ? need : cap);
}

bool gemv_peer_supported(const GemvArgs &a) {
  if (a.m != 1 || a.peer_world < 1 || a.peer_world > kPeerMax) return false;
  if (a.w.quant != JAL_Q4_0 && a.w.quant != JAL_Q8_0) return false;
  // the exchange lives in the one-round-trip RMSNorm prologue (rows up to
  // 1024 jobs of 8 elements) and in the segmented kernel's epilogue
  if (!a.peer_epoch || a.peer_phase < 0 || a.peer_phase > 254) return false;
  if (a.peer_in && (a.in_mode != GEMV_IN_NORM || a.w.cols > 8192 || a.x_stride % 2 != 0)) return false;
  if (a.out_mode == GEMV_OUT_PEER)
    for (int r = 0; r < a.peer_world; r++)
      if (!a.peer_out[r]) return false;
  int grid = a.grid;
  if (grid <= 0) {
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    grid = (int)(a.rows < sms ? a.rows : sms);
  }
  return w4_fits(a, grid);
}

void launch_gemv(const GemvArgs &a0, cudaStream_t s) {
  if (a0.rows <= 0) return;
  if (dense_quant(a0.w.quant)) {
    launch_gemv_dense(a0, s);
    return;
  }
  gemv_init();
  GemvArgs a = a0;
  // Token counts between template sizes run the next larger instantiation;
  // token slots t >= m quantize to zero and are never written.
  if (a.pf_bytes < 0) a.pf_bytes = prefetch_bytes();
  int w4_grid = a.grid;
  if (w4_grid <= 0) {
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    w4_grid = (int)(a.rows < sms ? a.rows : sms);
  }
  const bool peer = a.peer_in != nullptr || a.out_mode == GEMV_OUT_PEER;
  if (peer && !gemv_peer_supported(a))
    fail(JAL_ERR_CAPABILITY_MISMATCH, "tensor-parallel exchange: GEMV shape not on the segmented kernel");
  if ((use_w4() || peer) && w4_fits(a, w4_grid)) {
    const int grid = w4_grid;
    if (a.peer_in) {  // exchange input: RMSNorm rows into STORE (QKV, LM head) or SWIGLU (gate / up)
      if (a.out_mode != GEMV_OUT_STORE && a.out_mode != GEMV_OUT_SWIGLU)
        fail(JAL_ERR_CAPABILITY_MISMATCH, "tensor-parallel exchange input with output mode %d", a.out_mode);
      const bool sw = a.out_mode == GEMV_OUT_SWIGLU;
      if (a.w.quant == JAL_Q4_0) {
        if (sw) launch_w4_t<JAL_Q4_0, GEMV_OUT_SWIGLU | kPeerIn>(a, grid, s);
        else launch_w4_t<JAL_Q4_0, GEMV_OUT_STORE | kPeerIn>(a, grid, s);
      } else {
        if (sw) launch_w4_t<JAL_Q8_0, GEMV_OUT_SWIGLU | kPeerIn>(a, grid, s);
        else launch_w4_t<JAL_Q8_0, GEMV_OUT_STORE | kPeerIn>(a, grid, s);
      }
    } else if (a.w.quant == JAL_Q4_0) {
      if (a.out_mode == GEMV_OUT_STORE) launch_w4_t<JAL_Q4_0, GEMV_OUT_STORE>(a, grid, s);
      else if (a.out_mode == GEMV_OUT_ADD) launch_w4_t<JAL_Q4_0, GEMV_OUT_ADD>(a, grid, s);
      else if (a.out_mode == GEMV_OUT_PEER) launch_w4_t<JAL_Q4_0, GEMV_OUT_PEER>(a, grid, s);
      else launch_w4_t<JAL_Q4_0, GEMV_OUT_SWIGLU>(a, grid, s);
    } else {
      if (a.out_mode == GEMV_OUT_STORE) launch_w4_t<JAL_Q8_0, GEMV_OUT_STORE>(a, grid, s);
      else if (a.out_mode == GEMV_OUT_ADD) launch_w4_t<JAL_Q8_0, GEMV_OUT_ADD>(a, grid, s);
      else if (a.out_mode == GEMV_OUT_PEER) launch_w4_t<JAL_Q8_0, GEMV_OUT_PEER>(a, grid, s);
      else launch_w4_t<JAL_Q8_0, GEMV_OUT_SWIGLU>(a, grid, s);
    }
    return;
  }
  int grid = a.grid > 0 ? a.grid : gemv_default_grid(a);
  if (a.w.quant == JAL_Q4_0) {
    if (a.out_mode == GEMV_OUT_STORE) launch_q<JAL_Q4_0, GEMV_OUT_STORE>(a, grid, s);
    else if (a.out_mode == GEMV_OUT_ADD) launch_q<JAL_Q4_0, GEMV_OUT_ADD>(a, grid, s);
    else launch_q<JAL_Q4_0, GEMV_OUT_SWIGLU>(a, grid, s);
  } else {
    if (a.out_mode == GEMV_OUT_STORE) launch_q<JAL_Q8_0, GEMV_OUT_STORE>(a, grid, s);
    else if (a.out_mode == GEMV_OUT_ADD) launch_q<JAL_Q8_0, GEMV_OUT_ADD>(a, grid, s);
    else launch_q<JAL_Q8_0, GEMV_OUT_SWIGLU>(a, grid, s);
  }
}

}  // namespace jal
