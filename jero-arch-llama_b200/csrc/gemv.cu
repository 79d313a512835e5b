// Decode GEMV for the repacked Q4_0 / Q8_0 B200 layout (M <= 8 tokens).
//
// Semantics (repack_cache.rs:739-783): for every output row r and 16-element
// chunk ch, dot16 = sum(a_q8 * w_q) in int32 (exact), and the row value is
// the f32 sum over chunks of (f32(dot16) * a_sc[ch/2]) * w_sc[ch/2].  Each
// term is computed with correctly rounded multiplies, so it is bit-identical
// to the reference's term; only the order of the f32 sum differs (lanes own
// blocks, then a warp butterfly).
//
// Structure: persistent CTAs of 8 warps; warp w of CTA c owns logical rows
// gw, gw + nw, ... (gw = c*8 + w, nw = 8*grid).  A row is streamed in chunks
// of 32*U blocks (lane l loads blocks l, l+32, ... with 16-byte loads that do
// not allocate in L1), double-buffered in registers.  The first chunk is
// loaded before griddepcontrol.wait, so weight traffic starts while the
// previous kernel drains.  The activation prologue (optionally RMSNorm, then
// the QuantizedActQ8 quantizer) writes per-block int8 halves, the f32 scale
// and the two 16-element sums into shared memory.
#include <cuda_fp16.h>

#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Shared-memory activation layout for token t (nbp = nb rounded up to 4):
//   [lo: nbp x 16 B][hi: nbp x 16 B][scale: nbp x f32][sums: nbp x int2]
__host__ __device__ inline size_t act_bytes(int nbp) { return (size_t)nbp * 44; }

__device__ float block_reduce_sum(float v, float *red) {
  v = warp_sum(v);
  int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < kWarps ? red[l] : 0.0f;
    t = warp_sum(t);
    if (l == 0) red[32] = t;
  }
  __syncthreads();
  float r = red[32];
  __syncthreads();
  return r;
}

template <int M>
__device__ void gemv_prologue(const GemvArgs &a, char *smem, int nb, int nbp, float *red) {
  float inv_norm[M];
#pragma unroll
  for (int t = 0; t < M; t++) inv_norm[t] = 1.0f;
  const int K = nb * 32;
  if (a.in_mode == GEMV_IN_NORM) {
#pragma unroll
    for (int t = 0; t < M; t++) {
      if (t >= a.m) break;
      const float *x = a.x + t * a.x_stride;
      float ss = 0.0f;
      for (int i = threadIdx.x * 4; i < K; i += kThreads * 4) {
        float4 v = *(const float4 *)(x + i);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
      }
      ss = block_reduce_sum(ss, red);
      inv_norm[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int wb = warp; wb < M * nb; wb += kWarps) {
    const int t = wb / nb, b = wb % nb;
    char *base = smem + t * act_bytes(nbp);
    int8_t q;
    float scale;
    if (t >= a.m) {
      q = 0;
      scale = 0.0f;
    } else if (a.in_mode == GEMV_IN_Q8) {
      q = a.xq[t * a.xq_stride + b * 32 + lane];
      scale = a.xs[t * (a.xq_stride / 32) + b];
    } else {
      float v = a.x[t * a.x_stride + b * 32 + lane];
      if (a.in_mode == GEMV_IN_NORM) {
        float invn = inv_norm[0];
#pragma unroll
        for (int tt = 1; tt < M; tt++)
          if (tt == t) invn = inv_norm[tt];
        v = __fmul_rn(__fmul_rn(v, invn), a.norm_w[b * 32 + lane]);
      }
      if (!isfinite(v)) v = 0.0f;
      float amax = warp_max(fabsf(v));
      scale = act_scale_from_amax(amax);
      q = act_quant_one(v, act_inv_from_scale(scale));
    }
    int8_t *lo = (int8_t *)base + b * 16;
    int8_t *hi = (int8_t *)(base + nbp * 16) + b * 16;
    if (lane < 16) lo[lane] = q;
    else hi[lane - 16] = q;
    int s = q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      ((float *)(base + nbp * 32))[b] = scale;
      ((int *)(base + nbp * 36))[2 * b] = s;
    }
    if (lane == 16) ((int *)(base + nbp * 36))[2 * b + 1] = s;
  }
  __syncthreads();
}

template <int QUANT>
struct ChunkRegs;
template <>
struct ChunkRegs<JAL_Q4_0> {
  static constexpr int U = 4;  // blocks per lane per chunk (64 B / lane)
  uint4 w[U];
  uint16_t d[U];
};
template <>
struct ChunkRegs<JAL_Q8_0> {
  static constexpr int U = 2;  // blocks per lane per chunk (64 B / lane)
  uint4 w[2 * U];
  uint16_t d[U];
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

// Terms of one block for one token: (f32(dot16) * a_sc) * w_sc per chunk.
template <int QUANT>
__device__ __forceinline__ float block_terms(const ChunkRegs<QUANT> &r, int v, const char *base, int nbp, int b,
                                             float ws) {
  const int4 alo = ((const int4 *)base)[b];
  const int4 ahi = ((const int4 *)(base + nbp * 16))[b];
  const float as = ((const float *)(base + nbp * 32))[b];
  int dlo, dhi;
  if (QUANT == JAL_Q4_0) {
    const int2 sm = ((const int2 *)(base + nbp * 36))[b];
    const uint4 w = r.w[v];
    dlo = dp4a_us(w.x & 0x0F0F0F0Fu, alo.x, 0);
    dlo = dp4a_us(w.y & 0x0F0F0F0Fu, alo.y, dlo);
    dlo = dp4a_us(w.z & 0x0F0F0F0Fu, alo.z, dlo);
    dlo = dp4a_us(w.w & 0x0F0F0F0Fu, alo.w, dlo);
    dhi = dp4a_us((w.x >> 4) & 0x0F0F0F0Fu, ahi.x, 0);
    dhi = dp4a_us((w.y >> 4) & 0x0F0F0F0Fu, ahi.y, dhi);
    dhi = dp4a_us((w.z >> 4) & 0x0F0F0F0Fu, ahi.z, dhi);
    dhi = dp4a_us((w.w >> 4) & 0x0F0F0F0Fu, ahi.w, dhi);
    dlo -= 8 * sm.x;  // nibble n encodes n - 8
    dhi -= 8 * sm.y;
  } else {
    const uint4 w0 = r.w[2 * v], w1 = r.w[2 * v + 1];
    dlo = dp4a_ss((int)w0.x, alo.x, 0);
    dlo = dp4a_ss((int)w0.y, alo.y, dlo);
    dlo = dp4a_ss((int)w0.z, alo.z, dlo);
    dlo = dp4a_ss((int)w0.w, alo.w, dlo);
    dhi = dp4a_ss((int)w1.x, ahi.x, 0);
    dhi = dp4a_ss((int)w1.y, ahi.y, dhi);
    dhi = dp4a_ss((int)w1.z, ahi.z, dhi);
    dhi = dp4a_ss((int)w1.w, ahi.w, dhi);
  }
  float tlo = __fmul_rn(__fmul_rn(__int2float_rn(dlo), as), ws);
  float thi = __fmul_rn(__fmul_rn(__int2float_rn(dhi), as), ws);
  return tlo + thi;  // the pair is summed first, then added to the lane's running sum
}

__device__ __forceinline__ float swiglu_one(float g, float u) {
  // swiglu_compat (recipe.rs:3037-3047)
  float sig = g <= -20.0f ? 0.0f : (g >= 20.0f ? 1.0f : __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

// Last writer of each 32-row group quantizes it (QuantizedActQ8 of the
// SwiGLU output) so the down projection reads int8 directly.
__device__ void swiglu_group_quant(const GemvArgs &a, int t, int64_t lr) {
  const int64_t groups = (a.rows + 31) / 32, g = lr / 32;
  const int64_t need = a.rows - g * 32 < 32 ? a.rows - g * 32 : 32;
  __threadfence();
  unsigned old = atomicAdd(&a.group_cnt[t * groups + g], 1u);
  if ((int64_t)old != need - 1) return;
  __threadfence();
  const float *src = a.y + t * a.y_stride + g * 32;
  float v[32];
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++) {
    v[j] = j < need ? __ldcg(src + j) : 0.0f;
    if (!isfinite(v[j])) v[j] = 0.0f;
    amax = fmaxf(amax, fabsf(v[j]));
  }
  float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
  int8_t *dq = a.yq + t * groups * 32 + g * 32;
#pragma unroll
  for (int j = 0; j < 32; j++) dq[j] = j < need ? act_quant_one(v[j], inv) : (int8_t)0;
  a.ys[t * groups + g] = scale;
  a.group_cnt[t * groups + g] = 0u;
}

template <int QUANT, int M, int OUT>
__global__ void __launch_bounds__(kThreads, 2) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(16) char smem[];
  __shared__ float red[33];
  constexpr int U = ChunkRegs<QUANT>::U;
  constexpr int UNITS = OUT == GEMV_OUT_SWIGLU_Q ? 2 : 1;
  const int nb = (int)(a.w.cols / 32), nbp = (nb + 3) & ~3;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + warp, nw = (int64_t)gridDim.x * kWarps;
  const int parts = (nb + 32 * U - 1) / (32 * U);
  const int64_t my_rows = gw < a.rows ? (a.rows - 1 - gw) / nw + 1 : 0;
  const int64_t n_chunks = my_rows * UNITS * parts;

  ChunkRegs<QUANT> cur, nxt;
  if (n_chunks > 0) load_chunk<QUANT>(a.w, gw, 0, nb, lane, cur);
  pdl_wait();
  gemv_prologue<M>(a, smem, nb, nbp, red);
  pdl_trigger();

  float acc0[M], acc1[M];
#pragma unroll
  for (int t = 0; t < M; t++) acc0[t] = acc1[t] = 0.0f;

  int part = 0, unit = 0;
  int64_t li = 0;  // index of the logical row within this warp's list
  for (int64_t c = 0; c < n_chunks; c++) {
    // Position of chunk c + 1.
    int npart = part + 1, nunit = unit;
    int64_t nli = li;
    if (npart == parts) { npart = 0; nunit++; if (nunit == UNITS) { nunit = 0; nli++; } }
    if (c + 1 < n_chunks) {
      int64_t nrow = gw + nli * nw + (nunit ? a.up_offset : 0);
      load_chunk<QUANT>(a.w, nrow, npart, nb, lane, nxt);
    }
#pragma unroll
    for (int v = 0; v < U; v++) {
      int b = part * 32 * U + v * 32 + lane;
      if (b < nb) {
        float ws = f16_finite(cur.d[v]);
#pragma unroll
        for (int t = 0; t < M; t++) {
          float term = block_terms<QUANT>(cur, v, smem + t * act_bytes(nbp), nbp, b, ws);
          if (unit == 0) acc0[t] += term;
          else acc1[t] += term;
        }
      }
    }
    if (part == parts - 1 && unit == UNITS - 1) {
      const int64_t lr = gw + li * nw;
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int t = 0; t < M; t++) {
        float r0 = warp_sum(acc0[t]);
        float r1 = UNITS == 2 ? warp_sum(acc1[t]) : 0.0f;
        if (lane == t) { s0 = r0; s1 = r1; }
        acc0[t] = acc1[t] = 0.0f;
      }
      if (lane < a.m) {
        const int t = lane;
        float *yp = a.y + t * a.y_stride + lr;
        if (OUT == GEMV_OUT_STORE) {
          *yp = a.bias ? s0 + a.bias[lr] : s0;
        } else if (OUT == GEMV_OUT_ADD) {
          float p = a.bias ? s0 + a.bias[lr] : s0;
          *yp = *yp + p;
        } else {
          *yp = swiglu_one(s0, s1);
          swiglu_group_quant(a, t, lr);
        }
      }
    }
    part = npart;
    unit = nunit;
    li = nli;
    cur = nxt;
  }
}

template <int QUANT, int M, int OUT>
void launch_t(const GemvArgs &a, int grid, cudaStream_t s) {
  const int nb = (int)(a.w.cols / 32), nbp = (nb + 3) & ~3;
  size_t smem = act_bytes(nbp) * M;
  auto kern = k_gemv<QUANT, M, OUT>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, a);
}

template <int QUANT, int OUT>
void launch_m(const GemvArgs &a, int grid, cudaStream_t s) {
  switch (a.m) {
    case 1: launch_t<QUANT, 1, OUT>(a, grid, s); break;
    case 2: launch_t<QUANT, 2, OUT>(a, grid, s); break;
    case 3: case 4: launch_t<QUANT, 4, OUT>(a, grid, s); break;
    default: launch_t<QUANT, 8, OUT>(a, grid, s); break;
  }
}

int g_sm_count = 0;

}  // namespace

int gemv_default_grid(const GemvArgs &a) {
  if (!g_sm_count) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  int64_t need = (a.rows + kWarps - 1) / kWarps;
  int64_t cap = (int64_t)g_sm_count * 2;
  return (int)(need < cap ? need : cap);
}

void launch_gemv(const GemvArgs &a0, cudaStream_t s) {
  if (a0.rows <= 0) return;
  GemvArgs a = a0;
  // Token counts between template sizes run the next larger instantiation;
  // token slots t >= m quantize to zero and are never written.
  int grid = a.grid > 0 ? a.grid : gemv_default_grid(a);
  if (a.w.quant == JAL_Q4_0) {
    if (a.out_mode == GEMV_OUT_STORE) launch_m<JAL_Q4_0, GEMV_OUT_STORE>(a, grid, s);
    else if (a.out_mode == GEMV_OUT_ADD) launch_m<JAL_Q4_0, GEMV_OUT_ADD>(a, grid, s);
    else launch_m<JAL_Q4_0, GEMV_OUT_SWIGLU_Q>(a, grid, s);
  } else {
    if (a.out_mode == GEMV_OUT_STORE) launch_m<JAL_Q8_0, GEMV_OUT_STORE>(a, grid, s);
    else if (a.out_mode == GEMV_OUT_ADD) launch_m<JAL_Q8_0, GEMV_OUT_ADD>(a, grid, s);
    else launch_m<JAL_Q8_0, GEMV_OUT_SWIGLU_Q>(a, grid, s);
  }
}

}  // namespace jal
