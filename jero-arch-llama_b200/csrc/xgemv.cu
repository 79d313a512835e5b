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
// output rows.  K is cut into slabs of 32 blocks (1024 columns).  For a batch
// of up to 64 rows the CTA streams slab 0 of every row, then slab 1, and so
// on: a warp takes one (row, slab) unit at a time, lane l owning block
// 32 * slab + l; its quants and f16 scale arrive through a per-warp ring of
// cp.async copies (DEPTH units ahead, the first ones issued before
// griddepcontrol.wait), and its two chunk terms go to a shared-memory slab
// buffer.  After each slab one owner thread per row folds that slab's 64
// terms into the row's accumulator, in order, while the warps fill the
// other buffer with the next slab.  The fold of a row therefore keeps pace
// with its stream, and the only serial tail is the last slab's 64 adds.
//
// The activation prologue (optional RMSNorm, then QuantizedActQ8 per
// 32-block) is computed by every CTA into shared memory after the wait; the
// RMSNorm sum of squares is the reference's sequential sum, computed with
// exact::seq_sum_nonneg.
#include <cuda_fp16.h>

#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "exact.cuh"
#include "jal.h"

namespace jal {

namespace {

constexpr int kNT = 512, kNW = kNT / 32;
constexpr int kUnits = 64;   // physical rows per batch
constexpr int kTP = 68;      // term row pitch (floats): 64 terms + 4 (conflict-free owner reads)

template <int QUANT>
struct XCfg {
  static constexpr int BQ = QUANT == JAL_Q4_0 ? 16 : 32;  // quant bytes per block
  static constexpr int SLOT = 32 * BQ + 64;               // one unit: 32 blocks of quants + 32 f16 scales
  static constexpr int DEPTH = QUANT == JAL_Q4_0 ? 8 : 5;
};

// Shared memory carve-up (bytes, 16-aligned pieces).
struct XLayout {
  int nb, nslab, nbp;
  size_t act_q, act_m, terms, stage, xsq, sum, total;
};

template <int QUANT>
__host__ __device__ inline XLayout x_layout(int64_t cols, int in_mode) {
  XLayout L;
  L.nb = (int)(cols / 32);
  L.nslab = (L.nb + 31) / 32;
  L.nbp = L.nslab * 32;
  size_t o = 0;
  L.act_q = o; o += (size_t)L.nbp * 32;
  L.act_m = o; o += (size_t)L.nbp * 16;
  L.terms = o; o += (size_t)2 * kUnits * kTP * 4;
  L.stage = o; o += (size_t)kNW * XCfg<QUANT>::DEPTH * XCfg<QUANT>::SLOT;
  L.xsq = o; if (in_mode == GEMV_IN_NORM) o += (size_t)L.nb * 32 * 4;
  L.sum = o; if (in_mode == GEMV_IN_NORM) o += (sizeof(exact::SumSmem<kNT>) + 15) / 16 * 16;
  L.total = o;
  return L;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Position in a warp's unit sequence: batch, slab, k-th unit of the warp.
struct UnitCursor {
  int b = 0, s = 0, k = 0, cnt = 0;
};

// Activation prologue: QuantizedActQ8 of the (optionally RMSNorm'd) input,
// one warp per 32-block, lane = element.  act_q gets the int8 quants,
// act_m {scale, sum of quants 0..15, sum of quants 16..31, 0}.
template <typename SumSM>
__device__ void x_prologue(const GemvArgs &a, const XLayout &L, char *smem, SumSM *ssm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int8_t *aq = (int8_t *)(smem + L.act_q);
  float4 *am = (float4 *)(smem + L.act_m);
  const int K = L.nb * 32;
  for (int b = L.nb + warp; b < L.nbp; b += kNW) {  // padding blocks
    aq[b * 32 + lane] = 0;
    if (lane == 0) am[b] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (a.in_mode == GEMV_IN_Q8) {
    for (int b = warp; b < L.nb; b += kNW) {
      const int q = a.xq[(int64_t)b * 32 + lane];
      aq[b * 32 + lane] = (int8_t)q;
      int s = q;
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 8);
      const int s16 = __shfl_sync(0xffffffffu, s, 16);
      if (lane == 0) am[b] = make_float4(a.xs[b], __int_as_float(s), __int_as_float(s16), 0.f);
    }
    __syncthreads();
    return;
  }
  float inv = 1.0f;
  if (a.in_mode == GEMV_IN_NORM) {
    float *xsq = (float *)(smem + L.xsq);
    for (int i = tid; i < K; i += kNT) {
      const float v = a.x[i];
      xsq[i] = __fmul_rn(v, v);
    }
    __syncthreads();
    const float ss = exact::seq_sum_nonneg<kNT>(xsq, K, -0.0f, *ssm);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
  }
  for (int b = warp; b < L.nb; b += kNW) {
    const int i = b * 32 + lane;
    float v = a.x[i];
    if (a.in_mode == GEMV_IN_NORM) v = __fmul_rn(__fmul_rn(v, inv), a.norm_w[i]);
    if (!isfinite(v)) v = 0.0f;
    const float amax = warp_max(fabsf(v));
    const float scale = act_scale_from_amax(amax), is = act_inv_from_scale(scale);
    const int q = act_quant_one(v, is);
    aq[i] = (int8_t)q;
    int s = q;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 8);
    const int s16 = __shfl_sync(0xffffffffu, s, 16);
    if (lane == 0) am[b] = make_float4(scale, __int_as_float(s), __int_as_float(s16), 0.f);
  }
  __syncthreads();
}

template <int QUANT, int OUT>
__global__ void __launch_bounds__(kNT, 1) k_xgemv(const GemvArgs a) {
  using C = XCfg<QUANT>;
  constexpr int UNITS = OUT == GEMV_OUT_SWIGLU ? 2 : 1;
  constexpr int RBL = kUnits / UNITS;  // logical rows per batch
  extern __shared__ __align__(16) char smem[];
  const XLayout L = x_layout<QUANT>(a.w.cols, a.in_mode);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = a.rows / gridDim.x, rem = a.rows % gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * base + ((int64_t)blockIdx.x < rem ? blockIdx.x : rem);
  const int cnt = (int)(base + ((int64_t)blockIdx.x < rem ? 1 : 0));
  const int nbatch = (cnt + RBL - 1) / RBL;
  char *stage = smem + L.stage + (size_t)warp * C::DEPTH * C::SLOT;
  float *terms = (float *)(smem + L.terms);

  auto batch_units = [&](int b) { return min(RBL, cnt - b * RBL) * UNITS; };
  auto warp_cnt = [&](int b) {
    const int nun = batch_units(b);
    return nun > warp ? (nun - 1 - warp) / kNW + 1 : 0;
  };
  // Physical row of unit u in batch b (SWIGLU: gate rows, then up rows).
  auto unit_row = [&](int b, int u) -> int64_t {
    const int nl = min(RBL, cnt - b * RBL);
    const int64_t lr = r0 + (int64_t)b * RBL;
    if (UNITS == 2) return u < nl ? lr + u : a.up_offset + lr + (u - nl);
    return lr + u;
  };
  auto advance = [&](UnitCursor &c) {
    if (++c.k < c.cnt) return;
    c.k = 0;
    if (++c.s < L.nslab) return;
    c.s = 0;
    for (c.b++; c.b < nbatch; c.b++)
      if ((c.cnt = warp_cnt(c.b)) > 0) return;
  };
  auto first = [&](UnitCursor &c) {
    c = UnitCursor();
    for (c.b = 0; c.b < nbatch; c.b++)
      if ((c.cnt = warp_cnt(c.b)) > 0) return;
  };
  // Issue the copies of unit c into its slot; always commits one group.
  auto issue = [&](const UnitCursor &c, int slot) {
    if (c.b < nbatch) {
      const int64_t pr = unit_row(c.b, warp + c.k * kNW);
      const int blk = c.s * 32 + lane;
      char *dst = stage + slot * C::SLOT;
      if (blk < L.nb) {
        const uint8_t *src = a.w.qs + pr * a.w.qs_stride + (int64_t)blk * C::BQ;
        cp_async16(dst + lane * C::BQ, src);
        if (C::BQ == 32) cp_async16(dst + lane * C::BQ + 16, src + 16);
      }
      const int pb = blk & ~1;
      if (pb < L.nb) cp_async4(dst + 32 * C::BQ + pb * 2 - c.s * 64, (const char *)(a.w.d + pr * a.w.d_stride + pb));
    }
    cp_commit();
  };

  UnitCursor ld, cp;
  first(ld);
  first(cp);
  int q_ld = 0;
#pragma unroll 1
  for (int d = 0; d < C::DEPTH; d++) {
    issue(ld, q_ld % C::DEPTH);
    if (ld.b < nbatch) advance(ld);
    q_ld++;
  }
  pdl_wait();
  pdl_trigger();
  x_prologue(a, L, smem, (exact::SumSmem<kNT> *)(smem + L.sum));

  const int8_t *aq = (const int8_t *)(smem + L.act_q);
  const float4 *am = (const float4 *)(smem + L.act_m);
  int q_cp = 0, gslab = 0;
  float acc0 = 0.0f, acc1 = 0.0f;  // owner accumulators (gate/up for SWIGLU)
  for (int b = 0; b < nbatch; b++) {
    const int nl = min(RBL, cnt - b * RBL);
    const int mycnt = warp_cnt(b);
    for (int s = 0; s < L.nslab; s++) {
      float *tb = terms + (size_t)(gslab & 1) * kUnits * kTP;
      const int blk = s * 32 + lane;
      const bool live = blk < L.nb;
      // this lane's activation block for the slab
      int4 xlo = make_int4(0, 0, 0, 0), xhi = xlo;
      float asc = 0.f;
      int s0 = 0, s1 = 0;
      if (live) {
        xlo = *(const int4 *)(aq + blk * 32);
        xhi = *(const int4 *)(aq + blk * 32 + 16);
        const float4 m = am[blk];
        asc = m.x;
        s0 = __float_as_int(m.y);
        s1 = __float_as_int(m.z);
      }
      for (int k = 0; k < mycnt; k++) {
        cp_wait<C::DEPTH - 1>();
        const char *src = stage + (q_cp % C::DEPTH) * C::SLOT;
        if (live) {
          int d0, d1;
          if (QUANT == JAL_Q4_0) {
            const uint4 w = *(const uint4 *)(src + lane * 16);
            d0 = dp4a_us(w.x & 0x0F0F0F0Fu, xlo.x, 0);
            d0 = dp4a_us(w.y & 0x0F0F0F0Fu, xlo.y, d0);
            d0 = dp4a_us(w.z & 0x0F0F0F0Fu, xlo.z, d0);
            d0 = dp4a_us(w.w & 0x0F0F0F0Fu, xlo.w, d0);
            d1 = dp4a_us(w.x & 0xF0F0F0F0u, xhi.x, 0);
            d1 = dp4a_us(w.y & 0xF0F0F0F0u, xhi.y, d1);
            d1 = dp4a_us(w.z & 0xF0F0F0F0u, xhi.z, d1);
            d1 = dp4a_us(w.w & 0xF0F0F0F0u, xhi.w, d1);
            d0 -= 8 * s0;              // nibble n encodes n - 8
            d1 = (d1 >> 4) - 8 * s1;   // high nibbles were multiplied by 16 in place
          } else {
            const uint4 w0 = *(const uint4 *)(src + lane * 32), w1 = *(const uint4 *)(src + lane * 32 + 16);
            d0 = dp4a_ss((int)w0.x, xlo.x, 0);
            d0 = dp4a_ss((int)w0.y, xlo.y, d0);
            d0 = dp4a_ss((int)w0.z, xlo.z, d0);
            d0 = dp4a_ss((int)w0.w, xlo.w, d0);
            d1 = dp4a_ss((int)w1.x, xhi.x, 0);
            d1 = dp4a_ss((int)w1.y, xhi.y, d1);
            d1 = dp4a_ss((int)w1.z, xhi.z, d1);
            d1 = dp4a_ss((int)w1.w, xhi.w, d1);
          }
          const float ws = __half2float(__ushort_as_half(*(const uint16_t *)(src + 32 * C::BQ + lane * 2)));
          const float t0 = __fmul_rn(__fmul_rn(__int2float_rn(d0), asc), ws);
          const float t1 = __fmul_rn(__fmul_rn(__int2float_rn(d1), asc), ws);
          *(float2 *)(tb + (warp + k * kNW) * kTP + 2 * lane) = make_float2(t0, t1);
        }
        q_cp++;
        issue(ld, q_ld % C::DEPTH);
        if (ld.b < nbatch) advance(ld);
        q_ld++;
      }
      __syncthreads();  // slab terms complete; the other buffer's fold is done
      if (tid < nl) {
        const int nt = 2 * min(32, L.nb - s * 32);
        const float *r0p = tb + tid * kTP;
        const float *r1p = tb + (nl + tid) * kTP;
        int i = 0;
        for (; i + 4 <= nt; i += 4) {
          const float4 v = *(const float4 *)(r0p + i);
          acc0 = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc0, v.x), v.y), v.z), v.w);
          if (UNITS == 2) {
            const float4 u = *(const float4 *)(r1p + i);
            acc1 = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc1, u.x), u.y), u.z), u.w);
          }
        }
        for (; i < nt; i++) {
          acc0 = __fadd_rn(acc0, r0p[i]);
          if (UNITS == 2) acc1 = __fadd_rn(acc1, r1p[i]);
        }
      }
      gslab++;
    }
    if (tid < nl) {  // epilogue of the batch's rows
      const int64_t lr = r0 + (int64_t)b * RBL + tid;
      float *yp = a.y + lr;
      if (OUT == GEMV_OUT_STORE) {
        *yp = a.bias ? __fadd_rn(acc0, a.bias[lr]) : acc0;
      } else if (OUT == GEMV_OUT_ADD) {
        const float p = a.bias ? __fadd_rn(acc0, a.bias[lr]) : acc0;
        *yp = __fadd_rn(*yp, p);
      } else {
        *yp = exact::swiglu_ref(acc0, acc1);
      }
      acc0 = acc1 = 0.0f;
    }
  }
  cp_wait<0>();
}

template <int QUANT, int OUT>
void launch_x(const GemvArgs &a, int grid, cudaStream_t s) {
  const XLayout L = x_layout<QUANT>(a.w.cols, a.in_mode);
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
  return quant == JAL_Q4_0 ? x_layout<JAL_Q4_0>(cols, in_mode).total : x_layout<JAL_Q8_0>(cols, in_mode).total;
}

bool xgemv_supported(const GemvArgs &a) {
  if (a.m != 1 || (a.w.quant != JAL_Q4_0 && a.w.quant != JAL_Q8_0)) return false;
  if (a.w.cols % 32 != 0 || a.w.qs_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(a.w.qs) & 15) != 0) return false;
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
