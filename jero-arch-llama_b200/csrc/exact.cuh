// Reference-order f32 arithmetic at bandwidth.
//
// The reference folds its f32 reductions left to right with one rounding per
// step (Rust `Iterator::sum`, `acc += ...`).  The int8 activation quantizer
// that follows every projection input is discontinuous, so the decode path
// reproduces those folds bit for bit.  Folds whose length is the row length
// of a projection run in parallel across rows (one chain per row); the two
// long folds over one vector -- the RMSNorm sum of squares and the softmax
// denominator, both over non-negative terms -- use seq_sum_nonneg below,
// which returns the exact value of the sequential sum without a chain of n
// dependent adds.
//
// Method (sequential sum s_{i+1} = fl(s_i + t_i), t_i >= 0).  While s stays
// inside one binade [2^e, 2^(e+1)) the rounding grid is fixed (ulp U =
// 2^(e-23)), so fl(s + t) = s + U * k(t, parity of s / U): k is t / U rounded
// to nearest, a tie going to the k that makes the result's mantissa even.  A
// run of steps inside one binade is therefore an integer increment that
// depends only on the parity of the starting mantissa: a pair (inc0, inc1).
// Pairs compose associatively, so a block of threads
//   1. sums its segments in double and scans them (an estimate P_i of s_i,
//      within i * 2^-24 relative, which places each segment in a binade),
//   2. builds each segment's pair (or marks it sequential when it may cross a
//      binade, holds non-finite terms or starts below the normal range),
//   3. composes equal-binade neighbours with a segmented warp scan, and
//   4. one thread applies the short list of composed runs and sequential
//      segments to the start value.
// Step 4 checks each run: the start must lie in the run's binade and the
// mantissa plus the increment must stay below 2^24.  Because s only grows,
// that check is exact; a run that fails it is recomputed with plain adds.
// The estimate in step 1 therefore affects speed only, never the result.
#pragma once

#include <cstdint>

#include "libm_expf.h"

namespace jal {
namespace exact {

constexpr int kSeq = -10000;  // op binade marker: add the segment's terms one by one

// One entry of the run list: terms [a, b); binade e (or kSeq) in the low
// 16 bits of `ed`, inc1 - inc0 in the high 16 bits; inc0.
struct __align__(16) SumOp {
  int a, b;
  int ed;
  uint32_t inc0;
};

template <int NT>
struct SumSmem {
  double wtot[NT / 32];
  int wcount[NT / 32], woff[NT / 32];
  SumOp ops[NT];
  float result;
};

// Barrier over a group of NT threads: the whole block (bar 0) or the named
// barrier `bar` shared by exactly NT threads.
template <int NT>
__device__ __forceinline__ void group_sync(int bar) {
  if (bar == 0) __syncthreads();
  else asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(NT) : "memory");
}

// Reference-order result of s0 + t[0] + t[1] + ... + t[n-1] (f32, round to
// nearest even at every step) for non-negative terms and a non-negative start
// s0 (+0 or -0 included: Rust's f32 `sum` starts from -0.0, `let mut acc =
// 0.0` from +0.0).  All NT threads of a warp-aligned group call it with the
// same arguments: gtid is the thread's index in the group and bar the group's
// barrier (0 = the whole block, NT == blockDim.x).  t is readable by every
// thread of the group (shared or global memory).
template <int NT, typename SM>
__device__ float seq_sum_nonneg(const float *t, int n, float s0, SM &sm, int gtid = -1, int bar = 0) {
  static_assert(NT % 32 == 0 && NT <= 1024, "block size");
  constexpr int NW = NT / 32;
  const int tid = gtid < 0 ? (int)threadIdx.x : gtid, lane = tid & 31, warp = tid >> 5;
  if (n <= 0) return s0;
  int c = (n + NT - 1) / NT;
  if (c < 4) c = 4;
  const int nseg = (n + c - 1) / c;
  const bool active = tid < nseg;
  const int a = tid * c, b = active ? min(n, a + c) : a;

  // 1. segment sums in double, block-wide exclusive scan
  double D = 0.0;
  bool finite = true;
  for (int i = a; i < b; i++) {
    const float v = t[i];
    finite = finite && isfinite(v);
    D += (double)v;
  }
  double incl = D;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sm.wtot[warp] = incl;
  group_sync<NT>(bar);
  if (warp == 0) {
    double v = lane < NW ? sm.wtot[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane < NW) sm.wtot[lane] = v;
  }
  group_sync<NT>(bar);
  const double Pa = (double)s0 + (warp ? sm.wtot[warp - 1] : 0.0) + (incl - D), Pb = Pa + D;

  // 2. this segment's run increment pair, if it stays in one binade
  int e = kSeq;
  uint32_t inc0 = 0, inc1 = 0;
  if (active && tid > 0 && finite) {
    const double u = 5.9604644775390625e-8;  // 2^-24
    const double lo = Pa * (1.0 - (double)(a + 2) * u * 1.01), hi = Pb * (1.0 + (double)(b + 2) * u * 1.01);
    if (lo >= 1.1754943508222875e-38 && hi < 3.0e38) {
      const int el = (int)((__double_as_longlong(lo) >> 52) & 0x7FF) - 1023;
      const int eh = (int)((__double_as_longlong(hi) >> 52) & 0x7FF) - 1023;
      if (el == eh) {
        e = el;
        for (int i = a; i < b; i++) {
          const uint32_t bits = __float_as_uint(t[i]);
          int E = (int)(bits >> 23);
          uint32_t m = bits & 0x7FFFFFu;
          if (E) m |= 0x800000u;
          else E = 1;
          const int sh = 127 + e - E;  // t / U = m / 2^sh
          if (sh <= 0) { e = kSeq; break; }  // t >= 2^e: the step leaves the binade
          if (sh >= 25) continue;           // t < U / 2: adds nothing
          const uint32_t K = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
          if (rem == half) {  // tie: to the even result mantissa
            inc0 += K + ((inc0 + K) & 1u);
            inc1 += K + ((1u + inc1 + K) & 1u);
          } else {
            const uint32_t k = K + (rem > half ? 1u : 0u);
            inc0 += k;
            inc1 += k;
          }
          inc0 = min(inc0, 1u << 25);
          inc1 = min(inc1, 1u << 25);
        }
      }
    }
  }

  // 3. compose runs of equal binade within the warp (segmented inclusive scan)
  const bool mono = active && e != kSeq;
  const int e_prev = __shfl_up_sync(0xffffffffu, e, 1);
  const bool mono_prev = __shfl_up_sync(0xffffffffu, mono, 1);
  const bool head = !(mono && lane > 0 && mono_prev && e_prev == e);
  uint32_t c0 = inc0, c1 = inc1;
  int start = a;
  bool f = head;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t p0 = __shfl_up_sync(0xffffffffu, c0, o), p1 = __shfl_up_sync(0xffffffffu, c1, o);
    const int ps = __shfl_up_sync(0xffffffffu, start, o);
    const bool pf = __shfl_up_sync(0xffffffffu, f, o);
    if (lane >= o && !f) {  // previous steps first, then these
      const uint32_t n0 = p0 + ((p0 & 1u) ? c1 : c0);
      const uint32_t n1 = p1 + (((1u + p1) & 1u) ? c1 : c0);
      c0 = min(n0, 1u << 25);
      c1 = min(n1, 1u << 25);
      start = ps;
      f = pf;
    }
  }
  const bool next_head = __shfl_down_sync(0xffffffffu, head, 1);
  const bool tail = active && (lane == 31 || next_head || tid + 1 >= nseg);
  const unsigned tails = __ballot_sync(0xffffffffu, tail);
  if (lane == 0) sm.wcount[warp] = __popc(tails);
  group_sync<NT>(bar);
  if (tid == 0) {  // run-list offsets of the warps
    int o = 0;
    for (int w = 0; w < NW; w++) {
      sm.woff[w] = o;
      o += sm.wcount[w];
    }
    sm.wcount[0] = o;  // total
  }
  group_sync<NT>(bar);
  if (tail) {
    SumOp op;
    int ee = mono ? e : kSeq, delta = (int)c1 - (int)c0;
    if (delta < -32767 || delta > 32767) ee = kSeq;  // cannot happen for sane inputs; stay exact
    op.a = mono ? start : a;
    op.b = b;
    op.ed = (int)(((uint32_t)ee & 0xffffu) | ((uint32_t)delta << 16));
    op.inc0 = c0;
    sm.ops[sm.woff[warp] + __popc(tails & ((1u << lane) - 1u))] = op;
  }
  group_sync<NT>(bar);

  // 4. apply the runs in order (each entry prefetched one step ahead)
  if (tid == 0) {
    const int total = sm.wcount[0];
    float s = s0;
    SumOp cur = sm.ops[0];
    for (int k = 0; k < total; k++) {
      const SumOp nxt = k + 1 < total ? sm.ops[k + 1] : cur;
      const int e = (int)(short)(cur.ed & 0xffff);
      bool done = false;
      if (e != kSeq) {
        const uint32_t bits = __float_as_uint(s);
        if ((int)(bits >> 23) == e + 127) {  // positive, in the run's binade
          const uint32_t N = (bits & 0x7FFFFFu) | 0x800000u;
          const uint32_t inc = (N & 1u) ? (uint32_t)((int)cur.inc0 + (cur.ed >> 16)) : cur.inc0;
          if (N + inc < 0x1000000u) {
            s = __uint_as_float(bits + inc);
            done = true;
          }
        }
      }
      if (!done) {
        for (int i0 = cur.a; i0 < cur.b; i0 += 16) {  // 16 loads in flight, then the adds in order
          float v[16];
#pragma unroll
          for (int u = 0; u < 16; u++) v[u] = i0 + u < cur.b ? t[i0 + u] : 0.0f;
#pragma unroll
          for (int u = 0; u < 16; u++)
            if (i0 + u < cur.b) s = __fadd_rn(s, v[u]);
        }
      }
      cur = nxt;
    }
    sm.result = s;
  }
  group_sync<NT>(bar);
  const float r = sm.result;
  group_sync<NT>(bar);  // sm may be reused right after
  return r;
}

// exp as the reference computes it: libm's expf (libm_expf.h restates
// glibc's evaluation, bit for bit).
__device__ __forceinline__ float exp_ref(float x) { return libm::expf_ref(x); }

// swiglu_compat (recipe.rs:3037-3047).
__device__ __forceinline__ float swiglu_ref(float g, float u) {
  const float sig = g <= -20.0f ? 0.0f : (g >= 20.0f ? 1.0f : __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_ref(-g))));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

}  // namespace exact
}  // namespace jal
