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
// Pairs compose associatively, so a group of threads
//   1. sums its segments (an odd number of consecutive terms per thread, so
//      that strided shared-memory reads do not conflict, held in registers)
//      and scans them: an estimate P_i of s_i within (i + c + 1) * 2^-24
//      relative, which places each segment in a binade;
//   2. builds each segment's pair (or marks it sequential when it may cross a
//      binade, holds non-finite terms or starts below the normal range);
//   3. composes equal-binade neighbours (and neighbouring sequential
//      segments) with a segmented scan over the group, which leaves a short
//      list that alternates sequential segments and runs; and
//   4. one thread applies the list in order to the start value.
// Step 4 checks each run: the start must lie in the run's binade and so must
// the end (start plus increment).  Because s only grows, that check is exact;
// if one fails the whole sum is recomputed with plain adds, so the estimate
// in step 1 affects speed only, never the result.
#pragma once

#include <cstdint>

#include "libm_expf.h"

namespace jal {
namespace exact {

// One entry of a warp's run list.  A composed run: {inc0, inc1, exponent
// field of its binade (1..254)}; sequential segments: {first, end, 0}.
struct __align__(16) SumOp {
  uint32_t x, y, E, pad;
};

template <int NT>
struct SumSmem {
  double wtot[NT / 32];
  uint32_t tc0[NT / 32], tc1[NT / 32], tcls[NT / 32], cls0[NT / 32];  // each warp's last lane; class of lane 0
  int thl[NT / 32], wcount[NT / 32];
  int total;
  SumOp ops[NT];  // the list of runs, in order
  float result;
};

// Composition of run increments: (a0, a1) for the earlier steps, then (c0,
// c1); the result replaces (c0, c1).  Index = parity of the start mantissa.
__device__ __forceinline__ void compose_inc(uint32_t a0, uint32_t a1, uint32_t &c0, uint32_t &c1) {
  const uint32_t n0 = a0 + ((a0 & 1u) ? c1 : c0), n1 = a1 + (((1u + a1) & 1u) ? c1 : c0);
  c0 = min(n0, 1u << 25);
  c1 = min(n1, 1u << 25);
}

// Barrier over a group of NT threads: the whole block (bar 0) or the named
// barrier `bar` shared by exactly NT threads.
template <int NT>
__device__ __forceinline__ void group_sync(int bar) {
  if (bar == 0) __syncthreads();
  else asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(NT) : "memory");
}

constexpr int kSumChunk = 16;  // terms a thread holds in registers at once
constexpr int kSumSlack = 16;  // floats past the last term that may be read

// Terms [base, base + 16) clamped to [base, end) (end > base): every load is
// in bounds and all are in flight together; v[j] for base + j >= end repeats
// the last term and is masked by the callers.
__device__ __forceinline__ void load_chunk(const float *t, int base, int end, float (&v)[kSumChunk]) {
#pragma unroll
  for (int j = 0; j < kSumChunk; j++) v[j] = t[min(base + j, end - 1)];
}

// Reference-order result of s0 + t[0] + t[1] + ... + t[n-1] (f32, round to
// nearest even at every step) for non-negative terms and a non-negative start
// s0 (+0 or -0 included: Rust's f32 `sum` starts from -0.0, `let mut acc =
// 0.0` from +0.0).  All NT threads of a warp-aligned group call it with the
// same arguments: gtid is the thread's index in the group and bar the group's
// barrier (0 = the whole block, NT == blockDim.x).  t is readable by every
// thread of the group (shared or global memory) up to t[n + kSumSlack - 1]:
// the values past t[n - 1] are read and ignored.
template <int NT, typename SM>
__device__ float seq_sum_nonneg(const float *t, int n, float s0, SM &sm, int gtid = -1, int bar = 0) {
  static_assert(NT % 32 == 0 && NT <= 1024, "block size");
  constexpr int CH = kSumChunk;
  const int tid = gtid < 0 ? (int)threadIdx.x : gtid, lane = tid & 31, warp = tid >> 5;
  if (n <= 0) return s0;
  int c = (n + NT - 1) / NT;
  if (c < 3) c = 3;
  c |= 1;
  const int nseg = (n + c - 1) / c;
  const bool active = tid < nseg;
  const int a = tid * c, b = active ? min(n, a + c) : a;

  // 1. segment sums (pairwise in f32 within a chunk, relative error <= 4u
  // per chunk, then in double) and their block-wide scan; a non-finite term
  // makes its own and every later estimate non-finite, which sends those
  // segments to step 4's adds
  float v[CH];
  double D = 0.0;
  for (int base = a; base < b; base += CH) {
    load_chunk(t, base, b, v);
    float d[CH];
#pragma unroll
    for (int j = 0; j < CH; j++) d[j] = base + j < b ? v[j] : 0.0f;
#pragma unroll
    for (int w = 1; w < CH; w <<= 1)
#pragma unroll
      for (int j = 0; j < CH; j += 2 * w) d[j] = __fadd_rn(d[j], d[j + w]);
    D += (double)d[0];
  }
  double incl = D;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sm.wtot[warp] = incl;
  group_sync<NT>(bar);
  double before = lane < warp ? sm.wtot[lane] : 0.0;  // lane < warp < NT / 32 <= 32
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
  const double Pa = (double)s0 + before + (incl - D), Pb = Pa + D;

  // 2. this segment's run increment pair, if it stays in one binade.  A term
  // t adds k = t / U rounded to nearest, U = 2^(e-23); x = t / U = t *
  // 2^(23-e) is exact in f32, and for 0 <= x < 2^23 the f32 sum x + 2^23
  // rounds it to the nearest integer (ties to even) in its low mantissa
  // bits.  Only an exact half (a tie) depends on the running parity, which
  // both accumulators follow.
  uint32_t E = 0, inc0 = 0, inc1 = 0;
  if (active && tid > 0) {
    // s_i is within 1.01 * i * u of the exact prefix; the estimate adds
    // (c + 1) u from the f32 chunk sums (double rounding is far below that)
    const double u = 5.9604644775390625e-8;  // 2^-24
    const double lo = Pa * (1.0 - (double)(a + c + 3) * u * 1.01), hi = Pb * (1.0 + (double)(b + c + 3) * u * 1.01);
    if (lo >= 1.0e-30 && hi < 3.0e38) {  // e >= -100: 2^(23-e) is a normal f32
      const int el = (int)((__double_as_longlong(lo) >> 52) & 0x7FF) - 1023;
      const int eh = (int)((__double_as_longlong(hi) >> 52) & 0x7FF) - 1023;
      if (el == eh) {
        const float scale = __int_as_float((127 + 23 - el) << 23);  // 2^(23-e)
        bool out = false;
        for (int base = a; base < b; base += CH) {
          if (base != a || b - a > CH) load_chunk(t, base, b, v);  // one chunk: still in registers
#pragma unroll
          for (int j = 0; j < CH; j++) {
            const bool in = base + j < b;
            const float x = fminf(__fmul_rn(v[j], scale), 8388608.0f);  // t / U, exact below 2^23
            const float y = __fadd_rn(x, 8388608.0f);                     // 2^23 + nearest integer
            out |= in && x >= 8388608.0f;                                 // t >= 2^e: leaves the binade
            const uint32_t k = in ? __float_as_uint(y) - 0x4B000000u : 0u;  // nearest, ties to even
            const float r = __fsub_rn(x, __fsub_rn(y, 8388608.0f));
            // a tie x = K + 1/2 adds the K or K + 1 that leaves the result
            // mantissa even: it depends on the running parity
            const bool tie = in && fabsf(r) == 0.5f;
            const uint32_t K = r > 0.0f ? k : k - 1u;
            inc0 += tie ? K + ((inc0 + K) & 1u) : k;
            inc1 += tie ? K + ((1u + inc1 + K) & 1u) : k;
          }
          inc0 = min(inc0, 1u << 25);  // a run never adds more than 2^24; no wrap-around
          inc1 = min(inc1, 1u << 25);
        }
        if (!out) E = (uint32_t)(el + 127);
      }
    }
  }

  // 3. compose equal neighbours: runs of one binade, and runs of sequential
  // segments (class 0).  A segmented scan within each warp (heads from one
  // ballot), a carry from the run's part in earlier warps, then the runs'
  // ends (tails) write the list in order.  Neighbouring runs always differ
  // in class, and two binade runs are never adjacent (a binade change
  // happens inside a sequential segment), so the list alternates
  // sequential, run, sequential, ... from segment 0, which is sequential.
  const uint32_t cls = active ? E : 0xFFFFFFFFu;
  const uint32_t cls_up = __shfl_up_sync(0xffffffffu, cls, 1);
  const unsigned heads = __ballot_sync(0xffffffffu, lane == 0 || cls_up != cls);
  const int hl = 31 - __clz(heads & (0xffffffffu >> (31 - lane)));  // this lane's run head in the warp
  uint32_t c0 = inc0, c1 = inc1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t p0 = __shfl_up_sync(0xffffffffu, c0, o), p1 = __shfl_up_sync(0xffffffffu, c1, o);
    if (lane - o >= hl) compose_inc(p0, p1, c0, c1);  // previous steps first, then these
  }
  if (lane == 31) {
    sm.tc0[warp] = c0;
    sm.tc1[warp] = c1;
    sm.tcls[warp] = cls;
    sm.thl[warp] = hl;
  }
  if (lane == 0) sm.cls0[warp] = cls;
  group_sync<NT>(bar);
  // The run that lane 0 continues from earlier warps: a segmented scan over
  // the warps' tails (lane l = warp l), done by every warp.
  int start = (warp * 32 + hl) * c;  // first term of this lane's run
  {
    constexpr int NW = NT / 32;
    const bool lv = lane < NW;
    uint32_t q0 = lv ? sm.tc0[lane] : 0u, q1 = lv ? sm.tc1[lane] : 0u;
    const uint32_t tcl = lv ? sm.tcls[lane] : 0xFFFFFFFFu, cl0 = lv ? sm.cls0[lane] : 0xFFFFFFFFu;
    const int thl_l = lv ? sm.thl[lane] : 0;
    const uint32_t tcl_up = __shfl_up_sync(0xffffffffu, tcl, 1);
    const bool cont = lane > 0 && cl0 != 0xFFFFFFFFu && cl0 == tcl_up;  // warp lane's lane 0 continues a run
    const unsigned wheads = __ballot_sync(0xffffffffu, !(cont && thl_l == 0));
    const int wh = 31 - __clz(wheads & (0xffffffffu >> (31 - lane)));  // warp where warp lane's tail run starts
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t p0 = __shfl_up_sync(0xffffffffu, q0, o), p1 = __shfl_up_sync(0xffffffffu, q1, o);
      if (lane - o >= wh) compose_inc(p0, p1, q0, q1);
    }
    const int rs = (wh * 32 + __shfl_sync(0xffffffffu, thl_l, wh)) * c;
    const bool cont_w = __shfl_sync(0xffffffffu, cont, warp);
    const uint32_t k0 = __shfl_sync(0xffffffffu, q0, warp > 0 ? warp - 1 : 0);
    const uint32_t k1 = __shfl_sync(0xffffffffu, q1, warp > 0 ? warp - 1 : 0);
    const int rs_prev = __shfl_sync(0xffffffffu, rs, warp > 0 ? warp - 1 : 0);
    if (cont_w && hl == 0 && active) {
      compose_inc(k0, k1, c0, c1);
      start = rs_prev;
    }
  }
  const uint32_t cls_dn = __shfl_down_sync(0xffffffffu, cls, 1);
  const uint32_t next_cls = lane < 31 ? cls_dn : (warp + 1 < NT / 32 ? sm.cls0[warp + 1] : 0xFFFFFFFFu);
  const bool tail = active && next_cls != cls;
  const unsigned tails = __ballot_sync(0xffffffffu, tail);
  if (lane == 0) sm.wcount[warp] = __popc(tails);
  group_sync<NT>(bar);
  int off = lane < warp ? sm.wcount[lane] : 0;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) off += __shfl_xor_sync(0xffffffffu, off, o);
  if (tail) {
    SumOp op;
    op.x = E ? c0 : (uint32_t)start;
    op.y = E ? c1 : (uint32_t)b;
    op.E = E;
    op.pad = 0u;
    sm.ops[off + __popc(tails & ((1u << lane) - 1u))] = op;
  }
  if (tid == NT - 1) sm.total = off + __popc(tails);  // the last warp's offset + count
  group_sync<NT>(bar);

  // 4. apply the list: sequential entries at even places, runs at odd
  // places.  A run's checks (start and end in its binade) are collected and
  // tested once at the end; if one failed -- the estimate cannot place a run
  // wrongly, so this is a safety net only -- the sum is recomputed with
  // plain adds.
  if (tid == 0) {
    const int T = sm.total;
    float s = s0;
    bool ok = true;
    // Entry k + 2 is loaded and the terms of the next sequential entry are
    // in registers while entry k is applied; two list places per step.
    auto load_seq = [&](const SumOp &q, float (&x)[CH]) {
      const int base = q.E ? 0 : (int)q.x;  // a run's x is an increment, not a place
#pragma unroll
      for (int j = 0; j < CH; j++) x[j] = t[base + j];  // t has CH readable floats past its end
    };
    auto step = [&](int k, const SumOp &sq, const SumOp &run, const float (&x)[CH]) {
      ok = ok & (sq.E == 0u);  // the alternation holds by construction; checked all the same
      const int len = (int)sq.y - (int)sq.x;
#pragma unroll
      for (int j = 0; j < CH; j++) s = __fadd_rn(s, j < len ? x[j] : -0.0f);  // s + -0 == s for every s
      for (int i0 = (int)sq.x + CH; i0 < (int)sq.y; i0 += CH) {  // long sequential entries
        float y[CH];
#pragma unroll
        for (int j = 0; j < CH; j++) y[j] = t[i0 + j];
#pragma unroll
        for (int j = 0; j < CH; j++) s = __fadd_rn(s, i0 + j < (int)sq.y ? y[j] : -0.0f);
      }
      if (k + 1 < T) {
        const uint32_t bits = __float_as_uint(s);
        const uint32_t nb = bits + ((bits & 1u) ? run.y : run.x);  // mantissa parity = parity of the bits
        ok = ok & (run.E != 0u) & ((bits >> 23) == run.E) & ((nb >> 23) == run.E);  // start and end in the binade
        s = __uint_as_float(nb);
      }
    };
    auto at = [&](int k) { return sm.ops[k < T ? k : T - 1]; };
    SumOp sq = at(0), run = at(1), nsq = at(2), nrun = at(3);
    float xa[CH], xb[CH];
    load_seq(sq, xa);
    for (int k = 0; k < T; k += 4) {
      load_seq(nsq, xb);
      const SumOp sq2 = at(k + 4), run2 = at(k + 5);
      step(k, sq, run, xa);
      if (k + 2 >= T) break;
      load_seq(sq2, xa);
      const SumOp nsq2 = at(k + 6), nrun2 = at(k + 7);
      step(k + 2, nsq, nrun, xb);
      sq = sq2;
      run = run2;
      nsq = nsq2;
      nrun = nrun2;
    }
    if (!ok) {
      s = s0;
      for (int i0 = 0; i0 < n; i0 += CH) {
        float x[CH];
        load_chunk(t, i0, n, x);
#pragma unroll
        for (int j = 0; j < CH; j++)
          if (i0 + j < n) s = __fadd_rn(s, x[j]);
      }
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
