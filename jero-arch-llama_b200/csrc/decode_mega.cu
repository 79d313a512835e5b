// Persistent decode step (one token, fast numerics).
//
// One cooperative launch of one CTA per SM runs a whole decode token: the
// embedding, every layer's five phases (Q/K/V projection, attention, O
// projection + residual, gate/up projection + SwiGLU, down projection +
// residual) and the LM head with greedy argmax.  Phases are separated by a
// grid barrier instead of kernel boundaries, so no CTA has to be scheduled
// between phases, and each CTA starts the next phases' memory traffic before
// it waits:
//   - before each barrier, thread 0 asks the copy engine to prefetch this
//     CTA's first rows of the projection after next into L2;
//   - at the end of the Q/K/V phase the CTA starts the bulk copies of its
//     attention slice of the cache (positions below the current one).
// Projection phases run the segmented fast path of gemv_dev.cuh on the
// CTA's contiguous row range.  Attention splits every KV head over
// grid / n_kv CTAs; each writes its partial (max, denominator, P.V) to global
// memory and the last CTA of a head to finish merges the partials in split
// order and writes the head group's output and its QuantizedActQ8 form.
// Every wait is bounded: a grid barrier that gives up sets bit 8 of the
// context error word (a KV tile wait bit 2) and later barriers stop waiting,
// so the kernel always finishes.
//
// The phases are separate (non-inlined) device functions so that each gets
// its own register allocation; the projection phase uses 16-byte loads
// because ptxas rejects the 32-byte form in a non-inlined function.
#include <cuda_fp16.h>

#include "attn_dev.cuh"
#include "dev_util.cuh"
#include "device.hpp"
#include "gemv_dev.cuh"
#include "jal.h"

namespace jal {

namespace {

using namespace gdev;
using namespace adev;

constexpr int kMW = 8;  // warps per CTA (up to 255 registers per thread)
constexpr int kMT = kMW * 32;
constexpr uint32_t kGridSpin = 1u << 22;  // bounded polls of a grid barrier
constexpr int kErrAttnWait = 2, kErrGridWait = 8;
constexpr int64_t kPrefetchBytes = 64 * 1024;
constexpr size_t kAttnWs = 16 * 1024;  // attention workspace after the K/V ring
#ifndef JAL_MEGA_DQ4
#define JAL_MEGA_DQ4 4
#endif
constexpr int kDepthQ4 = JAL_MEGA_DQ4, kDepthQ8 = 3;  // rows in flight per warp

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Sense-reversing barrier over all CTAs of the cooperative grid.  bar[0]
// counts arrivals, bar[1] is the generation.  Once a wait gives up, this CTA
// stops waiting at later barriers (*broken).
__device__ __noinline__ void grid_sync(unsigned *bar, int *err, int *broken) {
  __syncthreads();
  if (threadIdx.x == 0 && !*broken) {
    unsigned *count = bar, *gen = bar + 1;
    const unsigned g = ld_acquire(gen);
    __threadfence();
    if (atomicAdd(count, 1u) == gridDim.x - 1) {
      atomicExch(count, 0u);
      __threadfence();
      st_release(gen, g + 1);
    } else {
      uint32_t it = 0;
      while (ld_acquire(gen) == g) {
        if (++it > kGridSpin) {
          *broken = 1;
          if (err) atomicOr(err, kErrGridWait);
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
  }
  __syncthreads();
}

__device__ __forceinline__ void cta_rows(int64_t rows, int64_t &r0, int64_t &cnt) {
  const int64_t base = rows / gridDim.x, rem = rows % gridDim.x, c = blockIdx.x;
  r0 = c * base + (c < rem ? c : rem);
  cnt = base + (c < rem ? 1 : 0);
}

// Thread 0: L2 prefetch of this CTA's first rows of a projection.
__device__ __forceinline__ void prefetch_rows(const DevMat &w, int64_t rows, int units, int64_t up_offset) {
  if (threadIdx.x != 0) return;
  int64_t r0, cnt;
  cta_rows(rows, r0, cnt);
  if (cnt <= 0) return;
  int64_t pr = kPrefetchBytes / (units * w.qs_stride);
  if (pr < 1) pr = 1;
  if (pr > cnt) pr = cnt;
  for (int u = 0; u < units; u++)
    l2_prefetch_bulk(w.qs + (r0 + (u ? up_offset : 0)) * w.qs_stride, (uint64_t)(pr * w.qs_stride));
}

// One projection on this CTA's contiguous row range (segmented fast path of
// the per-projection kernel, with the output mode a run-time value).
template <int QUANT>
__device__ __forceinline__ void gemv_phase(const GemvArgs &a, char *smem, float *red) {
  constexpr int DEPTH = QUANT == JAL_Q4_0 ? kDepthQ4 : kDepthQ8;
  const int out = a.out_mode;
  const int ush = out == GEMV_OUT_SWIGLU ? 1 : 0;  // log2 of units per row
  const int nb = (int)(a.w.cols / 32), nseg = seg_count(a.w.cols), nbp = nseg * kSegBlocks;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int seg = warp % nseg, phase = warp / nseg, nph = kMW / nseg;
  int64_t r0, cnt;
  cta_rows(a.rows, r0, cnt);
  const int my_rows = (phase < nph && cnt > phase) ? (int)((cnt - 1 - phase) / nph + 1) : 0;
  const int64_t gw = r0 + phase;
  const int total = my_rows << ush;
  float *part = (float *)(smem + w4_act_region(a.in_mode, nb, nseg));  // [cnt][nseg]
#define UNIT_ROW(k) (gw + (int64_t)((k) >> ush) * nph + ((ush && ((k) & 1)) ? a.up_offset : 0))
  gemv_prologue_pre<1, kMW>(a, smem, nb, nbp);
  gemv_prologue<1, kMW>(a, smem, nb, nbp, red);
  W4Row<QUANT> buf[DEPTH];
#pragma unroll
  for (int j = 0; j < DEPTH; j++)
    if (j < total) w4_load<QUANT, false>(a.w, UNIT_ROW(j), seg, nb, lane, buf[j]);
  W4Act x;
#pragma unroll
  for (int v = 0; v < 4; v++) {
    const int b = seg * kSegBlocks + 4 * lane + v;
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
        if (k + DEPTH < total) w4_load<QUANT, false>(a.w, UNIT_ROW(k + DEPTH), seg, nb, lane, buf[j]);
        s = warp_sum(s);
        const int li = phase + (k >> ush) * nph;
        if (ush && (k & 1) == 0) {
          gate = s;
        } else if (nseg > 1) {
          if (lane == 0) part[li * nseg + seg] = s;
        } else if (lane == 0) {
          const int64_t lr = r0 + li;
          float *yp = a.y + lr;
          if (out == GEMV_OUT_STORE) *yp = a.bias ? s + a.bias[lr] : s;
          else if (out == GEMV_OUT_ADD) *yp = *yp + (a.bias ? s + a.bias[lr] : s);
          else *yp = swiglu_one(gate, s);
        }
      }
    }
  }
#undef UNIT_ROW
  if (nseg > 1 && !ush) {
    __syncthreads();
    for (int li = threadIdx.x; li < cnt; li += kMT) {
      float s = 0.0f;
      for (int q = 0; q < nseg; q++) s += part[li * nseg + q];
      const int64_t lr = r0 + li;
      float *yp = a.y + lr;
      if (out == GEMV_OUT_STORE) *yp = a.bias ? s + a.bias[lr] : s;
      else *yp = *yp + (a.bias ? s + a.bias[lr] : s);
    }
  }
  __syncthreads();
}

// The one projection routine of the kernel: a single non-inlined function
// for every projection phase (ptxas splits the register file between
// several large callees of one kernel, which made each of them spill).
__device__ __noinline__ void gemv_run(const GemvArgs &a, char *smem, float *red) {
  if (a.w.quant == JAL_Q4_0) gemv_phase<JAL_Q4_0>(a, smem, red);
  else gemv_phase<JAL_Q8_0>(a, smem, red);
}

struct Slice {
  int h = 0, si = 0;
  int64_t pos = 0, s0 = 0, s1 = 0;
  int nt = 0;
  bool active = false;
};

template <int TP>
__device__ __forceinline__ Slice attn_slice(const MegaArgs &a) {
  Slice s;
  const int S = a.splits, c = blockIdx.x;
  s.active = c < a.n_kv * S;
  s.h = c / S;
  s.si = c % S;
  s.pos = *a.d_pos;
  const int64_t seq = s.pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t per = (seq - lo + S - 1) / S;
  s.s0 = lo + s.si * per;
  s.s1 = s.s0 + per < seq ? s.s0 + per : seq;
  const int64_t len = s.s1 > s.s0 ? s.s1 - s.s0 : 0;
  s.nt = (int)((len + TP - 1) / TP);
  return s;
}

// End of the Q/K/V phase: start the copies of this CTA's cache slice.
template <int HD, bool F16>
__device__ __forceinline__ void attn_issue(const MegaArgs &a, int layer, char *ring, uint64_t *bars) {
  using Gm = AttnGeom<HD, F16, kMW>;
  if (threadIdx.x != 0) return;
  const Slice sl = attn_slice<Gm::TP>(a);
  if (!sl.active) return;
  fence_proxy_async();  // the projection phase's shared-memory reads precede the copies
  for (int k = 0; k < sl.nt && k < kStages; k++) {
    const int64_t t0 = sl.s0 + (int64_t)k * Gm::TP;
    const int n = (int)(sl.s1 - t0 < Gm::TP ? sl.s1 - t0 : Gm::TP);
    issue_tile<HD, F16>(a.kv, layer, ring + k * kStageBytes, &bars[k], t0, n, sl.h);
  }
}

template <int HD, bool F16, int GP>
__device__ __noinline__ void attn_phase(const MegaArgs &a, const MegaLayer &L, int layer, char *ring,
                                        uint64_t *bars, uint32_t *par_s) {
  using Gm = AttnGeom<HD, F16, kMW>;
  constexpr int TP = Gm::TP, LG = Gm::LG, PPS = Gm::PPS, DPL = Gm::DPL, TPW = Gm::TPW, VD = Gm::VD;
  const Slice sl = attn_slice<TP>(a);
  if (!sl.active) return;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = (int)(a.n_heads_q / a.n_kv), h = sl.h, S = a.splits;
  const int64_t Q = a.n_heads_q * HD, KVD = a.n_kv * HD, pos = sl.pos, seq = pos + 1;
  // workspace after the ring
  char *ws = ring + kStages * kStageBytes;
  float(*q_s)[HD] = (float(*)[HD])ws;                   // [GP][HD]
  float *kn_s = (float *)(ws + GP * HD * 4);            // [HD]
  float *vn_s = kn_s + HD;                              // [HD]
  float *cs_s = vn_s + HD;                              // [2][HD/2]
  float *p_all = cs_s + HD;                             // [kMW][TPW * GP]
  float *wm_s = p_all + kMW * TPW * GP;                 // [64][GP]: warp, then split merge weights
  float *den = wm_s + 64 * GP;                          // [GP]
  int *flag_s = (int *)(den + GP);
  const bool rope = !L.skip_rope && pos > 0;
  const int half = (int)(a.rotary_dim / 2);
  if (rope) {
    const bool use_long = a.long_threshold >= 0 && seq > a.long_threshold;
    const float *ct = (use_long ? a.cos_long : a.cos_tab) + pos * half;
    const float *st = (use_long ? a.sin_long : a.sin_tab) + pos * half;
    for (int j = tid; j < half; j += kMT) {
      cs_s[j] = ct[j];
      cs_s[HD / 2 + j] = st[j];
    }
  }
  __syncthreads();
  const bool own_pos = pos >= sl.s0 && pos < sl.s1;
  const int64_t app = own_pos ? kv_elem(a.kv, layer, h, pos) : 0;
  for (int i = tid; i < (GP + 2) * HD; i += kMT) {
    const int g = i / HD, d = i % HD;
    if (g < GP && g >= G) {
      q_s[g][d] = 0.0f;
      continue;
    }
    const int64_t off = g < GP ? (int64_t)(h * G + g) * HD : (g == GP ? Q : Q + KVD) + (int64_t)h * HD;
    const float *bias = g < GP ? L.bq : (g == GP ? L.bk : L.bv);
    const int64_t boff = g < GP ? (int64_t)(h * G + g) * HD : (int64_t)h * HD;
    float o = a.qkv[off + d];
    if (bias) o = __fadd_rn(o, bias[boff + d]);
    if (rope && g <= GP && d < 2 * half) {
      const bool first = a.neox ? d < half : (d & 1) == 0;
      const int j = a.neox ? (first ? d : d - half) : d / 2;
      const int partner = a.neox ? (first ? d + half : d - half) : (d ^ 1);
      float other = a.qkv[off + partner];
      if (bias) other = __fadd_rn(other, bias[boff + partner]);
      const float c = cs_s[j], sn = cs_s[HD / 2 + j];
      const float x0 = first ? o : other, x1 = first ? other : o;
      o = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (g < GP) {
      q_s[g][d] = o;
    } else {
      if (F16) o = __half2float(__float2half_rn(o));
      if (g == GP) kn_s[d] = o;
      else vn_s[d] = o;
      if (own_pos) store_kv(g == GP ? a.kv.k : a.kv.v, a.kv.f16, app + d, o);
    }
  }
  __syncthreads();

  const int c = lane % LG, grp = lane / LG;
  float qr[GP][DPL];
#pragma unroll
  for (int g = 0; g < GP; g++)
#pragma unroll
    for (int k = 0; k < DPL; k++) qr[g][k] = q_s[g][c * DPL + k];
  float m_run[GP], acc[GP][VD];
  float l_lane = 0.0f;
#pragma unroll
  for (int g = 0; g < GP; g++) {
    m_run[g] = -INFINITY;
#pragma unroll
    for (int j = 0; j < VD; j++) acc[g][j] = 0.0f;
  }
  bool ok = true;
  float *pw = p_all + warp * TPW * GP;
  const uint32_t par = *par_s;
  for (int k = 0; k < sl.nt; k++) {
    const int st = k % kStages;
    const uint32_t parity = ((par >> st) & 1u) ^ (uint32_t)((k / kStages) & 1);
    if (!mbar_wait_bounded(&bars[st], parity)) ok = false;
    const int64_t t0 = sl.s0 + (int64_t)k * TP;
    const int n = (int)(sl.s1 - t0 < TP ? sl.s1 - t0 : TP);
    char *Ks = ring + st * kStageBytes;
    char *Vs = Ks + TP * Gm::ROW;
    if (own_pos && pos >= t0 && pos < t0 + n) {
      const int j = (int)(pos - t0);
      for (int d = tid; d < HD; d += kMT) {
        if (F16) {
          ((__half *)(Ks + j * Gm::ROW))[d] = __float2half_rn(kn_s[d]);
          ((__half *)(Vs + j * Gm::ROW))[d] = __float2half_rn(vn_s[d]);
        } else {
          ((float *)(Ks + j * Gm::ROW))[d] = kn_s[d];
          ((float *)(Vs + j * Gm::ROW))[d] = vn_s[d];
        }
      }
      __syncthreads();
    }
    float mt[GP];
#pragma unroll
    for (int g = 0; g < GP; g++) mt[g] = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < TPW / PPS; sp++) {
      const int jl = sp * PPS + grp;
      const int j = warp * TPW + jl;
      float d[GP];
#pragma unroll
      for (int g = 0; g < GP; g++) d[g] = 0.0f;
      if (j < n) {
        float kv[DPL];
        load_vals<F16, DPL>(Ks + j * Gm::ROW + c * 16, kv);
#pragma unroll
        for (int g = 0; g < GP; g++)
#pragma unroll
          for (int e = 0; e < DPL; e++) d[g] = fmaf(qr[g][e], kv[e], d[g]);
      }
#pragma unroll
      for (int o = 1; o < LG; o <<= 1)
#pragma unroll
        for (int g = 0; g < GP; g++) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
      float mine = -INFINITY;
#pragma unroll
      for (int g = 0; g < GP; g++) {
        const float sc = j < n ? __fmul_rn(d[g], a.scale) : -INFINITY;
        mt[g] = fmaxf(mt[g], sc);
        if (g == c) mine = sc;
      }
      if (c < GP) pw[jl * GP + c] = mine;
    }
#pragma unroll
    for (int o = LG; o < 32; o <<= 1)
#pragma unroll
      for (int g = 0; g < GP; g++) mt[g] = fmaxf(mt[g], __shfl_xor_sync(0xffffffffu, mt[g], o));
    float alpha[GP], mg = -INFINITY, ag = 0.0f;
#pragma unroll
    for (int g = 0; g < GP; g++) {
      const float mn = fmaxf(m_run[g], mt[g]);
      alpha[g] = m_run[g] == -INFINITY ? 0.0f : expf(m_run[g] - mn);
      m_run[g] = mn;
      if (g == lane % GP) { mg = mn; ag = alpha[g]; }
    }
    __syncwarp();
    float ls = 0.0f;
#pragma unroll
    for (int e = lane; e < TPW * GP; e += 32) {
      const float sv = pw[e];
      const float p = sv == -INFINITY ? 0.0f : expf(sv - mg);
      pw[e] = p;
      ls += p;
    }
#pragma unroll
    for (int o = GP; o < 32; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    l_lane = l_lane * ag + ls;
#pragma unroll
    for (int g = 0; g < GP; g++)
#pragma unroll
      for (int j = 0; j < VD; j++) acc[g][j] *= alpha[g];
    __syncwarp();
#pragma unroll 4
    for (int jl = 0; jl < TPW; jl++) {
      const int j = warp * TPW + jl;
      if (j >= n) break;
      float v[VD];
      load_vals<F16, VD>(Vs + j * Gm::ROW + lane * VD * Gm::ES, v);
      float p[GP];
#pragma unroll
      for (int g = 0; g < GP; g++) p[g] = pw[jl * GP + g];
#pragma unroll
      for (int g = 0; g < GP; g++)
#pragma unroll
        for (int e = 0; e < VD; e++) acc[g][e] = fmaf(p[g], v[e], acc[g][e]);
    }
    __syncthreads();
    if (tid == 0 && k + kStages < sl.nt) {
      fence_proxy_async();
      const int64_t t1 = sl.s0 + (int64_t)(k + kStages) * TP;
      const int n1 = (int)(sl.s1 - t1 < TP ? sl.s1 - t1 : TP);
      issue_tile<HD, F16>(a.kv, layer, Ks, &bars[st], t1, n1, h);
    }
  }
  if (!ok) {
    if (a.err) atomicOr(a.err, kErrAttnWait);
    for (int k = sl.nt > kStages ? sl.nt - kStages : 0; k < sl.nt; k++)
      mbar_wait_bounded(&bars[k % kStages], ((par >> (k % kStages)) & 1u) ^ (uint32_t)((k / kStages) & 1));
  }
  __syncthreads();
  if (tid == 0) {  // parity of the next use of each stage
    uint32_t np = par;
    for (int st = 0; st < kStages; st++)
      if (sl.nt > st && (((sl.nt - st + kStages - 1) / kStages) & 1)) np ^= 1u << st;
    *par_s = np;
  }
  // Warp merge into this split's partial (in the idle ring), then to global.
  float *acc_w = (float *)ring;             // [W][GP][HD]
  float *m_w = acc_w + kMW * GP * HD;       // [W][GP]
  float *l_w = m_w + kMW * GP;              // [W][GP]
#pragma unroll
  for (int g = 0; g < GP; g++)
#pragma unroll
    for (int j = 0; j < VD; j++) acc_w[(warp * GP + g) * HD + lane * VD + j] = acc[g][j];
  if (lane < GP) {
    float mm = -INFINITY;
#pragma unroll
    for (int g = 0; g < GP; g++)
      if (g == lane) mm = m_run[g];
    m_w[warp * GP + lane] = mm;
    l_w[warp * GP + lane] = l_lane;
  }
  __syncthreads();
  constexpr int PSTR = GP * HD + 2 * GP;  // acc[GP][HD], m[GP], l[GP]
  float *mine = a.attn_part + (size_t)(h * S + sl.si) * PSTR;
  if (tid < GP) {
    float M = -INFINITY;
    for (int w = 0; w < kMW; w++) M = fmaxf(M, m_w[w * GP + tid]);
    float l = 0.0f;
    for (int w = 0; w < kMW; w++) {
      const float mw = m_w[w * GP + tid];
      const float wt = mw == -INFINITY ? 0.0f : expf(mw - M);
      wm_s[w * GP + tid] = wt;
      l = fmaf(wt, l_w[w * GP + tid], l);
    }
    mine[GP * HD + tid] = M;
    mine[GP * HD + GP + tid] = l;
  }
  __syncthreads();
  for (int i = tid; i < GP * HD; i += kMT) {
    const int g = i / HD;
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kMW; w++) s = fmaf(wm_s[w * GP + g], acc_w[(w * GP) * HD + i], s);
    mine[i] = s;
  }
  // The last split of this head to finish merges all splits in split order.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    *flag_s = atomicAdd(&a.head_cnt[h], 1u) == (unsigned)(S - 1);
  }
  __syncthreads();
  if (!*flag_s) return;
  __threadfence();
  const float *allp = a.attn_part + (size_t)h * S * PSTR;
  float *mw = wm_s;  // [S][GP] merge weights (S <= 64)
  if (tid < GP) {
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, __ldcg(allp + (size_t)s * PSTR + GP * HD + tid));
    float dsum = 0.0f;
    for (int s = 0; s < S; s++) {
      const float ms = __ldcg(allp + (size_t)s * PSTR + GP * HD + tid);
      const float w = ms == -INFINITY ? 0.0f : expf(ms - M);
      mw[s * GP + tid] = w;
      dsum = fmaf(w, __ldcg(allp + (size_t)s * PSTR + GP * HD + GP + tid), dsum);
    }
    den[tid] = dsum;
  }
  __syncthreads();
  // Warp w finalises 32-blocks w, w + kMW, ... of the head group and
  // quantizes them (QuantizedActQ8; head boundaries are 32-aligned).
  for (int bi = warp; bi < G * HD / 32; bi += kMW) {
    const int e = bi * 32 + lane, g = e / HD;
    float num = 0.0f;
    for (int s = 0; s < S; s++) num = fmaf(mw[s * GP + g], __ldcg(allp + (size_t)s * PSTR + e), num);
    float o = den[g] > 0.0f ? __fdiv_rn(num, den[g]) : 0.0f;
    a.attn[(int64_t)h * G * HD + e] = o;
    if (!isfinite(o)) o = 0.0f;
    const float amax = warp_max(fabsf(o));
    const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
    const int64_t gb = ((int64_t)h * G * HD) / 32 + bi;
    a.attn_q[gb * 32 + lane] = act_quant_one(o, inv);
    if (lane == 0) a.attn_s[gb] = scale;
  }
  if (tid == 0) a.head_cnt[h] = 0u;
}

__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Greedy argmax over this CTA's logits rows, then over all CTAs (the last
// CTA to arrive); lowest index wins ties, NaN counts as -inf.
__device__ __noinline__ void argmax_phase(const MegaArgs &a, float *red) {
  int64_t r0, cnt;
  cta_rows(a.V, r0, cnt);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < cnt; i += kMT) {
    float v = a.logits[r0 + i];
    if (v != v) v = -INFINITY;
    if (am_better(v, (int)(r0 + i), bv, bi)) { bv = v; bi = (int)(r0 + i); }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  float *sv = red;
  int *si = (int *)(red + 16);
  __shared__ int last;
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < kMW; k++)
      if (am_better(sv[k], si[k], bv, bi)) { bv = sv[k]; bi = si[k]; }
    a.am_val[blockIdx.x] = bv;
    a.am_idx[blockIdx.x] = bi;
    __threadfence();
    last = atomicAdd(a.am_cnt, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  float fv = -INFINITY;
  int fi = 0x7fffffff;
  for (unsigned k = 0; k < gridDim.x; k++) {
    const float v = __ldcg(a.am_val + k);
    const int i = __ldcg(a.am_idx + k);
    if (am_better(v, i, fv, fi)) { fv = v; fi = i; }
  }
  const uint32_t tok = (uint32_t)(fi == 0x7fffffff ? 0 : fi);
  *a.d_token = tok;
  if (a.d_hist) a.d_hist[*a.d_pos + 1] = tok;
  *a.d_pos += 1;
  *a.am_cnt = 0u;
}

// ---- phases.  Each is a separate function that reads its arguments from
// the MegaArgs block in global memory, so that the kernel's own loop keeps
// almost nothing live across the calls (a call preserves the caller's live
// registers, which otherwise costs spills in every phase).

__device__ __noinline__ void ph_embed(const MegaArgs &a) {
  const int64_t H = a.H;
  const uint32_t tok = *a.d_token;
  const int64_t per = (H + gridDim.x - 1) / gridDim.x, e0 = blockIdx.x * per;
  const int64_t e1 = e0 + per < H ? e0 + per : H;
  const bool bad = tok >= (uint32_t)a.emb_rows;
  if (bad && blockIdx.x == 0 && threadIdx.x == 0 && a.err) atomicOr(a.err, 1);
  for (int64_t i = e0 + threadIdx.x; i < e1; i += kMT)
    a.hidden[i] = bad ? 0.0f : embed_value(a.emb, a.emb_quant, H, tok, i);
  const int64_t HD = a.kv.head_dim;
  prefetch_rows(a.layers[0].qkv, (a.n_heads_q + 2 * a.n_kv) * HD, 1, 0);
}

// Q/K/V projection (RMSNorm prologue); then this CTA's first KV tile copies
// and the L2 prefetch of its O-projection rows.
template <int HD, bool F16>
__device__ __noinline__ void ph_qkv(const MegaArgs &a, int l, char *smem, float *red, uint64_t *bars) {
  const MegaLayer &L = a.layers[l];
  const int64_t QKV = (a.n_heads_q + 2 * a.n_kv) * HD;
  GemvArgs g;
  g.w = L.qkv; g.rows = QKV; g.m = 1; g.in_mode = GEMV_IN_NORM;
  g.x = a.hidden; g.x_stride = a.H; g.norm_w = L.attn_norm; g.eps = a.eps;
  g.out_mode = GEMV_OUT_STORE; g.y = a.qkv; g.y_stride = QKV;
  gemv_run(g, smem, red);
  attn_issue<HD, F16>(a, l, smem, bars);
  prefetch_rows(L.wo, a.H, 1, 0);
}

template <int HD, bool F16, int GP>
__device__ __noinline__ void ph_attn(const MegaArgs &a, int l, char *smem, uint64_t *bars, uint32_t *par_s) {
  const MegaLayer &L = a.layers[l];
  attn_phase<HD, F16, GP>(a, L, l, smem, bars, par_s);
  prefetch_rows(L.gateup, a.F, 2, a.F);
}

// O projection + residual (+ bias).
__device__ __noinline__ void ph_o(const MegaArgs &a, int l, char *smem, float *red) {
  const MegaLayer &L = a.layers[l];
  const int64_t Q = a.n_heads_q * a.kv.head_dim;
  GemvArgs g;
  g.w = L.wo; g.rows = a.H; g.m = 1; g.in_mode = GEMV_IN_Q8;
  g.xq = a.attn_q; g.xs = a.attn_s; g.xq_stride = Q;
  g.out_mode = GEMV_OUT_ADD; g.y = a.hidden; g.y_stride = a.H; g.bias = L.bo;
  gemv_run(g, smem, red);
  prefetch_rows(L.wdown, a.H, 1, 0);
}

// gate/up projection + SwiGLU (RMSNorm prologue).
__device__ __noinline__ void ph_gateup(const MegaArgs &a, int l, char *smem, float *red) {
  const MegaLayer &L = a.layers[l];
  GemvArgs g;
  g.w = L.gateup; g.rows = a.F; g.m = 1; g.in_mode = GEMV_IN_NORM;
  g.x = a.hidden; g.x_stride = a.H; g.norm_w = L.ffn_norm; g.eps = a.eps;
  g.out_mode = GEMV_OUT_SWIGLU; g.y = a.ffn; g.y_stride = a.F; g.up_offset = a.F;
  gemv_run(g, smem, red);
  if (l + 1 < a.n_layers) prefetch_rows(a.layers[l + 1].qkv, (a.n_heads_q + 2 * a.n_kv) * a.kv.head_dim, 1, 0);
  else prefetch_rows(a.lm_head, a.V, 1, 0);
}

// down projection + residual.
__device__ __noinline__ void ph_down(const MegaArgs &a, int l, char *smem, float *red) {
  const MegaLayer &L = a.layers[l];
  GemvArgs g;
  g.w = L.wdown; g.rows = a.H; g.m = 1; g.in_mode = GEMV_IN_F32;
  g.x = a.ffn; g.x_stride = a.F;
  g.out_mode = GEMV_OUT_ADD; g.y = a.hidden; g.y_stride = a.H;
  gemv_run(g, smem, red);
  if (l + 1 < a.n_layers) prefetch_rows(a.layers[l + 1].wo, a.H, 1, 0);
}

// LM head (final RMSNorm prologue).
__device__ __noinline__ void ph_head(const MegaArgs &a, char *smem, float *red) {
  GemvArgs g;
  g.w = a.lm_head; g.rows = a.V; g.m = 1; g.in_mode = GEMV_IN_NORM;
  g.x = a.hidden; g.x_stride = a.H; g.norm_w = a.out_norm; g.eps = a.eps;
  g.out_mode = GEMV_OUT_STORE; g.y = a.logits; g.y_stride = a.V;
  gemv_run(g, smem, red);
}

template <int HD, bool F16, int GP>
__global__ void __launch_bounds__(kMT, 1) k_decode_mega(const MegaArgs *__restrict__ ap) {
  extern __shared__ __align__(128) char smem[];
  __shared__ float red[33];
  __shared__ __align__(8) uint64_t bars[kStages];
  __shared__ uint32_t par_s;
  __shared__ int broken;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) mbar_init(&bars[s], 1);
    fence_barrier_init();
    fence_proxy_async();
    par_s = 0;
    broken = 0;
  }
  __syncthreads();
  const MegaArgs &a = *ap;
  ph_embed(a);
  grid_sync(a.bar, a.err, &broken);
  const int n_layers = a.n_layers;
  for (int l = 0; l < n_layers; l++) {
    ph_qkv<HD, F16>(a, l, smem, red, bars);
    grid_sync(a.bar, a.err, &broken);
    ph_attn<HD, F16, GP>(a, l, smem, bars, &par_s);
    grid_sync(a.bar, a.err, &broken);
    ph_o(a, l, smem, red);
    grid_sync(a.bar, a.err, &broken);
    ph_gateup(a, l, smem, red);
    grid_sync(a.bar, a.err, &broken);
    ph_down(a, l, smem, red);
    grid_sync(a.bar, a.err, &broken);
  }
  ph_head(a, smem, red);
  argmax_phase(a, red);
}

template <int HD, bool F16, int GP>
const void *mega_fn() {
  return (const void *)k_decode_mega<HD, F16, GP>;
}

const void *pick_mega(int hd, int f16, int G) {
  const int gp = G <= 4 ? 4 : 0;
  if (hd == 128 && f16 && gp == 4) return mega_fn<128, true, 4>();
  if (hd == 128 && !f16 && gp == 4) return mega_fn<128, false, 4>();
  if (hd == 64 && f16 && gp == 4) return mega_fn<64, true, 4>();
  if (hd == 64 && !f16 && gp == 4) return mega_fn<64, false, 4>();
  return nullptr;
}

// Shared memory of one projection phase: activation region, plus the
// per-segment partials when the input spans several segments.
size_t proj_smem(int in_mode, int64_t cols, int64_t rows, int grid) {
  const int nb = (int)(cols / 32), nseg = seg_count(cols);
  return w4_smem(in_mode, nb, nseg, (rows + grid - 1) / grid);
}

size_t mega_smem(const MegaArgs &a, int grid) {
  const int64_t Q = a.n_heads_q * a.kv.head_dim, KV = a.n_kv * a.kv.head_dim;
  size_t m = (size_t)kStages * kStageBytes + kAttnWs;
  const size_t p[5] = {proj_smem(GEMV_IN_NORM, a.H, Q + 2 * KV, grid), proj_smem(GEMV_IN_Q8, Q, a.H, grid),
                       proj_smem(GEMV_IN_NORM, a.H, a.F, grid), proj_smem(GEMV_IN_F32, a.F, a.H, grid),
                       proj_smem(GEMV_IN_NORM, a.H, a.V, grid)};
  for (size_t v : p)
    if (v > m) m = v;
  return m;
}

}  // namespace

int mega_check(const MegaArgs &a, int grid) {
  if (grid < 1 || a.n_kv < 1 || a.n_heads_q % a.n_kv) return 0;
  if (!pick_mega((int)a.kv.head_dim, a.kv.f16, (int)(a.n_heads_q / a.n_kv))) return 0;
  // SwiGLU pairs need the whole gate/up row in one segment; other inputs
  // may span up to 16 segments (one warp each).
  if (seg_count(a.H) != 1) return 0;
  if (a.splits < 1 || a.splits > 64 || a.n_kv * a.splits > grid) return 0;
  return mega_smem(a, grid) <= (size_t)kGemvMaxSmem ? 1 : 0;
}

size_t mega_part_bytes(const MegaArgs &a) {
  constexpr int GP = 4;  // query heads per KV head in every instantiation
  return (size_t)a.n_kv * a.splits * (GP * a.kv.head_dim + 2 * GP) * sizeof(float);
}

int launch_decode_mega(const MegaArgs &a, const MegaArgs *dev_args, int grid, cudaStream_t s) {
  const void *fn = pick_mega((int)a.kv.head_dim, a.kv.f16, (int)(a.n_heads_q / a.n_kv));
  if (!fn) return 0;
  if (!mega_check(a, grid)) return 0;
  const size_t smem = mega_smem(a, grid);
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kMT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {(void *)&dev_args};
  return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? 1 : 0;
}

}  // namespace jal
