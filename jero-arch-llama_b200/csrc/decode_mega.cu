// Persistent decode step (one token, fast numerics).
//
// One cooperative launch of one CTA per SM runs a whole decode token: the
// embedding, every layer's five phases (Q/K/V projection, attention, O
// projection + residual, gate/up projection + SwiGLU, down projection +
// residual) and the LM head with greedy argmax.  Phases are separated by a
// grid barrier instead of kernel boundaries.
//
// Weight streaming.  Every byte a CTA reads from HBM in the step is known
// when the step starts: its contiguous row slice of each projection (the
// row-interleaved layout makes a row range one byte range) and the KV-cache
// tiles of its attention slice (positions before the current one).  Thread 0
// walks that sequence (the CTA's "stream": layer by layer Q/K/V rows, KV
// tiles, O rows, gate and up rows in pairs, down rows; then LM head rows)
// and keeps it flowing through a ring of kSlots x 32 KB shared-memory slots
// with bulk copies (cp.async.bulk, one mbarrier per slot).  The warps
// consume the slots in stream order and thread 0 refills each slot with the
// chunk kSlots ahead as soon as it is released, so HBM keeps streaming
// through grid barriers, activation prologues and attention, up to the
// ring's depth (bulk copies of >= 16 KB kept 4+ deep per SM sustain the
// full HBM rate).
//
// Projection phases: the activation (QuantizedActQ8 per 32-block, RMSNorm
// first where the layer has one) is formed in the work area of shared memory
// and held in registers per warp (warp w takes 128-block segment w % nseg of
// every row, lane l blocks l, l + 32, l + 64, l + 96 of the segment, so the
// shared-memory reads of a row are conflict-free); the weight rows come from
// the ring.  Attention: each KV head is split over up to `splits` CTAs (one
// split per attn_split_tokens attended positions); a CTA consumes its tiles
// from the ring, and with several splits the last CTA of a head to finish
// merges the partials in split order.  The gate/up phase also writes the
// SwiGLU row as QuantizedActQ8 (the CTA completing a 32-block quantizes
// it), which the down projection reads directly.
//
// Every wait is bounded: a grid barrier that gives up sets bit 8 of the
// context error word (a ring wait bit 2) and later barriers stop waiting, so
// the kernel always finishes.
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
constexpr int kErrRingWait = 2, kErrGridWait = 8;
constexpr int kSlots = 6;
constexpr int kSlotBytes = kStageBytes;  // 32 KB: one KV tile (K then V) or whole weight rows
constexpr size_t kRingBytes = (size_t)kSlots * kSlotBytes;
constexpr size_t kWorkBytes = 25 * 1024;  // activation / attention workspace after the ring
constexpr int kMaxLayers = 64;

// Dynamic shared memory: the ring, then the work area.  Functions address it
// through these file-scope symbols (not through pointer parameters) so that
// every access compiles to a shared-memory instruction.
extern __shared__ __align__(128) char mega_dsmem[];
__shared__ float mega_red[33];
__shared__ unsigned mega_done[kSlots];  // warps done with the chunk in each slot
__device__ __forceinline__ char *work_area() { return mega_dsmem + kRingBytes; }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Barrier over all CTAs of the cooperative grid: bar[0] counts arrivals
// over the whole launch (one per CTA per barrier) and barrier k completes
// when it reaches k * gridDim.x, so an arrival is a single atomic and the
// waiters poll one word.  The last CTA of the argmax phase returns the
// counter to zero.  A wait that gives up sets bit 8 of the error word and
// this CTA stops waiting at later barriers (*broken), still arriving at each
// so the count stays consistent.
struct GridBar {
  unsigned *bar;
  int *err;
  int *broken;
  unsigned *seq;  // barriers passed by this CTA (shared)
};

__device__ __noinline__ void grid_sync(const GridBar &g) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned k = *g.seq + 1;
    *g.seq = k;
    const unsigned target = k * gridDim.x;
    __threadfence();
    atomicAdd(g.bar, 1u);
    if (!*g.broken) {
      uint32_t it = 0;
      while (ld_acquire(g.bar) < target) {
        if (++it > kGridSpin) {
          *g.broken = 1;
          if (g.err) atomicOr(g.err, kErrGridWait);
          break;
        }
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

// Attention work of this CTA: KV head h, split si of S (S <= a.splits grows
// with the attended span, one split per attn_split_tokens positions), tiles
// of tp positions.
struct Slice {
  int h, si, S;
  int64_t pos, s0, s1;
  int nt;
  bool active;
};

__device__ __forceinline__ Slice attn_slice(const MegaArgs &a, int64_t pos, int tp) {
  Slice s;
  const int c = blockIdx.x;
  s.h = c / a.splits;
  s.si = c % a.splits;
  s.pos = pos;
  const int64_t seq = pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int64_t span = seq - lo, st = a.attn_split_tokens > 0 ? a.attn_split_tokens : 1;
  int64_t se = (span + st - 1) / st;
  se = se < 1 ? 1 : (se > a.splits ? a.splits : se);
  s.S = (int)se;
  s.active = c < a.n_kv * a.splits && s.si < s.S;
  const int64_t per = (span + s.S - 1) / s.S;
  s.s0 = lo + s.si * per;
  s.s1 = s.s0 + per < seq ? s.s0 + per : seq;
  const int64_t len = s.s1 > s.s0 ? s.s1 - s.s0 : 0;
  s.nt = s.active ? (int)((len + tp - 1) / tp) : 0;
  return s;
}

// ---- the CTA's stream ----------------------------------------------------
// A row slice of one projection, cut into chunks of rpc whole rows.
struct Rows {
  int64_t r0, cnt;
  int rpc, n;
};

__device__ __forceinline__ Rows make_rows(int64_t rows, int64_t qs_stride) {
  Rows r;
  cta_rows(rows, r.r0, r.cnt);
  const int64_t rpc = kSlotBytes / qs_stride;
  r.rpc = (int)(rpc < 1 ? 1 : rpc);
  r.n = (int)((r.cnt + r.rpc - 1) / r.rpc);
  return r;
}

// Per-CTA stream layout, computed once per launch (shared memory), with
// everything thread 0 needs to issue any chunk without touching global
// memory (except the KV page table).
struct Plan {
  int64_t pos;
  Slice sl;
  Rows q, o, gu, dn, head;  // gu: gate rows (its chunks come in gate/up pairs)
  int per_layer, total;     // chunks per layer; chunks in the launch
  int n_layers;
  int64_t up_offset;        // rows from a gate row to its up row (F)
  int64_t st[5];            // row bytes: Q/K/V, O, gate/up, down, LM head
  const uint8_t *head_qs;
  KvView kv;
  const uint8_t *qs[kMaxLayers][4];  // per layer: Q/K/V, O, gate/up, down
};

// All threads: the per-layer weight table; then thread 0 the rest.
__device__ __forceinline__ void make_plan(const MegaArgs &a, int64_t pos, int tp, Plan &p) {
  for (int i = threadIdx.x; i < a.n_layers * 4; i += kMT) {
    const MegaLayer &L = a.layers[i / 4];
    const int k = i % 4;
    p.qs[i / 4][k] = k == 0 ? L.qkv.qs : k == 1 ? L.wo.qs : k == 2 ? L.gateup.qs : L.wdown.qs;
  }
  if (threadIdx.x != 0) return;
  const int64_t HD = a.kv.head_dim, QKV = (a.n_heads_q + 2 * a.n_kv) * HD;
  const MegaLayer &L0 = a.layers[0];
  p.pos = pos;
  p.sl = attn_slice(a, pos, tp);
  p.st[0] = L0.qkv.qs_stride;
  p.st[1] = L0.wo.qs_stride;
  p.st[2] = L0.gateup.qs_stride;
  p.st[3] = L0.wdown.qs_stride;
  p.st[4] = a.lm_head.qs_stride;
  p.q = make_rows(QKV, p.st[0]);
  p.o = make_rows(a.H, p.st[1]);
  p.gu = make_rows(a.F, p.st[2]);
  p.dn = make_rows(a.H, p.st[3]);
  p.head = make_rows(a.V, p.st[4]);
  p.per_layer = p.q.n + p.sl.nt + p.o.n + 2 * p.gu.n + p.dn.n;
  p.n_layers = a.n_layers;
  p.total = a.n_layers * p.per_layer + p.head.n;
  p.up_offset = a.F;
  p.head_qs = a.lm_head.qs;
  p.kv = a.kv;
}

struct Ring {
  uint64_t *full;  // [kSlots] one mbarrier per slot (completes when its bytes land)
};

__device__ __forceinline__ char *slot_ptr(unsigned j) { return mega_dsmem + (j % kSlots) * kSlotBytes; }

__device__ __forceinline__ void issue_rows(const uint8_t *qs, int64_t stride, const Rows &rs, int i, int64_t row_offset,
                                           char *dst, uint64_t *bar) {
  const int64_t first = rs.r0 + (int64_t)i * rs.rpc;
  const int64_t n = rs.cnt - (int64_t)i * rs.rpc < rs.rpc ? rs.cnt - (int64_t)i * rs.rpc : rs.rpc;
  const uint32_t bytes = (uint32_t)(n * stride);
  mbar_expect_tx(bar, bytes);
  bulk_g2s(dst, qs + (first + row_offset) * stride, bytes, bar);
}

// KV tile o of layer l (several bulk copies when the tile spans pages).
template <int HD, bool F16>
__device__ __noinline__ void issue_kv(const Plan &p, char *dst, uint64_t *bar, int l, int o) {
  using Gm = AttnGeom<HD, F16, 1>;
  const int64_t t0 = p.sl.s0 + (int64_t)o * Gm::TP;
  const int n = (int)(p.sl.s1 - t0 < Gm::TP ? p.sl.s1 - t0 : Gm::TP);
  issue_tile<HD, F16>(p.kv, l, dst, bar, t0, n, p.sl.h);
}

// One thread: copy stream chunk j into its slot (nothing past the end).
template <int HD, bool F16>
__device__ __forceinline__ void ring_issue(const Plan &p, const Ring &r, unsigned j) {
  if ((int)j >= p.total) return;
  char *dst = slot_ptr(j);
  uint64_t *bar = &r.full[j % kSlots];
  const int lay_chunks = p.n_layers * p.per_layer;
  if ((int)j >= lay_chunks) {
    issue_rows(p.head_qs, p.st[4], p.head, (int)j - lay_chunks, 0, dst, bar);
    return;
  }
  const int l = (int)j / p.per_layer;
  int o = (int)j - l * p.per_layer;
  if (o < p.q.n) { issue_rows(p.qs[l][0], p.st[0], p.q, o, 0, dst, bar); return; }
  o -= p.q.n;
  if (o < p.sl.nt) { issue_kv<HD, F16>(p, dst, bar, l, o); return; }
  o -= p.sl.nt;
  if (o < p.o.n) { issue_rows(p.qs[l][1], p.st[1], p.o, o, 0, dst, bar); return; }
  o -= p.o.n;
  if (o < 2 * p.gu.n) { issue_rows(p.qs[l][2], p.st[2], p.gu, o / 2, (o & 1) ? p.up_offset : 0, dst, bar); return; }
  o -= 2 * p.gu.n;
  issue_rows(p.qs[l][3], p.st[3], p.dn, o, 0, dst, bar);
}

// All threads: wait until stream chunk j has landed.
__device__ __forceinline__ void ring_wait(const Ring &r, unsigned j, int *err) {
  if (!mbar_wait_bounded(&r.full[j % kSlots], (j / kSlots) & 1u) && err) atomicOr(err, kErrRingWait);
}

// After every thread is done with chunk j (the caller synchronises), one
// thread refills its slot with chunk j + kSlots: lane 0 of the last warp,
// which has the fewest rows of a chunk.  `wrote`: the slot was also written
// through the generic proxy, which must be ordered before the async-proxy
// refill.
constexpr int kProducer = (kMW - 1) * 32;
template <int HD, bool F16>
__device__ __forceinline__ void ring_release(const Plan &p, const Ring &r, unsigned j, bool wrote) {
  if (threadIdx.x == kProducer) {
    if (wrote) fence_proxy_async();
    ring_issue<HD, F16>(p, r, j + kSlots);
  }
}

// ---- projection phases -----------------------------------------------------
// SwiGLU rows [r0, r0 + cnt) of this CTA are in a.y.  Each 32-block they
// touch gets this CTA's row count added to its counter; the CTA that brings
// a block to 32 quantizes it (QuantizedActQ8, the same values the consumer
// would compute from the f32 row) and clears the counter.
__device__ __forceinline__ void quantize_done_blocks(const float *y, int8_t *yq, float *ys, unsigned *ycnt, int64_t r0,
                                                    int64_t cnt) {
  __shared__ int done_s[kMW];
  if (cnt <= 0) return;  // CTA-uniform
  const int64_t b0 = r0 / 32, b1 = (r0 + cnt - 1) / 32;
  __threadfence();  // this thread's rows are visible before the counters move
  __syncthreads();
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int64_t bb = b0; bb <= b1; bb += kMW) {
    if (threadIdx.x < kMW) {
      const int64_t b = bb + threadIdx.x;
      int done = 0;
      if (b <= b1) {
        const int64_t lo = r0 > b * 32 ? r0 : b * 32;
        const int64_t hi = r0 + cnt < b * 32 + 32 ? r0 + cnt : b * 32 + 32;
        const unsigned n = (unsigned)(hi - lo);
        done = atomicAdd(&ycnt[b], n) + n == 32u;
      }
      done_s[threadIdx.x] = done;
    }
    __syncthreads();
    const int64_t b = bb + w;
    if (b <= b1 && done_s[w]) {
      __threadfence();
      float v = __ldcg(y + b * 32 + lane);
      if (!isfinite(v)) v = 0.0f;
      const float amax = warp_max(fabsf(v));
      const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
      yq[b * 32 + lane] = act_quant_one(v, inv);
      if (lane == 0) {
        ys[b] = scale;
        ycnt[b] = 0u;
      }
    }
    __syncthreads();
  }
}


// GEMV_IN_PREQ prologue: the block-quantized (row x norm weights) and its
// scales go to shared memory like a Q8 input; warp 0 sums the producers'
// partial sums of squares (fixed order) for the norm scale, returned to
// every thread.
__device__ __forceinline__ float prologue_preq(const GemvArgs &g, char *smem, int nb, int nbp, float *red) {
  const int tid = threadIdx.x;
  if (tid < 32) {
    float ss = 0.0f;
    for (int i = tid; i < g.ss_n; i += 32) ss += __ldcg(g.ss_part + i);
    ss = warp_sum(ss);
    if (tid == 0) red[32] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)(nb * 32)), g.eps)));
  }
  for (int b = nb + tid; b < nbp; b += kMT) {
    ((uint4 *)smem)[b] = make_uint4(0, 0, 0, 0);
    ((uint4 *)(smem + nbp * 16))[b] = make_uint4(0, 0, 0, 0);
    put_scale_sum(smem, nbp, b, 0.0f, 0);
  }
  for (int b = tid; b < nb; b += kMT) {
    const int4 *q = (const int4 *)(g.xq + (size_t)b * 32);
    const int4 lo = __ldcg(q), hi = __ldcg(q + 1);
    const float sc = __ldcg(g.xs + b);
    int s = dp4a_ss(lo.x, 0x01010101, 0);
    s = dp4a_ss(lo.y, 0x01010101, s);
    s = dp4a_ss(lo.z, 0x01010101, s);
    s = dp4a_ss(lo.w, 0x01010101, s);
    s = dp4a_ss(hi.x, 0x01010101, s);
    s = dp4a_ss(hi.y, 0x01010101, s);
    s = dp4a_ss(hi.z, 0x01010101, s);
    s = dp4a_ss(hi.w, 0x01010101, s);
    ((int4 *)smem)[b] = lo;
    ((int4 *)(smem + nbp * 16))[b] = hi;
    put_scale_sum(smem, nbp, b, sc, s);
  }
  __syncthreads();
  return red[32];
}

// The finished hidden rows [r0, r0 + cnt) of this CTA (rows[i]) become the
// next RMSNorm input: u = row x norm weights, block-quantized by the CTA
// completing each 32-block, and this CTA's sum of squares of the rows.
__device__ __forceinline__ void next_norm_input(const float *norm, float *u, int8_t *q, float *s, unsigned *cnt_b,
                                                float *ss_out, const float *rows, int64_t r0, int64_t cnt) {
  __syncthreads();  // every row of the slice is final
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < cnt; i += kMT) {
    const float h = rows[i];
    ss = fmaf(h, h, ss);
    u[r0 + i] = __fmul_rn(h, norm[r0 + i]);
  }
  const float tot = block_reduce_sum<kMW>(ss, mega_red);
  if (threadIdx.x == 0) ss_out[blockIdx.x] = tot;
  quantize_done_blocks(u, q, s, cnt_b, r0, cnt);
}

// One projection over this CTA's row slice, weights from the ring.  j is the
// stream index of the phase's first chunk; returns the index after its last.
template <int QUANT, int HD, bool F16>
__device__ __forceinline__ unsigned gemv_stream(const MegaArgs &a, const Plan &p, const Ring &r, const GemvArgs &g,
                                             const Rows &rs, unsigned j) {
  char *work = work_area();
  float *red = mega_red;
  const int nb = (int)(g.w.cols / 32), nseg = seg_count(g.w.cols), nbp = nseg * kSegBlocks;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int seg = warp % nseg, phase = warp / nseg, nph = kMW / nseg;
  const bool swiglu = g.out_mode == GEMV_OUT_SWIGLU;
  if (g.out_mode == GEMV_OUT_ADD) {  // residual rows of this CTA, read once (visible after the prologue's barrier)
    float *yb = (float *)(work + w4_act_region(g.in_mode, nb, nseg)) + kSlots * rs.rpc * nseg;
    for (int i = threadIdx.x; i < rs.cnt; i += kMT) yb[i] = g.y[rs.r0 + i];
  }
  float invn = 1.0f;  // norm scale folded into the block scales (GEMV_IN_PREQ)
  if (g.in_mode == GEMV_IN_PREQ) {
    invn = prologue_preq(g, work, nb, nbp, red);
  } else if (g.in_mode == GEMV_IN_NORM && nb * 4 <= 4 * kMT) {
    prologue_m1_impl<kMW, 4, true>(g, work, nb, nbp, red);
  } else {
    gemv_prologue_pre<1, kMW>(g, work, nb, nbp);
    gemv_prologue<1, kMW>(g, work, nb, nbp, red);
  }
  int bq[4];
  unsigned vmask = 0;
#pragma unroll
  for (int v = 0; v < 4; v++) {
    const int b = seg * kSegBlocks + lane + 32 * v;
    bq[v] = b < nb ? b : 0;
    vmask |= (b < nb ? 1u : 0u) << v;
  }
  W4Act x;
#pragma unroll
  for (int v = 0; v < 4; v++) {
    const int b = seg * kSegBlocks + lane + 32 * v;  // < nbp; padding blocks are zero
    x.lo[v] = ((const int4 *)work)[b];
    x.hi[v] = ((const int4 *)(work + nbp * 16))[b];
    const float2 ss = ((const float2 *)(work + nbp * 32))[b];
    x.sc[v] = g.in_mode == GEMV_IN_PREQ ? __fmul_rn(ss.x, invn) : ss.x;
    x.sum[v] = __float_as_int(ss.y);
  }
  float *part = (float *)(work + w4_act_region(g.in_mode, nb, nseg));  // [kSlots][rpc][nseg]
  const int64_t qs = g.w.qs_stride, r0 = rs.r0, cnt = rs.cnt;
  const int rpc = rs.rpc, nch = rs.n;
  const bool add = g.out_mode == GEMV_OUT_ADD;
  float *y = g.y, *ybase = part + kSlots * rpc * nseg;  // ybase: [cnt] residual of this CTA's rows
  const float *bias = g.bias;
  uint64_t *full = r.full;
  int *err = a.err;
  // output row i of this CTA: y + bias (ADD) or bias (STORE) added to the dot
  auto finish = [&](int64_t i, float s) -> float {
    if (!add) return bias ? s + bias[r0 + i] : s;
    const float v = ybase[i] + (bias ? s + bias[r0 + i] : s);
    ybase[i] = v;  // the finished row, for the next RMSNorm input
    return v;
  };
  // Warps run through the chunks independently: each takes the rows of its
  // 128-block segment whose index in the CTA's slice is congruent to its
  // phase (balanced over the whole slice), then counts itself done with the
  // chunk; the last warp to finish a chunk combines the segment partials (in
  // segment order) and refills the chunk's slot.
  for (int c = 0; c < nch; c++) {
    const int64_t first = (int64_t)c * rpc;  // first row of the chunk, relative to r0
    const int n = (int)(cnt - first < rpc ? cnt - first : rpc);
    if (!mbar_wait_bounded(&full[j % kSlots], (j / kSlots) & 1u) && err) atomicOr(err, kErrRingWait);
    if (swiglu && !mbar_wait_bounded(&full[(j + 1) % kSlots], ((j + 1) / kSlots) & 1u) && err)
      atomicOr(err, kErrRingWait);
    const char *wg = slot_ptr(j);
    const char *wu = slot_ptr(j + 1);
    float *pslot = part + (j % kSlots) * rpc * nseg;  // [rpc][nseg]
    if (phase < nph) {
      int lr = (int)((phase - (int)(first % nph) + nph) % nph);
      if (swiglu) {
        for (; lr < n; lr += nph) {
          W4Row<QUANT> wa, wb;
          w4s_load<QUANT>(wg + (size_t)lr * qs, nb, bq, vmask, wa);
          w4s_load<QUANT>(wu + (size_t)lr * qs, nb, bq, vmask, wb);
          float sa = w4_dot<QUANT>(wa, x), sb = w4_dot<QUANT>(wb, x);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            sa += __shfl_xor_sync(0xffffffffu, sa, o);
            sb += __shfl_xor_sync(0xffffffffu, sb, o);
          }
          if (lane == 0) y[r0 + first + lr] = swiglu_one(sa, sb);
        }
      } else {
        for (; lr < n; lr += 2 * nph) {  // two rows at a time
          const int lr2 = lr + nph;
          const bool two = lr2 < n;
          W4Row<QUANT> wa, wb;
          w4s_load<QUANT>(wg + (size_t)lr * qs, nb, bq, vmask, wa);
          if (two) w4s_load<QUANT>(wg + (size_t)lr2 * qs, nb, bq, vmask, wb);
          float sa = w4_dot<QUANT>(wa, x), sb = two ? w4_dot<QUANT>(wb, x) : 0.0f;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            sa += __shfl_xor_sync(0xffffffffu, sa, o);
            sb += __shfl_xor_sync(0xffffffffu, sb, o);
          }
          if (lane == 0) {
            if (nseg > 1) {
              pslot[lr * nseg + seg] = sa;
              if (two) pslot[lr2 * nseg + seg] = sb;
            } else {
              y[r0 + first + lr] = finish(first + lr, sa);
              if (two) y[r0 + first + lr2] = finish(first + lr2, sb);
            }
          }
        }
      }
    }
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&mega_done[j % kSlots], 1u) == kMW - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence_block();
      if (nseg > 1 && !swiglu && lane < n) {
        float sum = 0.0f;
        for (int q = 0; q < nseg; q++) sum += pslot[lane * nseg + q];
        y[r0 + first + lane] = finish(first + lane, sum);
      }
      __syncwarp();
      if (lane == 0) {
        mega_done[j % kSlots] = 0u;
        ring_issue<HD, F16>(p, r, j + kSlots);
        if (swiglu) ring_issue<HD, F16>(p, r, j + 1 + kSlots);
      }
    }
    j += swiglu ? 2 : 1;
  }
  if (swiglu && g.yq) quantize_done_blocks(g.y, g.yq, g.ys, g.ycnt, rs.r0, rs.cnt);
  if (add && g.nx_u) next_norm_input(g.nx_norm, g.nx_u, g.nx_q, g.nx_s, g.nx_cnt, g.nx_ss, ybase, rs.r0, rs.cnt);
  __syncthreads();
  return j;
}

// ---- attention -------------------------------------------------------------
template <int HD, bool F16, int GP>
__device__ __forceinline__ unsigned attn_stream(const MegaArgs &a, const Plan &p, const Ring &r, int layer, unsigned j) {
  char *work = work_area();
  using Gm = AttnGeom<HD, F16, kMW>;
  constexpr int TP = Gm::TP, LG = Gm::LG, PPS = Gm::PPS, DPL = Gm::DPL, TPW = Gm::TPW, VD = Gm::VD;
  const Slice &sl = p.sl;
  if (!sl.active) return j;
  const MegaLayer &L = a.layers[layer];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = (int)(a.n_heads_q / a.n_kv), h = sl.h, S = a.splits;
  const int64_t Q = a.n_heads_q * HD, KVD = a.n_kv * HD, pos = sl.pos, seq = pos + 1;
  float(*q_s)[HD] = (float(*)[HD])work;                  // [GP][HD]
  float *kn_s = (float *)(work + GP * HD * 4);          // [HD]
  float *vn_s = kn_s + HD;                              // [HD]
  float *p_all = vn_s + HD;                             // [kMW][TPW * GP]
  float *wm_s = p_all + kMW * TPW * GP;                 // [64 + 1][GP]: warp, then split merge weights
  float *den = wm_s + 65 * GP;                          // [GP]
  int *flag_s = (int *)(den + GP);
  float *acc_w = (float *)(work + 8192);                // [kMW][GP][HD] warp partials
  float *m_w = acc_w + kMW * GP * HD;                   // [kMW][GP]
  float *l_w = m_w + kMW * GP;                          // [kMW][GP]
  const bool rope = !L.skip_rope && pos > 0;
  const int half = (int)(a.rotary_dim / 2);
  const bool use_long = a.long_threshold >= 0 && seq > a.long_threshold;
  const float *ct = (use_long ? a.cos_long : a.cos_tab) + pos * half;
  const float *st = (use_long ? a.sin_long : a.sin_tab) + pos * half;
  const bool own_pos = pos >= sl.s0 && pos < sl.s1;
  const int64_t app = own_pos ? kv_elem(a.kv, layer, h, pos) : 0;
  // q heads (GP rows, zero past G), then the new k and v: bias, RoPE
  // (recipe.rs:2750-2767) and, for k / v, the value the cache stores.  All
  // global loads of the pass are issued first, then the values are formed.
  constexpr int NIT = ((GP + 2) * HD + kMT - 1) / kMT;
  float xv[NIT], pv[NIT], cv[NIT], sv[NIT];
#pragma unroll
  for (int it = 0; it < NIT; it++) {
    const int i = tid + it * kMT;
    xv[it] = 0.0f; pv[it] = 0.0f; cv[it] = 1.0f; sv[it] = 0.0f;
    if (i < (GP + 2) * HD) {
      const int g = i / HD, d = i % HD;
      if (g >= GP || g < G) {
        const int64_t off = g < GP ? (int64_t)(h * G + g) * HD : (g == GP ? Q : Q + KVD) + (int64_t)h * HD;
        const float *bias = g < GP ? L.bq : (g == GP ? L.bk : L.bv);
        const int64_t boff = g < GP ? (int64_t)(h * G + g) * HD : (int64_t)h * HD;
        float o = a.qkv[off + d];
        if (bias) o = __fadd_rn(o, bias[boff + d]);
        xv[it] = o;
        if (rope && g <= GP && d < 2 * half) {
          const bool first = a.neox ? d < half : (d & 1) == 0;
          const int jj = a.neox ? (first ? d : d - half) : d / 2;
          const int partner = a.neox ? (first ? d + half : d - half) : (d ^ 1);
          float other = a.qkv[off + partner];
          if (bias) other = __fadd_rn(other, bias[boff + partner]);
          pv[it] = other;
          cv[it] = ct[jj];
          sv[it] = st[jj];
        }
      }
    }
  }
#pragma unroll
  for (int it = 0; it < NIT; it++) {
    const int i = tid + it * kMT;
    if (i >= (GP + 2) * HD) break;
    const int g = i / HD, d = i % HD;
    float o = xv[it];
    if (rope && g <= GP && d < 2 * half) {
      const bool first = a.neox ? d < half : (d & 1) == 0;
      const float other = pv[it], c = cv[it], sn = sv[it];
      const float x0 = first ? o : other, x1 = first ? other : o;
      o = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    if (g < GP) {
      q_s[g][d] = o;  // zero for g >= G
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
    for (int jj = 0; jj < VD; jj++) acc[g][jj] = 0.0f;
  }
  float *pw = p_all + warp * TPW * GP;
  for (int k = 0; k < sl.nt; k++, j++) {
    ring_wait(r, j, a.err);
    const int64_t t0 = sl.s0 + (int64_t)k * TP;
    const int n = (int)(sl.s1 - t0 < TP ? sl.s1 - t0 : TP);
    char *Ks = slot_ptr(j);
    char *Vs = Ks + TP * Gm::ROW;
    if (own_pos && pos >= t0 && pos < t0 + n) {  // the new k / v are not in the cache copy yet
      const int jp = (int)(pos - t0);
      for (int d = tid; d < HD; d += kMT) {
        if (F16) {
          ((__half *)(Ks + jp * Gm::ROW))[d] = __float2half_rn(kn_s[d]);
          ((__half *)(Vs + jp * Gm::ROW))[d] = __float2half_rn(vn_s[d]);
        } else {
          ((float *)(Ks + jp * Gm::ROW))[d] = kn_s[d];
          ((float *)(Vs + jp * Gm::ROW))[d] = vn_s[d];
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
      const int jt = warp * TPW + jl;
      float d[GP];
#pragma unroll
      for (int g = 0; g < GP; g++) d[g] = 0.0f;
      if (jt < n) {
        float kv[DPL];
        load_vals<F16, DPL>(Ks + jt * Gm::ROW + c * 16, kv);
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
        const float sc = jt < n ? __fmul_rn(d[g], a.scale) : -INFINITY;
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
      const float s = pw[e];
      const float pe = s == -INFINITY ? 0.0f : expf(s - mg);
      pw[e] = pe;
      ls += pe;
    }
#pragma unroll
    for (int o = GP; o < 32; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    l_lane = l_lane * ag + ls;
#pragma unroll
    for (int g = 0; g < GP; g++)
#pragma unroll
      for (int jj = 0; jj < VD; jj++) acc[g][jj] *= alpha[g];
    __syncwarp();
#pragma unroll 4
    for (int jl = 0; jl < TPW; jl++) {
      const int jt = warp * TPW + jl;
      if (jt >= n) break;
      float v[VD];
      load_vals<F16, VD>(Vs + jt * Gm::ROW + lane * VD * Gm::ES, v);
      float pg[GP];
#pragma unroll
      for (int g = 0; g < GP; g++) pg[g] = pw[jl * GP + g];
#pragma unroll
      for (int g = 0; g < GP; g++)
#pragma unroll
        for (int e = 0; e < VD; e++) acc[g][e] = fmaf(pg[g], v[e], acc[g][e]);
    }
    __syncthreads();
    ring_release<HD, F16>(p, r, j, own_pos);
  }
  // Warp merge of this CTA's split.
#pragma unroll
  for (int g = 0; g < GP; g++)
#pragma unroll
    for (int jj = 0; jj < VD; jj++) acc_w[(warp * GP + g) * HD + lane * VD + jj] = acc[g][jj];
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
  const int Se = sl.S;
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
    den[tid] = l;
    wm_s[64 * GP + tid] = M;
  }
  __syncthreads();
  const int64_t ob = (int64_t)h * G * HD;  // first output element of this head group
  if (Se == 1) {
    // The only split of this head: normalise and write the output directly.
    for (int bi = warp; bi < G * HD / 32; bi += kMW) {
      const int e = bi * 32 + lane, g = e / HD;
      float num = 0.0f;
#pragma unroll
      for (int w = 0; w < kMW; w++) num = fmaf(wm_s[w * GP + g], acc_w[(w * GP) * HD + e], num);
      float o = den[g] > 0.0f ? __fdiv_rn(num, den[g]) : 0.0f;
      a.attn[ob + e] = o;
      if (!isfinite(o)) o = 0.0f;
      const float amax = warp_max(fabsf(o));
      const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
      a.attn_q[ob + e] = act_quant_one(o, inv);
      if (lane == 0) a.attn_s[ob / 32 + bi] = scale;
    }
    __syncthreads();
    return j;
  }
  float *mine = a.attn_part + (size_t)(h * S + sl.si) * PSTR;
  if (tid < GP) {
    mine[GP * HD + tid] = wm_s[64 * GP + tid];
    mine[GP * HD + GP + tid] = den[tid];
  }
  for (int i = tid; i < GP * HD; i += kMT) {
    const int g = i / HD;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kMW; w++) v = fmaf(wm_s[w * GP + g], acc_w[(w * GP) * HD + i], v);
    mine[i] = v;
  }
  // The last split of this head to finish merges all splits in split order.
  __threadfence();
  __syncthreads();
  if (tid == 0) *flag_s = atomicAdd(&a.head_cnt[h], 1u) == (unsigned)(Se - 1);
  __syncthreads();
  if (!*flag_s) return j;
  __threadfence();
  const float *allp = a.attn_part + (size_t)h * S * PSTR;
  float *ms_s = acc_w;             // [Se][GP] split maxima, then merge weights
  float *ls_s = acc_w + 64 * GP;   // [Se][GP] split denominators
  for (int i = tid; i < Se * GP; i += kMT) {
    const int sp = i / GP, g = i % GP;
    ms_s[i] = __ldcg(allp + (size_t)sp * PSTR + GP * HD + g);
    ls_s[i] = __ldcg(allp + (size_t)sp * PSTR + GP * HD + GP + g);
  }
  __syncthreads();
  if (tid < GP) {
    float M = -INFINITY;
    for (int sp = 0; sp < Se; sp++) M = fmaxf(M, ms_s[sp * GP + tid]);
    float dsum = 0.0f;
    for (int sp = 0; sp < Se; sp++) {
      const float m = ms_s[sp * GP + tid];
      const float w = m == -INFINITY ? 0.0f : expf(m - M);
      ms_s[sp * GP + tid] = w;
      dsum = fmaf(w, ls_s[sp * GP + tid], dsum);
    }
    den[tid] = dsum;
  }
  __syncthreads();
  // Warp w finalises 32-blocks w, w + kMW, ... of the head group and
  // quantizes them (QuantizedActQ8; head boundaries are 32-aligned).
  for (int bi = warp; bi < G * HD / 32; bi += kMW) {
    const int e = bi * 32 + lane, g = e / HD;
    float num = 0.0f;
#pragma unroll 4
    for (int sp = 0; sp < Se; sp++) num = fmaf(ms_s[sp * GP + g], __ldcg(allp + (size_t)sp * PSTR + e), num);
    float o = den[g] > 0.0f ? __fdiv_rn(num, den[g]) : 0.0f;
    a.attn[ob + e] = o;
    if (!isfinite(o)) o = 0.0f;
    const float amax = warp_max(fabsf(o));
    const float scale = act_scale_from_amax(amax), inv = act_inv_from_scale(scale);
    a.attn_q[ob + e] = act_quant_one(o, inv);
    if (lane == 0) a.attn_s[ob / 32 + bi] = scale;
  }
  if (tid == 0) a.head_cnt[h] = 0u;
  __syncthreads();
  return j;
}

// ---- embedding and argmax ------------------------------------------------------
__device__ __noinline__ void ph_embed(const MegaArgs &a) {
  const int64_t H = a.H;
  const uint32_t tok = *a.d_token;
  const int64_t per = (H + gridDim.x - 1) / gridDim.x, e0 = blockIdx.x * per;
  const int64_t e1 = e0 + per < H ? e0 + per : H;
  const bool bad = tok >= (uint32_t)a.emb_rows;
  if (bad && blockIdx.x == 0 && threadIdx.x == 0 && a.err) atomicOr(a.err, 1);
  const float *norm = a.layers[0].attn_norm;
  float ss = 0.0f;
  for (int64_t i = e0 + threadIdx.x; i < e1; i += kMT) {
    const float h = bad ? 0.0f : embed_value(a.emb, a.emb_quant, H, tok, i);
    a.hidden[i] = h;
    ss = fmaf(h, h, ss);
    a.hu[i] = __fmul_rn(h, norm[i]);
  }
  // the first layer's RMSNorm input (see next_norm_input)
  const float tot = block_reduce_sum<kMW>(ss, mega_red);
  if (threadIdx.x == 0) a.hss[blockIdx.x] = tot;
  quantize_done_blocks(a.hu, a.hq, a.hs, a.hcnt, e0, e1 - e0);
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
  *a.bar = 0u;  // every CTA is past its last barrier wait
}

// ---- phases: build the projection's arguments and run it from the ring ------
template <int HD, bool F16, int QW>
__device__ __forceinline__ unsigned ph_proj(const MegaArgs &a, const Plan &p, const Ring &r, int kind, int l, unsigned j) {
  GemvArgs g;
  g.m = 1;
  const Rows *rs;
  g.eps = a.eps;
  g.ss_part = a.hss; g.ss_n = (int)gridDim.x;  // RMSNorm inputs (GEMV_IN_PREQ)
  if (kind == 4) {  // LM head (final RMSNorm)
    g.w = a.lm_head; g.rows = a.V; g.in_mode = GEMV_IN_PREQ; g.xq = a.hq; g.xs = a.hs;
    g.out_mode = GEMV_OUT_STORE; g.y = a.logits; g.y_stride = a.V;
    rs = &p.head;
  } else {
    const MegaLayer &L = a.layers[l];
    if (kind == 0) {  // Q/K/V (RMSNorm prologue)
      const int64_t QKV = (a.n_heads_q + 2 * a.n_kv) * HD;
      g.w = L.qkv; g.rows = QKV; g.in_mode = GEMV_IN_PREQ; g.xq = a.hq; g.xs = a.hs;
      g.out_mode = GEMV_OUT_STORE; g.y = a.qkv; g.y_stride = QKV;
      rs = &p.q;
    } else if (kind == 1) {  // O + residual (+ bias)
      g.w = L.wo; g.rows = a.H; g.in_mode = GEMV_IN_Q8;
      g.xq = a.attn_q; g.xs = a.attn_s; g.xq_stride = a.n_heads_q * HD;
      g.out_mode = GEMV_OUT_ADD; g.y = a.hidden; g.y_stride = a.H; g.bias = L.bo;
      g.nx_norm = L.ffn_norm;  // the gate/up phase's RMSNorm input
      g.nx_u = a.hu; g.nx_q = a.hq; g.nx_s = a.hs; g.nx_cnt = a.hcnt; g.nx_ss = a.hss;
      rs = &p.o;
    } else if (kind == 2) {  // gate/up + SwiGLU (RMSNorm prologue), also quantized
      g.w = L.gateup; g.rows = a.F; g.in_mode = GEMV_IN_PREQ; g.xq = a.hq; g.xs = a.hs;
      g.out_mode = GEMV_OUT_SWIGLU; g.y = a.ffn; g.y_stride = a.F; g.up_offset = a.F;
      g.yq = a.ffn_q; g.ys = a.ffn_s; g.ycnt = a.ffn_cnt;
      rs = &p.gu;
    } else {  // down + residual (input quantized by the gate/up phase)
      g.w = L.wdown; g.rows = a.H; g.in_mode = GEMV_IN_Q8;
      g.xq = a.ffn_q; g.xs = a.ffn_s; g.xq_stride = a.F;
      g.out_mode = GEMV_OUT_ADD; g.y = a.hidden; g.y_stride = a.H;
      g.nx_norm = l + 1 < a.n_layers ? a.layers[l + 1].attn_norm : a.out_norm;  // next RMSNorm input
      g.nx_u = a.hu; g.nx_q = a.hq; g.nx_s = a.hs; g.nx_cnt = a.hcnt; g.nx_ss = a.hss;
      rs = &p.dn;
    }
  }
  return gemv_stream<QW, HD, F16>(a, p, r, g, *rs, j);
}

// Q4_0 kernels inline every phase into the kernel (no calls between the
// phases' loops); Q8_0 rows need more registers, so there each phase stays
// a separate function.
template <int HD, bool F16, int QW>
__device__ __noinline__ unsigned ph_proj_call(const MegaArgs &a, const Plan &p, const Ring &r, int kind, int l,
                                              unsigned j) {
  return ph_proj<HD, F16, QW>(a, p, r, kind, l, j);
}
template <int HD, bool F16, int GP>
__device__ __noinline__ unsigned attn_call(const MegaArgs &a, const Plan &p, const Ring &r, int l, unsigned j) {
  return attn_stream<HD, F16, GP>(a, p, r, l, j);
}
template <int HD, bool F16, int GP, int QW>
__device__ __forceinline__ unsigned run_proj(const MegaArgs &a, const Plan &p, const Ring &r, int kind, int l,
                                             unsigned j) {
  if constexpr (QW == JAL_Q4_0) return ph_proj<HD, F16, QW>(a, p, r, kind, l, j);
  else return ph_proj_call<HD, F16, QW>(a, p, r, kind, l, j);
}
template <int HD, bool F16, int GP, int QW>
__device__ __forceinline__ unsigned run_attn(const MegaArgs &a, const Plan &p, const Ring &r, int l, unsigned j) {
  if constexpr (QW == JAL_Q4_0) return attn_stream<HD, F16, GP>(a, p, r, l, j);
  else return attn_call<HD, F16, GP>(a, p, r, l, j);
}

template <int HD, bool F16, int GP, int QW>
__global__ void __launch_bounds__(kMT, 1) k_decode_mega(const MegaArgs *__restrict__ ap) {
  __shared__ __align__(8) uint64_t full[kSlots];
  __shared__ int broken;
  __shared__ unsigned seq;
  __shared__ Plan plan;
  const MegaArgs &a = *ap;
  const Ring ring{full};
  if (threadIdx.x == 0) {
    broken = 0;
    seq = 0;
    for (int s = 0; s < kSlots; s++) {
      mbar_init(&full[s], 1);
      mega_done[s] = 0u;
    }
    fence_barrier_init();
  }
  make_plan(a, *a.d_pos, AttnGeom<HD, F16, 1>::TP, plan);
  __syncthreads();
  if (threadIdx.x == 0)
    for (int s = 0; s < kSlots; s++) ring_issue<HD, F16>(plan, ring, (unsigned)s);
  const GridBar gb{a.bar, a.err, &broken, &seq};
  ph_embed(a);
  grid_sync(gb);
  unsigned j = 0;  // stream index of the next chunk (the same in every thread)
  const int n_layers = a.n_layers;
  for (int l = 0; l < n_layers; l++) {
    j = run_proj<HD, F16, GP, QW>(a, plan, ring, 0, l, j);
    grid_sync(gb);
    j = run_attn<HD, F16, GP, QW>(a, plan, ring, l, j);
    grid_sync(gb);
    j = run_proj<HD, F16, GP, QW>(a, plan, ring, 1, l, j);
    grid_sync(gb);
    j = run_proj<HD, F16, GP, QW>(a, plan, ring, 2, l, j);
    grid_sync(gb);
    j = run_proj<HD, F16, GP, QW>(a, plan, ring, 3, l, j);
    grid_sync(gb);
  }
  j = run_proj<HD, F16, GP, QW>(a, plan, ring, 4, 0, j);
  argmax_phase(a, mega_red);
  // Every issued chunk was waited for; after a wait that gave up, wait again
  // (bounded) so that no copy is still landing when the CTA exits.
  if (threadIdx.x == 0)
    for (int k = plan.total > kSlots ? plan.total - kSlots : 0; k < plan.total; k++)
      mbar_wait_bounded(&full[k % kSlots], ((unsigned)k / kSlots) & 1u);
}

template <int HD, bool F16, int GP, int QW>
const void *mega_fn() {
  return (const void *)k_decode_mega<HD, F16, GP, QW>;
}

// One weight type for every projection (Q/K/V, O, gate/up, down, LM head).
int mega_quant(const MegaArgs &a) {
  const int q = a.lm_head.quant;
  if (q != JAL_Q4_0 && q != JAL_Q8_0) return -1;
  return q;
}

const void *pick_mega(int hd, int f16, int G, int qw) {
  if (G > 4) return nullptr;
#define JAL_PICK(HDV, F, QV) \
  if (hd == HDV && (f16 != 0) == F && qw == QV) return mega_fn<HDV, F, 4, QV>();
  JAL_PICK(128, true, JAL_Q4_0) JAL_PICK(128, false, JAL_Q4_0) JAL_PICK(64, true, JAL_Q4_0) JAL_PICK(64, false, JAL_Q4_0)
  JAL_PICK(128, true, JAL_Q8_0) JAL_PICK(128, false, JAL_Q8_0) JAL_PICK(64, true, JAL_Q8_0) JAL_PICK(64, false, JAL_Q8_0)
#undef JAL_PICK
  return nullptr;
}

// Work area of one projection phase: activation region plus the
// per-segment partials of one chunk's rows.
size_t proj_work(int in_mode, int64_t cols, int64_t qs_stride) {
  const int nb = (int)(cols / 32), nseg = seg_count(cols);
  int64_t rpc = kSlotBytes / qs_stride;
  if (rpc < 1) rpc = 1;
  return w4_act_region(in_mode, nb, nseg) + (size_t)kSlots * rpc * nseg * 4;
}

constexpr size_t mega_smem() { return kRingBytes + kWorkBytes; }

}  // namespace

int mega_check(const MegaArgs &a, int grid) {
  if (grid < 1 || a.n_kv < 1 || a.n_heads_q % a.n_kv) return 0;
  const int qw = mega_quant(a);
  const int64_t HD = a.kv.head_dim, Q = a.n_heads_q * HD;
  if (!pick_mega((int)HD, a.kv.f16, (int)(a.n_heads_q / a.n_kv), qw)) return 0;
  // SwiGLU pairs need the whole gate/up row in one segment; other inputs
  // may span up to one segment per warp.
  if (seg_count(a.H) != 1) return 0;
  if (seg_count(Q) > kMW || seg_count(a.F) > kMW) return 0;
  if (a.splits < 1 || a.splits > 64 || a.n_kv * a.splits > grid) return 0;
  // Whole rows per ring slot, and the work area of every phase.
  const int64_t row_q = (int64_t)(qw == JAL_Q4_0 ? 18 : 34);  // bytes per 32 weights
  const int64_t strides[3] = {a.H / 32 * row_q, Q / 32 * row_q, a.F / 32 * row_q};
  for (int64_t s : strides)
    if (s + 256 > kSlotBytes) return 0;
  const size_t resid = (size_t)(a.H / grid + 1) * 4;  // staged residual rows (O and down)
  if (a.n_layers > kMaxLayers) return 0;
  if (proj_work(GEMV_IN_Q8, a.F, a.F / 32 * row_q + 256) + resid > kWorkBytes) return 0;
  if (proj_work(GEMV_IN_Q8, Q, Q / 32 * row_q + 256) + resid > kWorkBytes) return 0;
  if (proj_work(GEMV_IN_PREQ, a.H, a.H / 32 * row_q) > kWorkBytes) return 0;
  if (8192 + (size_t)kMW * 4 * HD * 4 + 2 * kMW * 4 * 4 > kWorkBytes) return 0;  // attention workspace
  return 1;
}

size_t mega_part_bytes(const MegaArgs &a) {
  constexpr int GP = 4;  // query heads per KV head in every instantiation
  return (size_t)a.n_kv * a.splits * (GP * a.kv.head_dim + 2 * GP) * sizeof(float);
}

int prepare_decode_mega(const MegaArgs &a, int grid) {
  if (!mega_check(a, grid)) return 0;
  const void *fn = pick_mega((int)a.kv.head_dim, a.kv.f16, (int)(a.n_heads_q / a.n_kv), mega_quant(a));
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mega_smem()) == cudaSuccess;
}

int launch_decode_mega(const MegaArgs &a, const MegaArgs *dev_args, int grid, cudaStream_t s) {
  const void *fn = pick_mega((int)a.kv.head_dim, a.kv.f16, (int)(a.n_heads_q / a.n_kv), mega_quant(a));
  if (!fn) return 0;
  const size_t smem = mega_smem();
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
