// Device helpers shared by the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "jal.h"

namespace jal {

// f16_to_f32_finite (repack_cache.rs:160-181): IEEE half -> f32, with the
// Inf/NaN encodings mapped to +-0.0625.  Subnormals convert exactly.
__device__ __forceinline__ float f16_finite(uint16_t h) {
  if ((h & 0x7C00u) == 0x7C00u) return (h & 0x8000u) ? -0.0625f : 0.0625f;
  return __half2float(__ushort_as_half(h));
}

// bf16_to_f32_finite (repack_cache.rs:184-191).
__device__ __forceinline__ float bf16_finite(uint16_t h) {
  if (((h >> 7) & 0xFF) == 0xFF) return (h & 0x8000u) ? -0.0625f : 0.0625f;
  return __uint_as_float((uint32_t)h << 16);
}

// sanitize_f32_weight (repack_cache.rs:1028-1036).
__device__ __forceinline__ float sanitize_weight(float v) {
  if (!isfinite(v)) return 0.0f;
  if (fabsf(v) > 1.0e6f) return signbit(v) ? -0.0625f : 0.0625f;
  return v;
}

// Sum of four u8 x s8 products plus c (PTX dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }

// 16-byte streaming load that does not allocate in L1 (weights are read
// once per step).
__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// 32-byte streaming load (sm_100 256-bit vector load), no L1 allocation.
__device__ __forceinline__ void ldg_stream32(const void *p, uint32_t *o) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3]), "=r"(o[4]), "=r"(o[5]), "=r"(o[6]), "=r"(o[7])
               : "l"(p));
}
__device__ __forceinline__ uint2 ldg_stream8(const void *p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg_stream2(const uint16_t *p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Per-32-block activation quantization of QuantizedActQ8
// (repack_cache.rs:390-422): non-finite -> 0, scale = amax/127,
// inv = 1/scale, q = clamp(round(v*inv), -127, 127).  Correctly rounded
// division/multiplication keep every value bit-identical to the reference.
__device__ __forceinline__ float act_scale_from_amax(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f;
}
__device__ __forceinline__ float act_inv_from_scale(float scale) {
  return scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
}
__device__ __forceinline__ int8_t act_quant_one(float v, float inv) {
  float q = roundf(__fmul_rn(v, inv));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return (int8_t)q;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch controls (no-ops without the attribute).
// Bulk prefetch of [p, p + bytes) into L2 by the copy engine (no registers or
// shared memory held).  p must be 16-byte aligned; bytes is rounded down to a
// multiple of 16 and split into pieces of at most 1 GiB.
__device__ __forceinline__ void l2_prefetch_bulk(const void *p, uint64_t bytes) {
  const char *c = (const char *)p;
  bytes &= ~(uint64_t)15;
  while (bytes) {
    const uint32_t n = bytes > (1u << 30) ? (1u << 30) : (uint32_t)bytes;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
    c += n;
    bytes -= n;
  }
}

// Element i of embedding row tok (embed_tokens / decode_row_to_f32,
// recipe.rs:1395-1440, repack_cache.rs:1166-1301): f32 / f16 / bf16 rows
// sanitized, Q4_0 / Q5_0 / Q8_0 blocks dequantized as d * q.
__device__ __forceinline__ float embed_value(const uint8_t *emb, int quant, int64_t hidden, uint32_t tok, int64_t i) {
  if (quant == JAL_F32) return sanitize_weight(((const float *)emb)[(int64_t)tok * hidden + i]);
  if (quant == JAL_F16) return f16_finite(((const uint16_t *)emb)[(int64_t)tok * hidden + i]);
  if (quant == JAL_BF16) return bf16_finite(((const uint16_t *)emb)[(int64_t)tok * hidden + i]);
  const int64_t g = i / 32, e = i % 32;
  const int64_t bb = quant == JAL_Q4_0 ? 18 : quant == JAL_Q5_0 ? 22 : 34;
  const uint8_t *blk = emb + ((int64_t)tok * (hidden / 32) + g) * bb;
  const float d = f16_finite((uint16_t)(blk[0] | (blk[1] << 8)));
  int q;
  if (quant == JAL_Q4_0) {
    q = (int)(e < 16 ? (blk[2 + e] & 15) : (blk[2 + e - 16] >> 4)) - 8;
  } else if (quant == JAL_Q5_0) {
    const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
    const int j = e & 15;
    const uint32_t nib = e < 16 ? (blk[6 + j] & 15u) : (uint32_t)(blk[6 + j] >> 4);
    const uint32_t hb = ((qh >> (e < 16 ? j : j + 16)) & 1u) << 4;
    q = (int)(nib | hb) - 16;
  } else {
    q = (int8_t)blk[2 + e];
  }
  return d == 0.0f ? 0.0f : __fmul_rn(d, (float)q);
}

// ---- mbarrier / bulk-copy helpers (shared::cta barrier, own-CTA destination;
// no multicast)
constexpr uint64_t kWaitNs = 2000000000ull;  // a copy not landed after 2 s: give up
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Step trace (diagnostic): with t non-null (kTraceSlots per launch), a kernel
// records the globaltimer of its first CTA start in t[0] (atomic min; the
// slot starts at all ones), of its last warp's exit in t[1] (atomic max;
// starts at 0), and mark(k) the latest time any CTA reached phase k in
// t[2 + k].  Declared first in the kernel, so the exit stamp runs on every
// return path.
struct KernelTrace {
  unsigned long long *t;
  __device__ explicit KernelTrace(unsigned long long *p) : t(p) {
    if (t && threadIdx.x == 0) atomicMin(t, (unsigned long long)global_ns());
  }
  __device__ ~KernelTrace() {
    if (t && (threadIdx.x & 31) == 0) atomicMax(t + 1, (unsigned long long)global_ns());
  }
  __device__ void mark(int k) const {
    if (t) atomicMax(t + 2 + k, (unsigned long long)global_ns());
  }
};

// Waits for the phase with the given parity for at most limit_ns of wall
// time (0 = kWaitNs); false when the wait gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t lim = limit_ns ? limit_ns : kWaitNs, t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > lim) return false;
  }
}
// As mbar_wait_bounded, sleeping ~128 ns between polls: for a waiter that
// shares its SM sub-partition with latency-bound warps.
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t *bar, uint32_t parity, uint64_t limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t lim = limit_ns ? limit_ns : kWaitNs, t0 = global_ns();
  for (;;) {
    __nanosleep(128);
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > lim) return false;
  }
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Cross-GPU exchange over peer memory (tensor parallelism): flagged 64-bit
// words, stored and polled at system scope.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2u64(const unsigned long long *p, unsigned long long &a,
                                                     unsigned long long &b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
constexpr uint64_t kPeerWaitNs = 4000000000ull;  // a peer's words not there after 4 s: give up
// Eight consecutive flagged words at p (16-byte aligned): waits until every
// flag equals `flag` and adds their values to v[0..7] in order.  False when
// the wait gave up after limit_ns (0 = kPeerWaitNs; the values are then
// added as found).
__device__ __forceinline__ bool peer_take8(const unsigned long long *p, uint32_t flag, float (&v)[8],
                                           uint64_t limit_ns = 0) {
  const uint64_t lim = limit_ns ? limit_ns : kPeerWaitNs;
  unsigned long long w[8];
  uint64_t t0 = 0;
  bool ok = true;
  for (int it = 0;; it++) {
#pragma unroll
    for (int k = 0; k < 4; k++) ld_relaxed_sys_v2u64(p + 2 * k, w[2 * k], w[2 * k + 1]);
    bool all = true;
#pragma unroll
    for (int k = 0; k < 8; k++) all = all && (uint32_t)(w[k] >> 32) == flag;
    if (all) break;
    if (it == 0) t0 = global_ns();
    else if (global_ns() - t0 > lim) { ok = false; break; }
    __nanosleep(32);
  }
#pragma unroll
  for (int k = 0; k < 8; k++) v[k] = __fadd_rn(v[k], __uint_as_float((uint32_t)w[k]));
  return ok;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace jal
