// Device building blocks of decode attention over the paged KV cache, shared
// by the cluster kernel (attention.cu) and the persistent decode kernel
// (decode_mega.cu): KV indexing, the RoPE rotation, the tile geometry of
// the shared-memory K/V ring and its bulk-copy issue.
#pragma once

#include <cuda_fp16.h>

#include "dev_util.cuh"
#include "device.hpp"

namespace jal {
namespace adev {

constexpr int kStages = 3;           // shared-memory ring of K/V tiles
constexpr int kStageBytes = 32 * 1024;

__device__ __forceinline__ int64_t kv_elem(const KvView &kv, int64_t layer, int64_t h, int64_t pos) {
  int64_t page = kv.page_table[pos / kv.page_size], slot = pos % kv.page_size;
  return (((layer * kv.n_pages + page) * kv.n_kv + h) * kv.page_size + slot) * kv.head_dim;
}

__device__ __forceinline__ void store_kv(void *base, int f16, int64_t e, float v) {
  if (f16) ((__half *)base)[e] = __float2half_rn(v);
  else ((float *)base)[e] = v;
}

// Rotate pair (x0, x1) by (c, s): recipe.rs:2750-2767.
__device__ __forceinline__ void rot(float &x0, float &x1, float c, float s) {
  float a = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  float b = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  x0 = a;
  x1 = b;
}

// Tile geometry for head_dim HD, KV element type and WARPS warps per CTA.
template <int HD, bool F16, int WARPS>
struct AttnGeom {
  static constexpr int ES = F16 ? 2 : 4;              // bytes per element
  static constexpr int ROW = HD * ES;                 // bytes of one position's K (or V)
  static constexpr int TP = kStageBytes / (2 * ROW);  // positions per tile
  static constexpr int LG = ROW / 16;                 // lanes per position when scoring
  static constexpr int PPS = 32 / LG;                 // positions per warp step when scoring
  static constexpr int DPL = 16 / ES;                 // dims per lane when scoring
  static constexpr int TPW = TP / WARPS;              // positions per warp per tile
  static constexpr int VD = HD / 32;                  // dims per lane in P.V
  static_assert(TPW % PPS == 0, "tile split");
};

// Copies positions [t0, t0 + n) of KV head h (K then V) into a ring stage;
// one bulk copy per page run.  Caller: one thread.
template <int HD, bool F16>
__device__ void issue_tile(const KvView &kv, int64_t layer, char *stage, uint64_t *bar, int64_t t0, int n, int h) {
  using Gm = AttnGeom<HD, F16, 1>;
  mbar_expect_tx(bar, (uint32_t)(2 * n * Gm::ROW));
  int done = 0;
  while (done < n) {
    const int64_t p = t0 + done;
    const int64_t page = kv.page_table[p / kv.page_size], slot = p % kv.page_size;
    const int run = (int)(kv.page_size - slot < n - done ? kv.page_size - slot : n - done);
    const int64_t e = (((layer * kv.n_pages + page) * kv.n_kv + h) * kv.page_size + slot) * HD;
    bulk_g2s(stage + done * Gm::ROW, (const char *)kv.k + e * Gm::ES, (uint32_t)(run * Gm::ROW), bar);
    bulk_g2s(stage + Gm::TP * Gm::ROW + done * Gm::ROW, (const char *)kv.v + e * Gm::ES, (uint32_t)(run * Gm::ROW),
             bar);
    done += run;
  }
}

template <bool F16, int N>
__device__ __forceinline__ void load_vals(const char *p, float (&o)[N]) {
  if (F16) {
    if (N == 8) {
      const uint4 raw = *(const uint4 *)p;
      const __half2 *r = (const __half2 *)&raw;
#pragma unroll
      for (int k = 0; k < 4; k++) { float2 f = __half22float2(r[k]); o[2 * k] = f.x; o[2 * k + 1] = f.y; }
    } else if (N == 4) {
      const uint2 raw = *(const uint2 *)p;
      const __half2 *r = (const __half2 *)&raw;
#pragma unroll
      for (int k = 0; k < 2; k++) { float2 f = __half22float2(r[k]); o[2 * k] = f.x; o[2 * k + 1] = f.y; }
    } else {
      const __half2 *h2 = (const __half2 *)p;
#pragma unroll
      for (int k = 0; k < N / 2; k++) { float2 f = __half22float2(h2[k]); o[2 * k] = f.x; o[2 * k + 1] = f.y; }
    }
  } else {
    if (N == 4) {
      const float4 v = *(const float4 *)p;
      o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
    } else {
#pragma unroll
      for (int k = 0; k < N / 2; k++) { float2 f = ((const float2 *)p)[k]; o[2 * k] = f.x; o[2 * k + 1] = f.y; }
    }
  }
}

}  // namespace adev
}  // namespace jal
