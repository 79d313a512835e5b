// Prefill GEMM over the repacked Q4_0 / Q8_0 layout on the int8 tensor
// cores (mma.sync m16n8k32, s8 x s8 -> s32).
//
// y[t][r] = sum over 32-blocks of f32(dot32) * (a_sc[t][b] * w_sc[r][b]),
// the fast-path form of the decode GEMV (one FMA per block); against
// repack_cache.rs:739-783 (per-16-chunk terms (f32(dot16) * a_sc) * w_sc)
// only the f32 rounding and summation order differ.  The integer dot of a
// block is exact (|dot32| < 2^24).
//
// CTA tile: 128 tokens x 128 rows, 8 warps, K staged 4 blocks (128
// elements) at a time in shared memory.  Warp w computes tokens
// 16w..16w+15 against the 128 rows as 16 n-tiles of 8 rows, one MMA per
// block and n-tile.  MMA
// fragments (PTX m16n8k32 .s8, g = lane / 4, q = lane % 4): A (tokens x 32,
// row-major) regs = (token g, k 4q..4q+3), (g + 8, 4q..), (g, 16 + 4q..),
// (g + 8, 16 + 4q..); B (32 x 8 rows, column-major) regs = (row g, k
// 4q..4q+3), (g, 16 + 4q..); C = tokens g and g + 8, rows 2q and 2q + 1.
// A Q4_0 block's byte i holds elements i (low nibble) and i + 16 (high
// nibble), so one 32-bit load at byte 4q gives both B registers.
#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int BM = 128, BN = 128, KB = 4;  // tokens, rows, 32-blocks per stage
constexpr int kThreads = 256, kNT = BN / 8;  // 8 warps; n-tiles of 8 rows per warp

__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four nibbles 0..15 (one per byte) to signed bytes n - 8.
__device__ __forceinline__ uint32_t nib_s8(uint32_t v) { return ((v | 0x80808080u) - 0x08080808u) ^ 0x80808080u; }

template <int QUANT>
__global__ void __launch_bounds__(kThreads) k_gemm(const GemmArgs a) {
  constexpr int WB = QUANT == JAL_Q4_0 ? 16 : 32;  // weight bytes per block
  __shared__ __align__(16) uint8_t w_s[KB][BN][WB];
  __shared__ float wd_s[KB][BN];
  __shared__ __align__(16) int8_t x_s[KB][BM][32];
  __shared__ float as_s[KB][BM];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32, g = lane / 4, q = lane % 4;
  const int64_t t0 = (int64_t)blockIdx.y * BM, r0 = (int64_t)blockIdx.x * BN;
  const int64_t K = a.w.cols, nb = K / 32;
  float acc[kNT][4];
#pragma unroll
  for (int n = 0; n < kNT; n++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[n][i] = 0.0f;

  for (int64_t b0 = 0; b0 < nb; b0 += KB) {
    __syncthreads();
    // Weights: KB blocks x 64 rows.
    for (int i = tid; i < KB * BN * (WB / 16); i += kThreads) {
      int piece = i % (WB / 16), rr = (i / (WB / 16)) % BN, kb = i / (WB / 16) / BN;
      int64_t r = r0 + rr, b = b0 + kb;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < a.rows && b < nb) v = *(const uint4 *)(a.w.qs + r * a.w.qs_stride + b * WB + piece * 16);
      *(uint4 *)&w_s[kb][rr][piece * 16] = v;
    }
    for (int i = tid; i < KB * BN; i += kThreads) {
      int rr = i % BN, kb = i / BN;
      int64_t r = r0 + rr, b = b0 + kb;
      wd_s[kb][rr] = (r < a.rows && b < nb) ? f16_finite(a.w.d[r * a.w.d_stride + b]) : 0.0f;
    }
    // Activations: KB blocks x 64 tokens, and their block scales.
    for (int i = tid; i < KB * BM * 2; i += kThreads) {
      int half = i % 2, tt = (i / 2) % BM, kb = i / 2 / BM;
      int64_t t = t0 + tt, b = b0 + kb;
      int4 v = make_int4(0, 0, 0, 0);
      if (t < a.m && b < nb) v = *(const int4 *)(a.xq + t * K + b * 32 + half * 16);
      *(int4 *)&x_s[kb][tt][half * 16] = v;
    }
    for (int i = tid; i < KB * BM; i += kThreads) {
      int tt = i % BM, kb = i / BM;
      int64_t t = t0 + tt, b = b0 + kb;
      as_s[kb][tt] = (t < a.m && b < nb) ? a.xs[t * nb + b] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kb = 0; kb < KB; kb++) {
      const int ta = warp * 16 + g;  // tokens ta and ta + 8
      const uint32_t alo0 = *(const uint32_t *)&x_s[kb][ta][4 * q];
      const uint32_t alo1 = *(const uint32_t *)&x_s[kb][ta + 8][4 * q];
      const uint32_t ahi0 = *(const uint32_t *)&x_s[kb][ta][16 + 4 * q];
      const uint32_t ahi1 = *(const uint32_t *)&x_s[kb][ta + 8][16 + 4 * q];
      const float as0 = as_s[kb][ta], as1 = as_s[kb][ta + 8];
#pragma unroll
      for (int n = 0; n < kNT; n++) {
        const int rb = n * 8 + g;  // this lane's B row
        uint32_t blo, bhi;
        if (QUANT == JAL_Q4_0) {
          const uint32_t w = *(const uint32_t *)&w_s[kb][rb][4 * q];
          blo = nib_s8(w & 0x0F0F0F0Fu);
          bhi = nib_s8((w >> 4) & 0x0F0F0F0Fu);
        } else {
          blo = *(const uint32_t *)&w_s[kb][rb][4 * q];
          bhi = *(const uint32_t *)&w_s[kb][rb][16 + 4 * q];
        }
        int c[4] = {0, 0, 0, 0};
        mma_s8_16832(c, alo0, alo1, ahi0, ahi1, blo, bhi);
        const float ws0 = wd_s[kb][n * 8 + 2 * q], ws1 = wd_s[kb][n * 8 + 2 * q + 1];
        acc[n][0] = fmaf(__int2float_rn(c[0]), as0 * ws0, acc[n][0]);
        acc[n][1] = fmaf(__int2float_rn(c[1]), as0 * ws1, acc[n][1]);
        acc[n][2] = fmaf(__int2float_rn(c[2]), as1 * ws0, acc[n][2]);
        acc[n][3] = fmaf(__int2float_rn(c[3]), as1 * ws1, acc[n][3]);
      }
    }
  }
#pragma unroll
  for (int n = 0; n < kNT; n++) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t t = t0 + warp * 16 + g + (i < 2 ? 0 : 8);
      const int64_t r = r0 + n * 8 + 2 * q + (i & 1);
      if (t >= a.m || r >= a.rows) continue;
      float v = acc[n][i];
      if (a.bias) v += a.bias[r];
      float *yp = a.y + t * a.y_stride + r;
      *yp = a.accumulate ? *yp + v : v;
    }
  }
}

}  // namespace

void launch_gemm(const GemmArgs &a, cudaStream_t s) {
  if (a.m <= 0 || a.rows <= 0) return;
  dim3 grid((unsigned)((a.rows + BN - 1) / BN), (unsigned)((a.m + BM - 1) / BM));
  if (a.w.quant == JAL_Q4_0) k_gemm<JAL_Q4_0><<<grid, kThreads, 0, s>>>(a);
  else k_gemm<JAL_Q8_0><<<grid, kThreads, 0, s>>>(a);
}

}  // namespace jal
