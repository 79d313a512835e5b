// Prefill GEMM over the repacked Q4_0 / Q8_0 layout, CUDA-core version.
//
// y[t][r] = sum over 16-element chunks of (f32(dot16) * a_sc[t][ch/2]) *
// w_sc[r][ch/2] (repack_cache.rs:739-783, gemm_rows :808-837): the same
// integer partials and the same per-term rounding as the decode GEMV, with
// a different f32 summation order.
//
// CTA tile: 32 tokens x 64 rows, 128 threads, K staged 4 blocks (128
// elements) at a time.  Shared memory is block-major so that lanes reading
// consecutive rows (or the same token) never conflict.  Thread (tm, tn)
// computes tokens tm*4..tm*4+3 against rows tn, tn+16, tn+32, tn+48.
#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int BM = 32, BN = 64, KB = 4;  // tokens, rows, 32-blocks per stage

template <int QUANT>
__global__ void __launch_bounds__(128) k_gemm(const GemmArgs a) {
  constexpr int WB = QUANT == JAL_Q4_0 ? 16 : 32;  // weight bytes per block
  __shared__ __align__(16) uint8_t w_s[KB][BN][WB];
  __shared__ float wd_s[KB][BN];
  __shared__ __align__(16) int8_t alo_s[KB][BM][16];
  __shared__ __align__(16) int8_t ahi_s[KB][BM][16];
  __shared__ float as_s[KB][BM];
  __shared__ int2 asum_s[KB][BM];
  const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;
  const int64_t t0 = (int64_t)blockIdx.y * BM, r0 = (int64_t)blockIdx.x * BN;
  const int64_t K = a.w.cols, nb = K / 32;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

  for (int64_t b0 = 0; b0 < nb; b0 += KB) {
    __syncthreads();
    // Weights: KB blocks x 64 rows.
    for (int i = tid; i < KB * BN * (WB / 16); i += 128) {
      int piece = i % (WB / 16), rr = (i / (WB / 16)) % BN, kb = i / (WB / 16) / BN;
      int64_t r = r0 + rr, b = b0 + kb;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < a.rows && b < nb) v = *(const uint4 *)(a.w.qs + r * a.w.qs_stride + b * WB + piece * 16);
      *(uint4 *)&w_s[kb][rr][piece * 16] = v;
    }
    for (int i = tid; i < KB * BN; i += 128) {
      int rr = i % BN, kb = i / BN;
      int64_t r = r0 + rr, b = b0 + kb;
      wd_s[kb][rr] = (r < a.rows && b < nb) ? f16_finite(a.w.d[r * a.w.d_stride + b]) : 0.0f;
    }
    // Activations: KB blocks x 32 tokens (+ scales and 16-element sums).
    for (int i = tid; i < KB * BM * 2; i += 128) {
      int half = i % 2, tt = (i / 2) % BM, kb = i / 2 / BM;
      int64_t t = t0 + tt, b = b0 + kb;
      int4 v = make_int4(0, 0, 0, 0);
      if (t < a.m && b < nb) v = *(const int4 *)(a.xq + t * K + b * 32 + half * 16);
      if (half == 0) *(int4 *)alo_s[kb][tt] = v;
      else *(int4 *)ahi_s[kb][tt] = v;
      int s = dp4a_ss(v.x, 0x01010101, 0);
      s = dp4a_ss(v.y, 0x01010101, s);
      s = dp4a_ss(v.z, 0x01010101, s);
      s = dp4a_ss(v.w, 0x01010101, s);
      if (half == 0) asum_s[kb][tt].x = s;
      else asum_s[kb][tt].y = s;
    }
    for (int i = tid; i < KB * BM; i += 128) {
      int tt = i % BM, kb = i / BM;
      int64_t t = t0 + tt, b = b0 + kb;
      as_s[kb][tt] = (t < a.m && b < nb) ? a.xs[t * nb + b] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kb = 0; kb < KB; kb++) {
      uint4 wv[4][WB / 16];
      float wsc[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        wv[j][0] = *(const uint4 *)&w_s[kb][tn + 16 * j][0];
        if (WB == 32) wv[j][WB / 16 - 1] = *(const uint4 *)&w_s[kb][tn + 16 * j][16];
        wsc[j] = wd_s[kb][tn + 16 * j];
      }
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int tt = tm * 4 + i;
        const int4 al = *(const int4 *)alo_s[kb][tt];
        const int4 ah = *(const int4 *)ahi_s[kb][tt];
        const float as = as_s[kb][tt];
        const int2 sm = asum_s[kb][tt];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          int dlo, dhi;
          if (QUANT == JAL_Q4_0) {
            const uint4 w = wv[j][0];
            dlo = dp4a_us(w.x & 0x0F0F0F0Fu, al.x, 0);
            dlo = dp4a_us(w.y & 0x0F0F0F0Fu, al.y, dlo);
            dlo = dp4a_us(w.z & 0x0F0F0F0Fu, al.z, dlo);
            dlo = dp4a_us(w.w & 0x0F0F0F0Fu, al.w, dlo);
            dhi = dp4a_us((w.x >> 4) & 0x0F0F0F0Fu, ah.x, 0);
            dhi = dp4a_us((w.y >> 4) & 0x0F0F0F0Fu, ah.y, dhi);
            dhi = dp4a_us((w.z >> 4) & 0x0F0F0F0Fu, ah.z, dhi);
            dhi = dp4a_us((w.w >> 4) & 0x0F0F0F0Fu, ah.w, dhi);
            dlo -= 8 * sm.x;
            dhi -= 8 * sm.y;
          } else {
            const uint4 w0 = wv[j][0], w1 = wv[j][WB / 16 - 1];
            dlo = dp4a_ss((int)w0.x, al.x, 0);
            dlo = dp4a_ss((int)w0.y, al.y, dlo);
            dlo = dp4a_ss((int)w0.z, al.z, dlo);
            dlo = dp4a_ss((int)w0.w, al.w, dlo);
            dhi = dp4a_ss((int)w1.x, ah.x, 0);
            dhi = dp4a_ss((int)w1.y, ah.y, dhi);
            dhi = dp4a_ss((int)w1.z, ah.z, dhi);
            dhi = dp4a_ss((int)w1.w, ah.w, dhi);
          }
          float tlo = __fmul_rn(__fmul_rn(__int2float_rn(dlo), as), wsc[j]);
          float thi = __fmul_rn(__fmul_rn(__int2float_rn(dhi), as), wsc[j]);
          acc[i][j] += tlo + thi;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int64_t t = t0 + tm * 4 + i;
    if (t >= a.m) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int64_t r = r0 + tn + 16 * j;
      if (r >= a.rows) continue;
      float v = acc[i][j];
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
  if (a.w.quant == JAL_Q4_0) k_gemm<JAL_Q4_0><<<grid, 128, 0, s>>>(a);
  else k_gemm<JAL_Q8_0><<<grid, 128, 0, s>>>(a);
}

}  // namespace jal
