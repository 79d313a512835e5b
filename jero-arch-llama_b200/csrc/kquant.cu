// K-quant matrices (Q4_K, Q5_K, Q6_K) in the repacked path.
//
// Repack (unpack_row_i8 for the super-block types, repack_cache.rs:890-993):
// every 256-element super-block becomes 256 int8 quants (Q4_K: 0..15, Q5_K:
// 0..31, Q6_K: -32..31) in the row's quant plane, plus one f32 scale per
// group (Q4_K / Q5_K: 32 elements, d * sc; Q6_K: 16 elements, d * sc) and,
// for Q4_K / Q5_K, one f32 min per group (dmin * m), in planes of their own.
// The f16 fields are read with f16_to_f32_finite (Inf / NaN -> +-0.0625).
//
// Projection in the reference's order (the BlockScaledI8 arm of
// eval_row_range, repack_cache.rs:739-783): per row, over the 16-element
// chunks in order, acc += (f32(dot16) * a_sc[block]) * w_sc[group]; after the
// first chunk of every group that has a min, acc -= x_sum * w_mn, where x_sum
// is the group's sanitized f32 activation summed left to right from +0.0.
// One CTA of 16 warps takes 16 rows of one token: the token's QuantizedActQ8
// row (and the group sums) in shared memory; each warp's lanes form the
// chunk terms of its row into a term row in shared memory, and lane 0 folds
// them in chunk order.
#include <cuda_fp16.h>

#include <cstring>
#include <vector>

#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int kKqWarps = 16, kKqThreads = 32 * kKqWarps;

// repack_cache.rs:194-206: the 6-bit scales and mins of a Q4_K / Q5_K block.
__device__ __forceinline__ void kq_scales(const uint8_t *s, int j, uint32_t &sc, uint32_t &m) {
  if (j < 4) {
    sc = s[j] & 0x3Fu;
    m = s[j + 4] & 0x3Fu;
  } else {
    sc = (uint32_t)((s[j + 4] & 0x0Fu) | ((s[j - 4] >> 6) << 4));
    m = (uint32_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

// One thread per (row, super-block).
template <int QUANT>
__global__ void k_repack_kq(const uint8_t *__restrict__ raw, int64_t rows, int64_t nsb, int64_t raw_row,
                            int8_t *__restrict__ qs, int64_t qs_stride, float *__restrict__ ks,
                            float *__restrict__ km, int64_t k_stride) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nsb) return;
  const int64_t r = i / nsb, sb = i % nsb;
  int8_t *q = qs + r * qs_stride + sb * 256;
  if (QUANT == JAL_Q6_K) {
    const uint8_t *blk = raw + r * raw_row + sb * 210;
    const float d = f16_finite((uint16_t)(blk[208] | (blk[209] << 8)));
    const uint8_t *ql = blk, *qh = blk + 128, *sc = blk + 192;
    for (int sub = 0; sub < 16; sub++) ks[r * k_stride + sb * 16 + sub] = __fmul_rn(d, (float)(int8_t)sc[sub]);
    for (int half = 0; half < 2; half++) {
      const int n = half * 128, lo = half * 64, hi = half * 32;
      for (int l = 0; l < 32; l++) {
        q[n + l] = (int8_t)((int)((ql[lo + l] & 0x0F) | ((qh[hi + l] & 0x03) << 4)) - 32);
        q[n + l + 32] = (int8_t)((int)((ql[lo + l + 32] & 0x0F) | (((qh[hi + l] >> 2) & 0x03) << 4)) - 32);
        q[n + l + 64] = (int8_t)((int)(((ql[lo + l] >> 4) & 0x0F) | (((qh[hi + l] >> 4) & 0x03) << 4)) - 32);
        q[n + l + 96] = (int8_t)((int)(((ql[lo + l + 32] >> 4) & 0x0F) | (((qh[hi + l] >> 6) & 0x03) << 4)) - 32);
      }
    }
    return;
  }
  constexpr bool Q5 = QUANT == JAL_Q5_K;
  const uint8_t *blk = raw + r * raw_row + sb * (Q5 ? 176 : 144);
  const float d = f16_finite((uint16_t)(blk[0] | (blk[1] << 8)));
  const float dmin = f16_finite((uint16_t)(blk[2] | (blk[3] << 8)));
  for (int sub = 0; sub < 8; sub++) {
    uint32_t sc, m;
    kq_scales(blk + 4, sub, sc, m);
    ks[r * k_stride + sb * 8 + sub] = __fmul_rn(d, (float)sc);
    km[r * k_stride + sb * 8 + sub] = __fmul_rn(dmin, (float)m);
  }
  const uint8_t *qsr = blk + (Q5 ? 48 : 16), *qh = blk + 16;
  uint32_t u1 = 1, u2 = 2;
  for (int chunk = 0; chunk < 4; chunk++) {
    for (int l = 0; l < 32; l++) {
      const uint32_t hb1 = Q5 && (qh[l] & u1) ? 16u : 0u, hb2 = Q5 && (qh[l] & u2) ? 16u : 0u;
      q[chunk * 64 + l] = (int8_t)((qsr[chunk * 32 + l] & 0x0Fu) + hb1);
      q[chunk * 64 + 32 + l] = (int8_t)((qsr[chunk * 32 + l] >> 4) + hb2);
    }
    u1 <<= 2;
    u2 <<= 2;
  }
}

// grid (ceil(rows / 16), m): token blockIdx.y, rows blockIdx.x * 16 + warp.
template <bool MINS>
__global__ void __launch_bounds__(kKqThreads) k_kq_gemm(const DevMat w, const float *__restrict__ x,
                                                        const int8_t *__restrict__ xq, const float *__restrict__ xs,
                                                        float *__restrict__ y, int group) {
  extern __shared__ __align__(16) char smem[];
  const int64_t K = w.cols, nb = K / 32, nch = K / 16, ng = K / group, t = blockIdx.y;
  const int cps = group / 16;  // chunks per scale group
  int8_t *aq = (int8_t *)smem;                    // [K]
  float *asc = (float *)(smem + K);               // [nb]
  float *xsum = asc + nb;                         // [ng]
  float *terms = xsum + ng;                       // [warps][nch + 4]
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  for (int64_t i = tid; i < K / 16; i += kKqThreads) ((uint4 *)aq)[i] = ((const uint4 *)(xq + t * K))[i];
  for (int64_t i = tid; i < nb; i += kKqThreads) asc[i] = xs[t * nb + i];
  if (MINS)
    for (int64_t g = tid; g < ng; g += kKqThreads) {
      float s = 0.0f;
      for (int e = 0; e < group; e++) {
        const float v = x[t * K + g * group + e];
        s = __fadd_rn(s, isfinite(v) ? v : 0.0f);
      }
      xsum[g] = s;
    }
  __syncthreads();
  const int64_t r = (int64_t)blockIdx.x * kKqWarps + warp;
  if (r >= w.rows) return;
  float *tw = terms + (size_t)warp * (nch + 4);
  const int8_t *wr = (const int8_t *)w.qs + r * w.qs_stride;
  const float *ws = w.ks + r * w.k_stride;
  for (int64_t c = lane; c < nch; c += 32) {
    const uint4 wv = *(const uint4 *)(wr + c * 16), av = *(const uint4 *)(aq + c * 16);
    int d = dp4a_ss((int)wv.x, (int)av.x, 0);
    d = dp4a_ss((int)wv.y, (int)av.y, d);
    d = dp4a_ss((int)wv.z, (int)av.z, d);
    d = dp4a_ss((int)wv.w, (int)av.w, d);
    tw[c] = __fmul_rn(__fmul_rn(__int2float_rn(d), asc[c / 2]), ws[c / cps]);
  }
  __syncwarp();
  if (lane) return;
  const float *wm = MINS ? w.km + r * w.k_stride : nullptr;
  float acc = 0.0f;
  for (int64_t c = 0; c < nch; c++) {
    acc = __fadd_rn(acc, tw[c]);
    if (MINS && c % cps == 0) acc = __fsub_rn(acc, __fmul_rn(xsum[c / cps], wm[c / cps]));
  }
  y[t * w.rows + r] = acc;
}

size_t kq_smem(int64_t K, int group) {
  return (size_t)K + (size_t)(K / 32) * 4 + (size_t)(K / group) * 4 + (size_t)kKqWarps * (K / 16 + 4) * 4;
}

}  // namespace

bool kquant(int q) { return q == JAL_Q4_K || q == JAL_Q5_K || q == JAL_Q6_K; }
int kquant_group(int q) { return q == JAL_Q6_K ? 16 : 32; }

void launch_repack_kquant(const uint8_t *raw, int quant, int64_t rows, int64_t cols, int8_t *qs, int64_t qs_stride,
                          float *ks, float *km, int64_t k_stride, cudaStream_t s) {
  const int64_t nsb = cols / 256, n = rows * nsb;
  if (n == 0) return;
  const int64_t raw_row = nsb * (quant == JAL_Q4_K ? 144 : quant == JAL_Q5_K ? 176 : 210);
  const unsigned blocks = (unsigned)((n + 127) / 128);
  if (quant == JAL_Q4_K) k_repack_kq<JAL_Q4_K><<<blocks, 128, 0, s>>>(raw, rows, nsb, raw_row, qs, qs_stride, ks, km, k_stride);
  else if (quant == JAL_Q5_K) k_repack_kq<JAL_Q5_K><<<blocks, 128, 0, s>>>(raw, rows, nsb, raw_row, qs, qs_stride, ks, km, k_stride);
  else k_repack_kq<JAL_Q6_K><<<blocks, 128, 0, s>>>(raw, rows, nsb, raw_row, qs, qs_stride, ks, km, k_stride);
}

void launch_kq_gemm(const DevMat &w, const float *x, const int8_t *xq, const float *xs, int64_t m, float *y,
                    cudaStream_t s) {
  if (m <= 0 || w.rows <= 0) return;
  const int group = kquant_group(w.quant);
  const size_t smem = kq_smem(w.cols, group);
  if (smem > 220 * 1024) fail(JAL_ERR_CAPABILITY_MISMATCH, "K-quant projection: %lld columns do not fit", (long long)w.cols);
  const dim3 grid((unsigned)((w.rows + kKqWarps - 1) / kKqWarps), (unsigned)m);
  if (w.km) {
    cudaFuncSetAttribute(k_kq_gemm<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_kq_gemm<true><<<grid, kKqThreads, smem, s>>>(w, x, xq, xs, y, group);
  } else {
    cudaFuncSetAttribute(k_kq_gemm<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_kq_gemm<false><<<grid, kKqThreads, smem, s>>>(w, x, xq, xs, y, group);
  }
}

// The reference's portable layout (repack_cache.rs:639-694) on the host:
// tiles [(row / 8) * k_chunks + chunk][row % 8][16], scales and mins
// [(row / 8) * groups + group][row % 8].
void export_kquant_ref(const DevMat &w, int8_t *tiles, float *scales, float *mins) {
  const int64_t rows = w.rows, K = w.cols, nch = K / 16, ng = K / kquant_group(w.quant), nt = (rows + 7) / 8;
  std::vector<int8_t> q((size_t)rows * K);
  std::vector<float> sc((size_t)rows * ng), mn(w.km ? (size_t)rows * ng : 0);
  JAL_CUDA(cudaMemcpy2D(q.data(), K, w.qs, w.qs_stride, K, rows, cudaMemcpyDeviceToHost));
  JAL_CUDA(cudaMemcpy2D(sc.data(), ng * 4, w.ks, w.k_stride * 4, ng * 4, rows, cudaMemcpyDeviceToHost));
  if (w.km) JAL_CUDA(cudaMemcpy2D(mn.data(), ng * 4, w.km, w.k_stride * 4, ng * 4, rows, cudaMemcpyDeviceToHost));
  if (tiles) memset(tiles, 0, (size_t)nt * nch * 128);
  if (scales) memset(scales, 0, (size_t)nt * ng * 8 * 4);
  if (mins) memset(mins, 0, (size_t)nt * ng * 8 * 4);
  for (int64_t r = 0; r < rows; r++) {
    const int64_t t = r / 8, j = r % 8;
    if (tiles)
      for (int64_t c = 0; c < nch; c++) memcpy(tiles + (t * nch + c) * 128 + j * 16, &q[r * K + c * 16], 16);
    for (int64_t g = 0; g < ng; g++) {
      if (scales) scales[(t * ng + g) * 8 + j] = sc[r * ng + g];
      if (mins && w.km) mins[(t * ng + g) * 8 + j] = mn[r * ng + g];
    }
  }
}

}  // namespace jal
