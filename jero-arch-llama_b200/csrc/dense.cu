// Dense (F16 / BF16 / F32) decode GEMV: the streaming LM head of models whose
// output.weight is stored unquantized (repack_cache.rs:1978-2013,
// dispatch.rs:241-276).  Rows stay in their GGUF element type in HBM (2 or 4
// bytes per weight) and are sanitised on load exactly as repack_dense does
// (repack_cache.rs:613-637: f16 / bf16 Inf and NaN to +-0.0625, f32 through
// sanitize_f32_weight); the activation is the f32 row (RMSNorm'd for
// GEMV_IN_NORM) with non-finite values zeroed, as QuantizedActQ8 keeps it.
//
// Fast kernel: one CTA of 16 warps per SM over a contiguous row range; a
// warp streams one row at a time in 16-byte chunks (64 elements per lane in
// flight) against the activation in shared memory.  Reference-order
// kernel: one thread per row, acc += w * x in column order without
// contraction (eval_row_range's dense branch, repack_cache.rs:739-751).
#include <cuda_fp16.h>

#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "gemv_dev.cuh"
#include "jal.h"

namespace jal {

namespace {

constexpr int kDenseWarps = 16;

template <int QUANT>
struct DenseElt {
  static constexpr int kBytes = QUANT == JAL_F32 ? 4 : 2;
  static constexpr int kPerChunk = 16 / kBytes;  // elements per 16-byte chunk
  // chunks in flight per lane: 64 elements either way (measured on the
  // 128256x4096 head: 4.8 TB/s for F16 with 8, 5.1 TB/s for F32 with 16)
  static constexpr int kUnroll = QUANT == JAL_F32 ? 16 : 8;
  __device__ static float at(const void *p, int64_t i) {
    if (QUANT == JAL_F32) return sanitize_weight(((const float *)p)[i]);
    if (QUANT == JAL_F16) return f16_finite(((const uint16_t *)p)[i]);
    return bf16_finite(((const uint16_t *)p)[i]);
  }
  // Dot of one 16-byte chunk with kPerChunk activation values.
  __device__ static float dot(const uint4 v, const float *x, float acc) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    if (QUANT == JAL_F32) {
#pragma unroll
      for (int k = 0; k < 4; k++) acc = fmaf(sanitize_weight(__uint_as_float(u[k])), x[k], acc);
    } else {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const uint16_t lo = (uint16_t)(u[k] & 0xFFFFu), hi = (uint16_t)(u[k] >> 16);
        const float w0 = QUANT == JAL_F16 ? f16_finite(lo) : bf16_finite(lo);
        const float w1 = QUANT == JAL_F16 ? f16_finite(hi) : bf16_finite(hi);
        acc = fmaf(w0, x[2 * k], acc);
        acc = fmaf(w1, x[2 * k + 1], acc);
      }
    }
    return acc;
  }
};

template <int QUANT>
__global__ void __launch_bounds__(kDenseWarps * 32, 1) k_gemv_dense(const GemvArgs a) {
  using E = DenseElt<QUANT>;
  extern __shared__ __align__(16) float xs[];  // [cols] activation
  __shared__ float red[33];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int64_t cols = a.w.cols;
  const int64_t base = a.rows / gridDim.x, rem = a.rows % gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * base + ((int64_t)blockIdx.x < rem ? blockIdx.x : rem);
  const int64_t cnt = base + ((int64_t)blockIdx.x < rem ? 1 : 0);
  pdl_wait();
  pdl_trigger();
  // Activation: RMSNorm (same formula as the quantizing prologues) or f32.
  float ss = 0.0f;
  for (int64_t c = tid; c < cols; c += kDenseWarps * 32) {
    const float v = a.x[c];
    xs[c] = v;
    ss = fmaf(v, v, ss);
  }
  float invn = 1.0f;
  const bool norm = a.in_mode == GEMV_IN_NORM;
  if (norm) {
    const float tot = gdev::block_reduce_sum<kDenseWarps>(ss, red);
    invn = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)cols), a.eps)));
  }
  for (int64_t c = tid; c < cols; c += kDenseWarps * 32) {  // each thread rewrites its own elements
    float t = xs[c];
    if (norm) t = __fmul_rn(__fmul_rn(t, invn), a.norm_w[c]);
    xs[c] = isfinite(t) ? t : 0.0f;
  }
  __syncthreads();

  const int64_t nch = cols / E::kPerChunk;
  for (int64_t r = r0 + warp; r < r0 + cnt; r += kDenseWarps) {
    const uint4 *row = (const uint4 *)((const char *)a.w.dense + r * cols * E::kBytes);
    float acc = 0.0f;
    for (int64_t c0 = lane; c0 < nch; c0 += 32 * E::kUnroll) {
      uint4 v[E::kUnroll];
#pragma unroll
      for (int u = 0; u < E::kUnroll; u++) {
        const int64_t c = c0 + 32 * u;
        v[u] = c < nch ? ldg_stream16(row + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < E::kUnroll; u++) {
        const int64_t c = c0 + 32 * u;
        if (c < nch) acc = E::dot(v[u], xs + c * E::kPerChunk, acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) a.y[r] = a.bias ? acc + a.bias[r] : acc;
  }
}

template <int QUANT>
__global__ void k_strict_gemv_dense(const DevMat w, const float *__restrict__ x, int64_t rows,
                                    float *__restrict__ y) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const void *row = (const char *)w.dense + r * w.cols * DenseElt<QUANT>::kBytes;
  float acc = 0.0f;
  for (int64_t c = 0; c < w.cols; c++) {
    const float xv = x[c];
    acc = __fadd_rn(acc, __fmul_rn(DenseElt<QUANT>::at(row, c), isfinite(xv) ? xv : 0.0f));
  }
  y[r] = acc;
}

template <int QUANT>
void launch_dense_t(const GemvArgs &a, int grid, size_t smem, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_gemv_dense<QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kDenseWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_gemv_dense<QUANT>, a);
}

}  // namespace

bool dense_quant(int q) { return q == JAL_F32 || q == JAL_F16 || q == JAL_BF16; }

void launch_gemv_dense(const GemvArgs &a, cudaStream_t s) {
  if (a.rows <= 0) return;
  if (!dense_quant(a.w.quant) || !a.w.dense)
    fail(JAL_ERR_INVALID_ARGUMENT, "dense GEMV on a matrix of quant %d", a.w.quant);
  if (a.m != 1 || (a.in_mode != GEMV_IN_NORM && a.in_mode != GEMV_IN_F32) || a.out_mode != GEMV_OUT_STORE ||
      a.peer_in || a.w.cols % 32 != 0)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "dense GEMV: one token, f32 or RMSNorm input, stored rows, cols a multiple of 32");
  const size_t smem = (size_t)a.w.cols * 4;
  if (smem > (size_t)kGemvMaxSmem) fail(JAL_ERR_CAPABILITY_MISMATCH, "dense GEMV: %lld columns", (long long)a.w.cols);
  int grid = a.grid;
  if (grid <= 0) {
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    grid = (int)(a.rows < sms ? a.rows : sms);
  }
  if (a.w.quant == JAL_F16) launch_dense_t<JAL_F16>(a, grid, smem, s);
  else if (a.w.quant == JAL_BF16) launch_dense_t<JAL_BF16>(a, grid, smem, s);
  else launch_dense_t<JAL_F32>(a, grid, smem, s);
}

void launch_strict_gemv_dense(const DevMat &w, const float *x, int64_t rows, float *y, cudaStream_t s) {
  if (rows <= 0) return;
  const unsigned blocks = (unsigned)((rows + 127) / 128);
  if (w.quant == JAL_F16) k_strict_gemv_dense<JAL_F16><<<blocks, 128, 0, s>>>(w, x, rows, y);
  else if (w.quant == JAL_BF16) k_strict_gemv_dense<JAL_BF16><<<blocks, 128, 0, s>>>(w, x, rows, y);
  else k_strict_gemv_dense<JAL_F32><<<blocks, 128, 0, s>>>(w, x, rows, y);
}

}  // namespace jal
