// Prefill GEMM over the repacked Q4_0 / Q8_0 layout on the int8 tensor
// cores (mma.sync m16n8k16, s8 x s8 -> s32), in the reference's f32 order.
//
// y[t][r] = the left-to-right f32 sum from +0.0, over the 16-element chunks
// of the row in order, of (f32(dot16) * a_sc[t][b]) * w_sc[r][b]
// (repack_cache.rs:739-783, gemm_rows :808-837); bias and the residual are
// added after the fold.  Each 32-block is two m16n8k16 MMAs, one per chunk,
// so every chunk's integer dot (|dot16| < 2^24, exact in f32) gets its own
// term, and the accumulator of each (token, row) takes the terms in chunk
// order: the result equals the reference bit for bit.
//
// CTA tile: 128 tokens x 128 rows, 8 warps, K staged 4 blocks (128
// elements) at a time in shared memory, two stages alternating: the next
// stage's blocks are in flight (cp.async) while the current one is used.  Warp w computes tokens
// 16w..16w+15 against the 128 rows as 16 n-tiles of 8 rows.  MMA fragments
// (PTX m16n8k16 .s8, g = lane / 4, q = lane % 4): A (tokens x 16, row-major)
// regs = (token g, k 4q..4q+3), (g + 8, 4q..); B (16 x 8 rows, column-major)
// reg = (row g, k 4q..4q+3); C = tokens g and g + 8, rows 2q and 2q + 1.
// A Q4_0 block's byte i holds elements i (low nibble, chunk 0) and i + 16
// (high nibble, chunk 1), so one 32-bit load at byte 4q gives the B
// registers of both chunks.
#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int BM = 128, BN = 128, KB = 4;  // tokens, rows, 32-blocks per stage
constexpr int kThreads = 256, kNT = BN / 8;  // 8 warps; n-tiles of 8 rows per warp

__device__ __forceinline__ void mma_s8_16816(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// Term of one chunk: (f32(dot16) * a_sc) * w_sc.
__device__ __forceinline__ float chunk_term(int dot, float as, float ws) {
  return __fmul_rn(__fmul_rn(__int2float_rn(dot), as), ws);
}

// Four nibbles 0..15 (one per byte) to signed bytes n - 8.
__device__ __forceinline__ uint32_t nib_s8(uint32_t v) { return ((v | 0x80808080u) - 0x08080808u) ^ 0x80808080u; }

// One K stage of the CTA tile in shared memory (two of them alternate).
template <int WB>
struct GemmStage {
  uint8_t w[KB][BN][WB];  // weight blocks, rows 16-byte aligned
  int8_t x[KB][BM][32];   // activation blocks
  float wd[KB][BN];       // weight block scales
  float as[KB][BM];       // activation block scales
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0) : "memory");
}

template <int QUANT>
__global__ void __launch_bounds__(kThreads) k_gemm(const GemmArgs a) {
  constexpr int WB = QUANT == JAL_Q4_0 ? 16 : 32;  // weight bytes per block
  constexpr int NSW = KB * BN / kThreads, NSA = KB * BM / kThreads;  // scales per thread per stage
  using Stage = GemmStage<WB>;
  extern __shared__ __align__(16) char gsm[];
  Stage *st = reinterpret_cast<Stage *>(gsm);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32, g = lane / 4, q = lane % 4;
  const int64_t t0 = (int64_t)blockIdx.y * BM, r0 = (int64_t)blockIdx.x * BN;
  const int64_t K = a.w.cols, nb = K / 32;
  float acc[kNT][4];
#pragma unroll
  for (int n = 0; n < kNT; n++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[n][i] = 0.0f;

  // Quant and activation blocks of a stage go to shared memory by cp.async
  // (zero-filled outside the matrix); the scales pass through registers.
  auto issue = [&](Stage &sb, int64_t b0) {
    for (int i = tid; i < KB * BN * (WB / 16); i += kThreads) {
      const int piece = i % (WB / 16), rr = (i / (WB / 16)) % BN, kb = i / (WB / 16) / BN;
      const int64_t r = r0 + rr, b = b0 + kb;
      const bool ok = r < a.rows && b < nb;
      cp_async16(&sb.w[kb][rr][piece * 16], ok ? a.w.qs + r * a.w.qs_stride + b * WB + piece * 16 : a.w.qs, ok);
    }
    for (int i = tid; i < KB * BM * 2; i += kThreads) {
      const int half = i % 2, tt = (i / 2) % BM, kb = i / 2 / BM;
      const int64_t t = t0 + tt, b = b0 + kb;
      const bool ok = t < a.m && b < nb;
      cp_async16(&sb.x[kb][tt][half * 16], ok ? a.xq + t * K + b * 32 + half * 16 : a.xq, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float wreg[NSW], areg[NSA];
  auto load_scales = [&](int64_t b0) {
#pragma unroll
    for (int j = 0; j < NSW; j++) {
      const int i = tid + j * kThreads, rr = i % BN, kb = i / BN;
      const int64_t r = r0 + rr, b = b0 + kb;
      wreg[j] = (r < a.rows && b < nb) ? f16_finite(a.w.d[r * a.w.d_stride + b]) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < NSA; j++) {
      const int i = tid + j * kThreads, tt = i % BM, kb = i / BM;
      const int64_t t = t0 + tt, b = b0 + kb;
      areg[j] = (t < a.m && b < nb) ? a.xs[t * nb + b] : 0.0f;
    }
  };
  auto store_scales = [&](Stage &sb) {
#pragma unroll
    for (int j = 0; j < NSW; j++) {
      const int i = tid + j * kThreads;
      sb.wd[i / BN][i % BN] = wreg[j];
    }
#pragma unroll
    for (int j = 0; j < NSA; j++) {
      const int i = tid + j * kThreads;
      sb.as[i / BM][i % BM] = areg[j];
    }
  };

  const int64_t nst = (nb + KB - 1) / KB;
  issue(st[0], 0);
  load_scales(0);
  store_scales(st[0]);
  for (int64_t sidx = 0; sidx < nst; sidx++) {
    Stage &cur = st[sidx & 1];
    if (sidx + 1 < nst) {  // the other buffer was last read before the previous barrier
      issue(st[(sidx + 1) & 1], (sidx + 1) * KB);
      load_scales((sidx + 1) * KB);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
#pragma unroll
    for (int kb = 0; kb < KB; kb++) {
      const int ta = warp * 16 + g;  // tokens ta and ta + 8
      const uint32_t alo0 = *(const uint32_t *)&cur.x[kb][ta][4 * q];
      const uint32_t alo1 = *(const uint32_t *)&cur.x[kb][ta + 8][4 * q];
      const uint32_t ahi0 = *(const uint32_t *)&cur.x[kb][ta][16 + 4 * q];
      const uint32_t ahi1 = *(const uint32_t *)&cur.x[kb][ta + 8][16 + 4 * q];
      const float as0 = cur.as[kb][ta], as1 = cur.as[kb][ta + 8];
#pragma unroll
      for (int n = 0; n < kNT; n++) {
        const int rb = n * 8 + g;  // this lane's B row
        uint32_t blo, bhi;
        if (QUANT == JAL_Q4_0) {
          const uint32_t w = *(const uint32_t *)&cur.w[kb][rb][4 * q];
          blo = nib_s8(w & 0x0F0F0F0Fu);
          bhi = nib_s8((w >> 4) & 0x0F0F0F0Fu);
        } else {
          blo = *(const uint32_t *)&cur.w[kb][rb][4 * q];
          bhi = *(const uint32_t *)&cur.w[kb][rb][16 + 4 * q];
        }
        int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
        mma_s8_16816(c0, alo0, alo1, blo);  // chunk 0: elements 0..15
        mma_s8_16816(c1, ahi0, ahi1, bhi);  // chunk 1: elements 16..31
        const float ws0 = cur.wd[kb][n * 8 + 2 * q], ws1 = cur.wd[kb][n * 8 + 2 * q + 1];
        acc[n][0] = __fadd_rn(__fadd_rn(acc[n][0], chunk_term(c0[0], as0, ws0)), chunk_term(c1[0], as0, ws0));
        acc[n][1] = __fadd_rn(__fadd_rn(acc[n][1], chunk_term(c0[1], as0, ws1)), chunk_term(c1[1], as0, ws1));
        acc[n][2] = __fadd_rn(__fadd_rn(acc[n][2], chunk_term(c0[2], as1, ws0)), chunk_term(c1[2], as1, ws0));
        acc[n][3] = __fadd_rn(__fadd_rn(acc[n][3], chunk_term(c0[3], as1, ws1)), chunk_term(c1[3], as1, ws1));
      }
    }
    __syncthreads();  // every warp is done with `cur` before it is refilled
    if (sidx + 1 < nst) store_scales(st[(sidx + 1) & 1]);
  }
#pragma unroll
  for (int n = 0; n < kNT; n++) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t t = t0 + warp * 16 + g + (i < 2 ? 0 : 8);
      const int64_t r = r0 + n * 8 + 2 * q + (i & 1);
      if (t >= a.m || r >= a.rows) continue;
      float v = acc[n][i];
      if (a.bias) v = __fadd_rn(v, a.bias[r]);
      float *yp = a.y + t * a.y_stride + r;
      *yp = a.accumulate ? __fadd_rn(*yp, v) : v;
    }
  }
}

// ---- few tokens (M <= 16): batched decode ---------------------------------
// The same chunk dots and the same per-(token, row) fold as k_gemm, tiled for
// a skinny M: one m16 tile of tokens, CTAs of 32 rows (4 warps, one n-tile of
// 8 rows each) so that even 3584-row projections spread over ~110 CTAs, and a
// 4-stage cp.async ring of 16 blocks per stage for the bytes in flight.
// Everything past the matrix or the token count is zero-filled and adds +0
// terms, which leave every row's sum unchanged.
constexpr int SBM = 16, SBN = 32, SKB = 16, SNS = 4, kSkThreads = 128;

// Stage tiles keep each row's (token's) 16 blocks contiguous, so one warp's
// copies read 512 consecutive bytes of a row, and pad rows by 16 bytes, so
// the 8 rows (tokens) of an MMA fragment fall in different banks.
template <int WB>
struct SkStage {
  static constexpr int WP = SKB * WB + 16, XP = SKB * 32 + 16;
  uint8_t w[SBN][WP];          // weight blocks of a row, in K order
  int8_t x[SBM][XP];           // activation blocks of a token, in K order
  uint16_t wd[SBN][SKB];       // weight block scales (f16 bits)
  float as[SBM][SKB + 1];      // activation block scales
};

__device__ __forceinline__ void cp_async4(void *smem, const void *gmem, bool valid) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(valid ? 4 : 0) : "memory");
}

template <int QUANT, bool HI>
__global__ void __launch_bounds__(kSkThreads) k_gemm_skinny(const GemmArgs a) {
  constexpr int WB = QUANT == JAL_Q4_0 ? 16 : 32;
  using Stage = SkStage<WB>;
  constexpr int WPC = SKB * WB / 16;  // 16-byte pieces of a row per stage
  extern __shared__ __align__(16) char gsm[];
  Stage *st = reinterpret_cast<Stage *>(gsm);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32, g = lane / 4, q = lane % 4;
  const int64_t r0 = (int64_t)blockIdx.x * SBN, K = a.w.cols, nb = K / 32;
  const int m = (int)a.m;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  auto issue = [&](int64_t sidx) {
    Stage &sb = st[sidx % SNS];
    const int64_t b0 = sidx * SKB;
    for (int i = tid; i < SBN * WPC; i += kSkThreads) {
      const int rr = i / WPC, off = i % WPC;
      const int64_t r = r0 + rr, b = b0 + off * 16 / WB;
      const bool ok = r < a.rows && b < nb;
      cp_async16(&sb.w[rr][off * 16], ok ? a.w.qs + r * a.w.qs_stride + b0 * WB + off * 16 : a.w.qs, ok);
    }
    for (int i = tid; i < SBM * SKB * 2; i += kSkThreads) {
      const int tt = i / (SKB * 2), off = i % (SKB * 2);
      const int64_t b = b0 + off / 2;
      const bool ok = tt < m && b < nb;
      cp_async16(&sb.x[tt][off * 16], ok ? a.xq + tt * K + b0 * 32 + off * 16 : a.xq, ok);
    }
    for (int i = tid; i < SBN * SKB / 2; i += kSkThreads) {  // two scales per copy (the run is padded to 8)
      const int rr = i / (SKB / 2), pr = i % (SKB / 2);
      const int64_t r = r0 + rr, b = b0 + 2 * pr;
      const bool ok = r < a.rows && b < nb;
      cp_async4(&sb.wd[rr][2 * pr], ok ? a.w.d + r * a.w.d_stride + b : a.w.d, ok);
    }
    for (int i = tid; i < SBM * SKB; i += kSkThreads) {
      const int tt = i / SKB, kb = i % SKB;
      const int64_t b = b0 + kb;
      const bool ok = tt < m && b < nb;
      cp_async4(&sb.as[tt][kb], ok ? a.xs + tt * nb + b : a.xs, ok);
    }
  };
  const int64_t nst = (nb + SKB - 1) / SKB;
  for (int s = 0; s < SNS - 1; s++) {
    if (s < nst) issue(s);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const int rb = warp * 8 + g;  // this lane's B row
  for (int64_t sidx = 0; sidx < nst; sidx++) {
    if (sidx + SNS - 1 < nst) issue(sidx + SNS - 1);  // into the slot freed at the end of the last stage
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(SNS - 1) : "memory");
    __syncthreads();
    const Stage &cur = st[sidx % SNS];
#pragma unroll 4
    for (int kb = 0; kb < SKB; kb++) {
      const uint32_t alo0 = *(const uint32_t *)&cur.x[g][kb * 32 + 4 * q];
      const uint32_t ahi0 = *(const uint32_t *)&cur.x[g][kb * 32 + 16 + 4 * q];
      const uint32_t alo1 = HI ? *(const uint32_t *)&cur.x[g + 8][kb * 32 + 4 * q] : 0u;
      const uint32_t ahi1 = HI ? *(const uint32_t *)&cur.x[g + 8][kb * 32 + 16 + 4 * q] : 0u;
      uint32_t blo, bhi;
      if (QUANT == JAL_Q4_0) {
        const uint32_t w = *(const uint32_t *)&cur.w[rb][kb * 16 + 4 * q];
        blo = nib_s8(w & 0x0F0F0F0Fu);
        bhi = nib_s8((w >> 4) & 0x0F0F0F0Fu);
      } else {
        blo = *(const uint32_t *)&cur.w[rb][kb * 32 + 4 * q];
        bhi = *(const uint32_t *)&cur.w[rb][kb * 32 + 16 + 4 * q];
      }
      int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
      mma_s8_16816(c0, alo0, alo1, blo);
      mma_s8_16816(c1, ahi0, ahi1, bhi);
      const float as0 = cur.as[g][kb];
      const float ws0 = f16_finite(cur.wd[warp * 8 + 2 * q][kb]), ws1 = f16_finite(cur.wd[warp * 8 + 2 * q + 1][kb]);
      acc[0] = __fadd_rn(__fadd_rn(acc[0], chunk_term(c0[0], as0, ws0)), chunk_term(c1[0], as0, ws0));
      acc[1] = __fadd_rn(__fadd_rn(acc[1], chunk_term(c0[1], as0, ws1)), chunk_term(c1[1], as0, ws1));
      if (HI) {
        const float as1 = cur.as[g + 8][kb];
        acc[2] = __fadd_rn(__fadd_rn(acc[2], chunk_term(c0[2], as1, ws0)), chunk_term(c1[2], as1, ws0));
        acc[3] = __fadd_rn(__fadd_rn(acc[3], chunk_term(c0[3], as1, ws1)), chunk_term(c1[3], as1, ws1));
      }
    }
    __syncthreads();  // every warp is done with this slot before it is refilled
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
  for (int i = 0; i < (HI ? 4 : 2); i++) {
    const int64_t t = g + (i < 2 ? 0 : 8);
    const int64_t r = r0 + warp * 8 + 2 * q + (i & 1);
    if (t >= a.m || r >= a.rows) continue;
    float v = acc[i];
    if (a.bias) v = __fadd_rn(v, a.bias[r]);
    float *yp = a.y + t * a.y_stride + r;
    *yp = a.accumulate ? __fadd_rn(*yp, v) : v;
  }
}

template <int QUANT>
void launch_skinny(const GemmArgs &a, cudaStream_t s) {
  constexpr size_t smem = SNS * sizeof(SkStage<QUANT == JAL_Q4_0 ? 16 : 32>);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_gemm_skinny<QUANT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(k_gemm_skinny<QUANT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  const dim3 grid((unsigned)((a.rows + SBN - 1) / SBN));
  if (a.m > 8) k_gemm_skinny<QUANT, true><<<grid, kSkThreads, smem, s>>>(a);
  else k_gemm_skinny<QUANT, false><<<grid, kSkThreads, smem, s>>>(a);
}

}  // namespace

void launch_gemm(const GemmArgs &a, cudaStream_t s) {
  if (a.m <= 0 || a.rows <= 0) return;
  // Few tokens with scale runs that 4-byte copies can read (16-byte rows,
  // scales padded to a multiple of 8): the skinny tiling.
  if (a.m <= SBM && a.w.d_stride % 8 == 0 && (reinterpret_cast<uintptr_t>(a.w.d) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(a.xs) & 3) == 0) {
    if (a.w.quant == JAL_Q4_0) launch_skinny<JAL_Q4_0>(a, s);
    else launch_skinny<JAL_Q8_0>(a, s);
    return;
  }
  dim3 grid((unsigned)((a.rows + BN - 1) / BN), (unsigned)((a.m + BM - 1) / BM));
  static bool attr = false;
  constexpr size_t s4 = 2 * sizeof(GemmStage<16>), s8 = 2 * sizeof(GemmStage<32>);
  if (!attr) {
    cudaFuncSetAttribute(k_gemm<JAL_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s4);
    cudaFuncSetAttribute(k_gemm<JAL_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s8);
    attr = true;
  }
  if (a.w.quant == JAL_Q4_0) k_gemm<JAL_Q4_0><<<grid, kThreads, s4, s>>>(a);
  else k_gemm<JAL_Q8_0><<<grid, kThreads, s8, s>>>(a);
}

}  // namespace jal
