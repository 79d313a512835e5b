// Decode attention output in the reference's f32 order (the last loop of
// gqa_attention_prefill_portable, recipe.rs:3008-3019):
//   out_d = sum over the active positions t, in order, of w_t * v_td
// from +0.0, one rounding per product and per sum, where w_t = e_t * inv was
// formed by the score kernel (xattn.cu) and stored per position.
//
// The sum is a chain of n_ctx dependent adds per (head, dim), so its speed is
// the per-step latency of one chain.  A warp that also loads, converts and
// multiplies issues four to five instructions per step and runs at ~12
// cycles a step; fed ready products, four at a time, it runs at the add
// latency (~4.7 cycles).  So one CTA per (query head, 32 dims):
//   - a loader thread streams the 32-dim slice of each V stage (R positions
//     inside one page) with 2D tensor copies (no multicast) into a ring;
//   - producer warps form the products w_t * v_td of a stage into a product
//     ring;
//   - one chain warp (lane = dim) adds a stage's products in order.
// Stages whose rows predate this step are fetched before
// griddepcontrol.wait; the stage holding the current position, written by
// the score kernel, after it.  The chain warp then writes the output slice
// and its QuantizedActQ8 block (32 dims = one block) for the O projection.
// Every wait is bounded: a wait that gives up sets bit value 2 of the
// context's error word and the kernel runs to its end.
#include <cuda.h>
#include <cuda_fp16.h>

#include "attn_dev.cuh"
#include "common.hpp"
#include "dev_util.cuh"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr int kVS = 6;        // V stages in flight
constexpr int kPS = 4;        // product stages
constexpr int kProd = 2;      // producer warps
constexpr int kVT = 32 * (2 + kProd);  // chain warp, producer warps, loader warp
constexpr int kMaxR = 64;     // positions per stage
constexpr int kErrCopyWait = 2;
// Product stage: [32 dims][kPStr] floats, a dim's positions contiguous so the
// chain lane reads four of them with one 16-byte load.  Position r of dim d
// sits at column r ^ (8 (d / 8)): the producers' stores (8 positions x 4 dim
// groups per warp instruction) then hit 32 different banks, and the chain's
// 16-byte reads (row stride 68 words, 8 lanes per phase) stay conflict-free.
constexpr int kPStr = kMaxR + 4;
__device__ __forceinline__ int pcol(int r, int d) { return r ^ (8 * (d >> 3)); }

template <bool F16>
struct VA {
  static constexpr int ES = F16 ? 2 : 4;
  static constexpr int SROW = 32 * ES;     // bytes of one position's 32-dim slice
  static constexpr int CH = 16 / ES;       // elements per 16-byte piece
  static constexpr int LPR = SROW / 16;    // producer lanes per position
  static constexpr int RPG = 32 / LPR;     // positions per producer warp step
  static constexpr int STAGE = kMaxR * SROW;
};

struct VLayout {
  size_t vring, prod, w, srow, total;
};

__host__ __device__ inline int v_max_stages(int n_ctx) { return n_ctx / 8 + 2; }

template <bool F16>
__host__ __device__ inline VLayout v_layout(int n_ctx) {
  VLayout L;
  size_t o = 0;
  L.vring = o; o += (size_t)kVS * VA<F16>::STAGE;       // 128-byte aligned pieces (tensor copy targets)
  L.prod = o; o += (size_t)kPS * 32 * kPStr * 4;
  L.w = o; o += ((size_t)n_ctx * 4 + 127) / 128 * 128;
  L.srow = o; o += ((size_t)v_max_stages(n_ctx) * 16 + 127) / 128 * 128;
  L.total = o;
  return L;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <bool F16>
__global__ void __launch_bounds__(kVT, 1) k_xattn_v(const __grid_constant__ CUtensorMap tmv, const AttnVArgs a, int n_ctx,
                                                   int R) {
  const KernelTrace trace(a.trace);
  using A = VA<F16>;
  extern __shared__ __align__(128) char smem[];
  __shared__ __align__(8) uint64_t vfull[kVS], vempty[kVS], pfull[kPS], pempty[kPS];
  __shared__ int bad_s;
  const VLayout L = v_layout<F16>(n_ctx);
  char *vring = smem + L.vring;
  float *prod = (float *)(smem + L.prod);
  float *w_s = (float *)(smem + L.w);
  int4 *srow = (int4 *)(smem + L.srow);  // {tensor row, first position, positions, 0} per stage

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int hd = (int)a.kv.head_dim, nsl = hd / 32;
  const int hq = blockIdx.x / nsl, sl = blockIdx.x % nsl;
  const int G = (int)(a.n_heads_q / a.kv.n_kv), h = hq / G;
  const int64_t pos = *a.d_pos, seq = pos + 1;
  const int64_t lo = (a.window > 0 && seq > a.window) ? seq - a.window : 0;
  const int nv = seq > lo ? (int)((seq + R - 1) / R - lo / R) : 0;

  if (tid == 0) {
    for (int s = 0; s < kVS; s++) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], kProd);
    }
    for (int s = 0; s < kPS; s++) {
      mbar_init(&pfull[s], kProd);
      mbar_init(&pempty[s], 1);
    }
    bad_s = 0;
    fence_barrier_init();
  }
  // Stage k: positions [max(lo, (lo / R + k) R), min(seq, (lo / R + k + 1) R)),
  // inside one page; its tensor row is the first position's.
  for (int k = tid; k < nv; k += kVT) {
    const int64_t base = (lo / R + k) * R;
    const int64_t t0 = base > lo ? base : lo, t1 = base + R < seq ? base + R : seq;
    const int64_t page = a.kv.page_table[t0 / a.kv.page_size], slot = t0 % a.kv.page_size;
    const int64_t row = ((a.layer * a.kv.n_pages + page) * a.kv.n_kv + h) * a.kv.page_size + slot;
    srow[k] = make_int4((int)row, (int)t0, (int)(t1 - t0), 0);
  }
  __syncthreads();
  bool ok = true;

  if (warp == 1 + kProd) {  // loader
    if (lane == 0) {
      // (The test hook's extra bytes go on the last stage, whose barrier no
      // later stage re-arms.)
      const uint32_t bytes = (uint32_t)(R * A::SROW);
      // Rows written before this step first (the current position's stage
      // is the score kernel's output).
      int issued = 0;
      for (; issued < nv && issued < kVS; issued++) {
        const int4 st = srow[issued];
        if (st.y + st.z > pos) break;
        mbar_expect_tx(&vfull[issued], bytes + (issued == nv - 1 ? a.test_extra_tx : 0u));
        tma_load_2d(vring + issued * A::STAGE, &tmv, 32 * sl, st.x, &vfull[issued]);
      }
      pdl_wait();
      trace.mark(0);  // the grid dependency resolved
      for (int k = issued; k < nv; k++) {
        const int slot = k % kVS;
        if (k >= kVS && !mbar_wait_sleepy(&vempty[slot], (uint32_t)(((k - kVS) / kVS) & 1), a.wait_ns)) ok = false;
        fence_proxy_async();
        const int4 st = srow[k];
        mbar_expect_tx(&vfull[slot], bytes + (k == nv - 1 ? a.test_extra_tx : 0u));
        tma_load_2d(vring + slot * A::STAGE, &tmv, 32 * sl, st.x, &vfull[slot]);
      }
    }
  } else {
    pdl_wait();
    // Weights of this head, by position (the score kernel's output).
    const float *wg = a.w + (int64_t)hq * a.w_stride;
    for (int64_t t = lo + (tid - 0); t < seq; t += 32 * (1 + kProd)) w_s[t - lo] = wg[t];
    asm volatile("bar.sync 1, %0;" ::"n"(32 * (1 + kProd)) : "memory");
    if (tid == 0) trace.mark(1);  // weights in shared memory
    if (warp == 0) {  // chain: lane = dim
      float o = 0.0f;
      int ps = 0;
      uint32_t pp = 0;
      for (int k = 0; k < nv; k++) {
        if (!mbar_wait_bounded(&pfull[ps], pp, a.wait_ns)) ok = false;
        if (k == 0 && lane == 0) trace.mark(2);  // first product stage ready
        const int n = srow[k].z;
        const float *pr = prod + ((size_t)ps * 32 + lane) * kPStr;  // this dim's row
        const int sw = 8 * (lane >> 3);
        if (n == kMaxR) {  // a full stage: block b + 1's loads go out before block b's adds
          float4 x[2][4];
#pragma unroll
          for (int u = 0; u < 4; u++) x[0][u] = *(const float4 *)(pr + ((4 * u) ^ sw));
#pragma unroll
          for (int b = 0; b < kMaxR / 16; b++) {
            if (b + 1 < kMaxR / 16) {
#pragma unroll
              for (int u = 0; u < 4; u++) x[(b + 1) & 1][u] = *(const float4 *)(pr + ((16 * (b + 1) + 4 * u) ^ sw));
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
              const float4 v = x[b & 1][u];
              o = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(o, v.x), v.y), v.z), v.w);
            }
          }
        } else {
          for (int r = 0; r < n; r++) o = __fadd_rn(o, pr[r ^ sw]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&pempty[ps]);
        if (++ps == kPS) {
          ps = 0;
          pp ^= 1u;
        }
      }
      if (lane == 0) trace.mark(3);  // chain done
      const int64_t e = (int64_t)hq * hd + 32 * sl + lane;
      a.out[e] = o;
      const float v = isfinite(o) ? o : 0.0f;
      const float amax = warp_max(fabsf(v));
      const float scale = act_scale_from_amax(amax), is = act_inv_from_scale(scale);
      a.out_q[e] = act_quant_one(v, is);
      if (lane == 0) a.out_s[e / 32] = scale;
    } else {  // producer p: positions p, p + kProd, ... (in steps of RPG) of each stage
      const int p = warp - 1, rr = lane / A::LPR, q = lane % A::LPR;
      int vs = 0, ps = 0;
      uint32_t vp = 0, pp = 0;
      for (int k = 0; k < nv; k++) {
        if (!mbar_wait_bounded(&vfull[vs], vp, a.wait_ns)) ok = false;
        if (k >= kPS && !mbar_wait_bounded(&pempty[ps], pp ^ 1u, a.wait_ns)) ok = false;
        const int4 st = srow[k];
        const char *vsrc = vring + vs * A::STAGE;
        float *dst = prod + (size_t)ps * 32 * kPStr;
        const float *wst = w_s + (st.y - lo);
        auto make = [&](int r, uint4 raw, float wv) {  // products of position r, dims CH q .. CH q + CH - 1
          float pv[A::CH];
          if (F16) {
            const __half2 *hh = (const __half2 *)&raw;
#pragma unroll
            for (int j = 0; j < A::CH / 2; j++) {
              const float2 f = __half22float2(hh[j]);
              pv[2 * j] = __fmul_rn(wv, f.x);
              pv[2 * j + 1] = __fmul_rn(wv, f.y);
            }
          } else {
            pv[0] = __fmul_rn(wv, __uint_as_float(raw.x));
            pv[1] = __fmul_rn(wv, __uint_as_float(raw.y));
            pv[2] = __fmul_rn(wv, __uint_as_float(raw.z));
            pv[3] = __fmul_rn(wv, __uint_as_float(raw.w));
          }
#pragma unroll
          for (int j = 0; j < A::CH; j++) {
            const int d = A::CH * q + j;
            dst[d * kPStr + pcol(r, d)] = pv[j];
          }
        };
        if (st.z == kMaxR) {  // a full stage: all of this warp's loads first, then the products
          constexpr int GPP = kMaxR / A::RPG / kProd;  // position groups per producer warp
          uint4 raw[GPP];
          float wv[GPP];
#pragma unroll
          for (int i = 0; i < GPP; i++) {
            const int r = (p + kProd * i) * A::RPG + rr;
            raw[i] = *(const uint4 *)(vsrc + r * A::SROW + 16 * q);
            wv[i] = wst[r];
          }
#pragma unroll
          for (int i = 0; i < GPP; i++) make((p + kProd * i) * A::RPG + rr, raw[i], wv[i]);
        } else {
          for (int g = p; g * A::RPG < st.z; g += kProd) {
            const int r = g * A::RPG + rr;
            if (r < st.z) make(r, *(const uint4 *)(vsrc + r * A::SROW + 16 * q), wst[r]);
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&pfull[ps]);
          mbar_arrive(&vempty[vs]);
        }
        if (++vs == kVS) {
          vs = 0;
          vp ^= 1u;
        }
        if (++ps == kPS) {
          ps = 0;
          pp ^= 1u;
        }
      }
    }
  }
  if (!ok) atomicOr(&bad_s, 1);
  __syncthreads();
  if (bad_s && tid == 0 && a.err) atomicOr(a.err, kErrCopyWait);
}

template <bool F16>
void launch_v(const CUtensorMap &tm, const AttnVArgs &a, int n_ctx, int R, cudaStream_t s) {
  const size_t smem = v_layout<F16>(n_ctx).total;
  cudaFuncSetAttribute(k_xattn_v<F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.n_heads_q * (a.kv.head_dim / 32)));
  cfg.blockDim = dim3(kVT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = a.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_xattn_v<F16>, tm, a, n_ctx, R);
}

}  // namespace

bool xattn_v_supported(int64_t head_dim, int64_t page_size, int64_t n_ctx) {
  if (head_dim % 32 != 0 || head_dim > 256 || page_size % 8 != 0) return false;
  return v_layout<false>((int)n_ctx).total <= 220 * 1024;
}

bool make_kv_tensor_map(const KvView &kv, const void *base, void *tm_out) {
  using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = (Encode)fn;
  }
  const int esz = kv.f16 ? 2 : 4;
  const int R = kv_stage_rows(kv.page_size);
  const cuuint64_t dims[2] = {(cuuint64_t)kv.head_dim,
                              (cuuint64_t)(kv.n_layers * kv.n_pages * kv.n_kv * kv.page_size)};
  const cuuint64_t strides[1] = {(cuuint64_t)(kv.head_dim * esz)};
  const cuuint32_t box[2] = {32u, (cuuint32_t)R}, estr[2] = {1u, 1u};
  CUtensorMap *tm = (CUtensorMap *)tm_out;
  return encode(tm, kv.f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims,
                strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int kv_stage_rows(int64_t page_size) {
  int R = 1;
  while (R * 2 <= kMaxR && page_size % (R * 2) == 0) R *= 2;
  return R;
}

void launch_xattn_v(const void *tm, const AttnVArgs &a, int64_t n_ctx, cudaStream_t s) {
  if (!xattn_v_supported(a.kv.head_dim, a.kv.page_size, n_ctx))
    fail(JAL_ERR_CAPABILITY_MISMATCH, "reference-order decode attention output: unsupported shape");
  const int R = kv_stage_rows(a.kv.page_size);
  const CUtensorMap &m = *(const CUtensorMap *)tm;
  if (a.kv.f16) launch_v<true>(m, a, (int)n_ctx, R, s);
  else launch_v<false>(m, a, (int)n_ctx, R, s);
}

}  // namespace jal
