// Allocation-free variant of the quantize-then-project path of
// jal_cached_matrix_gemm.
//
// Some callers cannot call cudaMalloc: a serving loop that has handed all
// free device memory to another allocator's pool (a new cudaMalloc would
// fail), or one that must not allocate once it is running because
// cudaMalloc/cudaFree can synchronise the whole device and stall other
// streams.  For them the int8 activations and their per-32-block scales live
// in one file-scope device array of fixed size instead of a per-call buffer.
//
// The array is part of this library's device image: every GPU on which the
// library's kernels are loaded holds kNoAllocScratchBytes until the process
// exits.  Host code cannot use the array's name as a device address, so its
// address is looked up with cudaGetSymbolAddress once per device (with that
// device current) on the first call there, and passed to the kernels.
#include <cuda_runtime.h>

#include <mutex>

#include "common.hpp"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)2 << 20;  // 2 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_gemm_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};

// Device address of g_gemm_scratch on `dev`, which must be the current device.
void *scratch_address(int dev) {
  if (dev < 0 || dev >= kMaxDevices) fail(JAL_ERR_INVALID_ARGUMENT, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      fail(JAL_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
    }
    g_addr[dev] = p;
  }
  return g_addr[dev];
}

size_t round256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

void gemm_noalloc(const DevMat &w, const float *x, int64_t m, float *y, cudaStream_t s) {
  const int64_t K = w.cols, nb = K / 32;
  // Layout of the scratch: q8 [m][K] int8, then (256-byte aligned) scales [m][nb] f32.
  if ((uint64_t)m > kNoAllocScratchBytes / (uint64_t)K)
    fail(JAL_ERR_TENSOR_BOUNDS, "no-alloc GEMM: m=%lld x cols=%lld needs more than the %zu-byte scratch",
         (long long)m, (long long)K, kNoAllocScratchBytes);
  const size_t q8_bytes = round256((size_t)m * (size_t)K), need = q8_bytes + (size_t)m * (size_t)nb * 4;
  if (need > kNoAllocScratchBytes)
    fail(JAL_ERR_TENSOR_BOUNDS, "no-alloc GEMM: m=%lld x cols=%lld needs %zu bytes of scratch, the maximum is %zu",
         (long long)m, (long long)K, need, kNoAllocScratchBytes);
  int dev = 0;
  JAL_CUDA(cudaGetDevice(&dev));
  char *base = (char *)scratch_address(dev);
  int8_t *q8 = (int8_t *)base;
  float *sc = (float *)(base + q8_bytes);
  // Every byte the kernels read below is written first by the quantizer, so
  // nothing has to start at zero.
  launch_act_quant(x, m, K, K, q8, sc, s);
  if (m <= kGemvMaxM) {
    GemvArgs a;
    a.w = w; a.rows = w.rows; a.m = (int)m; a.in_mode = GEMV_IN_Q8; a.xq = q8; a.xs = sc;
    a.xq_stride = K; a.out_mode = GEMV_OUT_STORE; a.y = y; a.y_stride = w.rows;
    launch_gemv(a, s);
  } else {
    GemmArgs a;
    a.w = w; a.m = m; a.rows = w.rows; a.xq = q8; a.xs = sc; a.y = y; a.y_stride = w.rows;
    launch_gemm(a, s);
  }
  JAL_CUDA(cudaGetLastError());
}

}  // namespace jal
