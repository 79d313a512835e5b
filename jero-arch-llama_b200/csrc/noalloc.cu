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
// exits.  Host code cannot use the array's name as a device address, so each
// call looks the address up with cudaGetSymbolAddress on the current device
// (a cheap table lookup once the image is loaded there; looking it up every
// time also stays right after a device reset reloads the image elsewhere) and
// passes it to the kernels.  The first call on a device may load the image,
// so it must not be made inside a stream capture.
#include <cuda_runtime.h>

#include "common.hpp"
#include "device.hpp"
#include "jal.h"

namespace jal {

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)2 << 20;  // 2 MiB

static __device__ __align__(256) unsigned char g_gemm_scratch[kNoAllocScratchBytes];

// Device address of g_gemm_scratch on `dev`, which must be the current device.
void *scratch_address(int dev) {
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_scratch);
  if (e != cudaSuccess || !p) {
    cudaGetLastError();
    fail(JAL_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
  }
  return p;
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
  project_q8(w, q8, sc, m, y, s);
  JAL_CUDA(cudaGetLastError());
}

}  // namespace jal
