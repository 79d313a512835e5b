// Tensor-parallel shard plan and the NCCL calls it needs (loaded at run time).
#include "tp.hpp"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "common.hpp"

namespace jal {

TpPlan tp_plan(uint64_t n_heads_q, uint64_t n_heads_kv, uint64_t ffn_dim, uint64_t vocab, int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world) fail(JAL_ERR_INVALID_ARGUMENT, "tensor parallel rank %d of %d", rank, world);
  if (n_heads_kv % (uint64_t)world || n_heads_q % (uint64_t)world)
    fail(JAL_ERR_CAPABILITY_MISMATCH, "%llu KV heads / %llu query heads do not split over %d ranks",
         (unsigned long long)n_heads_kv, (unsigned long long)n_heads_q, world);
  if (ffn_dim % (32ull * (uint64_t)world))
    fail(JAL_ERR_CAPABILITY_MISMATCH, "ffn dim %llu does not split into whole 32-blocks over %d ranks",
         (unsigned long long)ffn_dim, world);
  TpPlan p;
  p.rank = rank;
  p.world = world;
  p.kv_n = n_heads_kv / world;
  p.kv_lo = p.kv_n * rank;
  p.q_n = n_heads_q / world;  // the query heads of this rank's KV heads (heads grouped by KV head)
  p.q_lo = p.q_n * rank;
  p.f_n = ffn_dim / world;
  p.f_lo = p.f_n * rank;
  p.v_pad = (vocab + world - 1) / world;
  p.v_lo = p.v_pad * rank < vocab ? p.v_pad * rank : vocab;
  p.v_n = p.v_lo + p.v_pad <= vocab ? p.v_pad : vocab - p.v_lo;
  return p;
}

namespace {

struct Nccl {
  void *h = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};

const Nccl &nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.get_unique_id = (decltype(n.get_unique_id))dlsym(h, "ncclGetUniqueId");
    n.comm_init_rank = (decltype(n.comm_init_rank))dlsym(h, "ncclCommInitRank");
    n.comm_destroy = (decltype(n.comm_destroy))dlsym(h, "ncclCommDestroy");
    n.all_reduce = (decltype(n.all_reduce))dlsym(h, "ncclAllReduce");
    n.all_gather = (decltype(n.all_gather))dlsym(h, "ncclAllGather");
    n.error_string = (decltype(n.error_string))dlsym(h, "ncclGetErrorString");
    if (n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.all_gather && n.error_string)
      n.h = h;
  });
  if (!n.h) fail(JAL_ERR_CAPABILITY_MISMATCH, "tensor parallelism needs libnccl.so.2 (not loadable)");
  return n;
}

void check(ncclResult_t r, const char *what) {
  if (r != ncclSuccess) fail(JAL_ERR_NCCL, "%s failed: %s", what, nccl().error_string(r));
}

}  // namespace

TpComm::~TpComm() {
  if (comm) nccl().comm_destroy((ncclComm_t)comm);
}

void tp_unique_id(uint8_t *out128) {
  ncclUniqueId id;
  check(nccl().get_unique_id(&id), "ncclGetUniqueId");
  static_assert(sizeof(id) == 128, "NCCL unique id size");
  memcpy(out128, &id, sizeof(id));
}

TpComm *tp_init(const uint8_t *id128, int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world) fail(JAL_ERR_INVALID_ARGUMENT, "tensor parallel rank %d of %d", rank, world);
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  auto t = new TpComm();
  t->rank = rank;
  t->world = world;
  cudaGetDevice(&t->device);
  ncclComm_t c = nullptr;
  ncclResult_t r = nccl().comm_init_rank(&c, world, id, rank);
  if (r != ncclSuccess) {
    delete t;
    check(r, "ncclCommInitRank");
  }
  t->comm = c;
  return t;
}

void tp_all_reduce(const TpComm &t, float *buf, size_t n, cudaStream_t s) {
  check(nccl().all_reduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)t.comm, s), "ncclAllReduce");
}

void tp_all_gather(const TpComm &t, const float *send, float *recv, size_t n, cudaStream_t s) {
  check(nccl().all_gather(send, recv, n, ncclFloat32, (ncclComm_t)t.comm, s), "ncclAllGather");
}

TpSymmetric::~TpSymmetric() {
  for (int r = 0; r < world && r < kTpMaxWorld; r++)
    if (r != rank && peer[r]) cudaIpcCloseMemHandle(peer[r]);
  if (local) cudaFree(local);
}

TpSymmetric *tp_symmetric_alloc(const TpComm &t, size_t bytes, cudaStream_t s) {
  const int W = t.world;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handle size");
  // one scratch: [W][64] handle bytes, then one float (the failure count)
  void *scratch = nullptr;
  JAL_CUDA(cudaMalloc(&scratch, (size_t)W * 64 + 64));
  auto sym = new TpSymmetric();
  sym->rank = t.rank;
  sym->world = W;
  float bad = W > kTpMaxWorld ? 1.0f : 0.0f;
  cudaIpcMemHandle_t h = {};
  if (cudaMalloc(&sym->local, bytes) != cudaSuccess || cudaMemsetAsync(sym->local, 0, bytes, s) != cudaSuccess ||
      cudaIpcGetMemHandle(&h, sym->local) != cudaSuccess) {
    cudaGetLastError();
    bad = 1.0f;
  }
  // The zeroing above is ordered before the exchange on `s`, so no peer can
  // signal into this allocation before it is clean.
  char *hs = (char *)scratch;
  JAL_CUDA(cudaMemcpyAsync(hs + (size_t)t.rank * 64, &h, 64, cudaMemcpyHostToDevice, s));
  check(nccl().all_gather(hs + (size_t)t.rank * 64, hs, 64, ncclUint8, (ncclComm_t)t.comm, s), "ncclAllGather");
  std::vector<cudaIpcMemHandle_t> all((size_t)W);
  JAL_CUDA(cudaMemcpyAsync(all.data(), hs, (size_t)W * 64, cudaMemcpyDeviceToHost, s));
  JAL_CUDA(cudaStreamSynchronize(s));
  if (bad == 0.0f) {
    for (int r = 0; r < W; r++) {
      if (r == t.rank) { sym->peer[r] = sym->local; continue; }
      if (cudaIpcOpenMemHandle(&sym->peer[r], all[(size_t)r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        sym->peer[r] = nullptr;
        bad = 1.0f;
      }
    }
  }
  float *fb = (float *)(hs + (size_t)W * 64);
  JAL_CUDA(cudaMemcpyAsync(fb, &bad, 4, cudaMemcpyHostToDevice, s));
  check(nccl().all_reduce(fb, fb, 1, ncclFloat32, ncclSum, (ncclComm_t)t.comm, s), "ncclAllReduce");
  float total = 0.0f;
  JAL_CUDA(cudaMemcpyAsync(&total, fb, 4, cudaMemcpyDeviceToHost, s));
  JAL_CUDA(cudaStreamSynchronize(s));
  cudaFree(scratch);
  if (total != 0.0f) {
    delete sym;
    return nullptr;
  }
  return sym;
}

}  // namespace jal
