// Tensor parallelism (Megatron-style, one process per GPU).
//
// Shard plan: Q/K/V by heads (whole KV heads per rank, each rank the query
// heads of its KV heads), gate/up by output rows, O and down by input columns
// (whole 32-element blocks), the LM head by vocabulary rows; embedding, norms
// and the O bias (rank 0 only) are replicated.  Per layer one all-reduce
// after O and one after down; logits are all-gathered (each rank's slice
// padded to the same length) before the greedy argmax.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy the process
// already has when PyTorch is loaded), so single-GPU users need no NCCL.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace jal {

struct TpPlan {
  int rank = 0, world = 1;
  uint64_t q_lo = 0, q_n = 0;    // query heads of this rank
  uint64_t kv_lo = 0, kv_n = 0;  // KV heads
  uint64_t f_lo = 0, f_n = 0;    // FFN rows (gate / up) and down input columns
  uint64_t v_lo = 0, v_n = 0;    // vocabulary rows of the LM head
  uint64_t v_pad = 0;            // per-rank logits slice length (all-gather)
};

// Shard plan for a model; fails (JAL_ERR_CAPABILITY_MISMATCH) when the
// heads or the FFN width do not split evenly into whole heads / blocks.
TpPlan tp_plan(uint64_t n_heads_q, uint64_t n_heads_kv, uint64_t ffn_dim, uint64_t vocab, int rank, int world);

struct TpComm {
  int rank = 0, world = 1, device = 0;
  void *comm = nullptr;  // ncclComm_t
  ~TpComm();
};

// 128-byte NCCL unique id (rank 0 creates it; the caller distributes it).
void tp_unique_id(uint8_t *out128);
TpComm *tp_init(const uint8_t *id128, int rank, int world);
// In-place f32 sum over the ranks / all-gather of `n` floats per rank.
void tp_all_reduce(const TpComm &t, float *buf, size_t n, cudaStream_t s);
void tp_all_gather(const TpComm &t, const float *send, float *recv, size_t n, cudaStream_t s);

constexpr int kTpMaxWorld = 8;

// Symmetric device memory: every rank allocates `bytes` (zeroed), the CUDA
// IPC handles are all-gathered through NCCL and each rank maps the others'
// allocations, so peer[r] is rank r's allocation in this process (peer[rank]
// == local).  Collective: all ranks call it in the same order.
struct TpSymmetric {
  int rank = 0, world = 1;
  void *local = nullptr;
  void *peer[kTpMaxWorld] = {};
  ~TpSymmetric();
};
// nullptr on every rank when any rank cannot map a peer (no peer access, or
// more than kTpMaxWorld ranks); the ranks agree through an all-reduce.
TpSymmetric *tp_symmetric_alloc(const TpComm &t, size_t bytes, cudaStream_t s);

}  // namespace jal
