// Peer-memory communication: symmetric buffers mapped into every rank of a
// single-node job through CUDA IPC, and the launch arguments of the fused
// all-reduce + optimizer kernel (comm.cu).
#pragma once
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>
#include <string>
#include <vector>

#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {

struct FusedARArgs {
  int world = 1, rank = 0;
  const void* const* peer_grads = nullptr;  // device array [world]: gradient buffer of every rank
  void* const* peer_values = nullptr;       // device array [world]: compute-dtype parameters of every rank
  uint32_t* const* peer_flags = nullptr;    // device array [world]: flag buffer of every rank
  uint32_t* my_flags = nullptr;
  unsigned int* cta_counter = nullptr;      // per-bucket arrival counter (local, zero between launches)
  int64_t start = 0, end = 0;               // element range of the bucket in the flat buffers
  int bucket = 0;
  float* master = nullptr;                  // local fp32 master parameters (full flat buffer)
  float* m = nullptr;                       // optimizer state (may be null)
  float* v = nullptr;
  const OptimHyper* hyper = nullptr;
  int kind = OPT_ADAM;
  float scale = 1.f;                        // 1 / world
  const int64_t* epoch_ptr = nullptr;       // device step counter
  int one_shot = 0;
  int values_are_master = 0;
  uint32_t* err = nullptr;
  uint64_t budget_ns = 5000000000ull;
  // Push two-shot (fused_allreduce_optimizer_push): every rank stores the
  // gradient slices it does not own into the owners' receive buffers, so all
  // NVLink traffic is stores and every reduction read is local.
  void* const* peer_recv = nullptr;         // device array [world]: receive buffer of every rank
  const void* my_recv = nullptr;
  int64_t recv_off = 0;                     // element offset of this bucket's shard inside one slot
  int64_t recv_slot = 0;                    // elements per slot; a rank has world-1 slots
  uint32_t* const* peer_cflags = nullptr;   // device array [world]: chunk-flag table of every rank
  uint32_t* my_cflags = nullptr;
  int cbucket = 0;                          // row of this bucket in the chunk-flag table
  int64_t chunk = 0;                        // elements of each rank's shard handled by one CTA
  // LL one-shot (fused_allreduce_optimizer_ll): [2 parities][world-1 slots]
  // [ll_cap] 8-byte {fp32 gradient, epoch} words in every rank's ll buffer.
  void* const* peer_ll = nullptr;
  const void* my_ll = nullptr;
  int64_t ll_off = 0;                       // element offset of this bucket inside a slot
  int64_t ll_cap = 0;                       // elements per slot
  // NVLS two-shot (fused_allreduce_optimizer_nvls): NVLink-multicast
  // addresses of the gradient and parameter buffers (the same flat layout as
  // peer_grads / peer_values, every rank's memory bound to the object).
  void* mc_grads = nullptr;
  void* mc_values = nullptr;
};

// Chunk-flag table of the push two-shot kernel: [PUSH_MAX_BUCKETS]
// [PUSH_MAX_CHUNKS][world] uint32 epochs; one entry per (CTA, sub-chunk).
constexpr int PUSH_MAX_BUCKETS = 128;
constexpr int PUSH_MAX_CHUNKS = 2048;
constexpr int PUSH_SUB = 2;  // sub-chunks per CTA
// Elements of each rank's shard handled by one CTA when the kernel runs
// `ctas` CTAs: a multiple of 1024, at least 2048, and at most
// PUSH_MAX_CHUNKS / PUSH_SUB CTAs.
inline int64_t push_chunk_elems(int64_t shard, int ctas) {
  const int64_t g = std::max<int64_t>(1, std::min<int64_t>(ctas, PUSH_MAX_CHUNKS / PUSH_SUB));
  const int64_t c = (shard + g - 1) / g;
  return std::max<int64_t>(2048, (c + 1023) / 1024 * 1024);
}

void fused_allreduce_optimizer(const FusedARArgs& a, DType grad_dt, DType value_dt, int ctas, cudaStream_t s);
// Generic in-place sum (or mean) all-reduce of [start, end) of the symmetric
// buffer whose per-rank bases are a.peer_grads.
void p2p_allreduce(const FusedARArgs& a, DType dt, bool average, int ctas, cudaStream_t s);
// Broadcast (mode 0, from `root`), all-gather (1: `out` holds world blocks of
// numel) and reduce-scatter (2: `out` holds this rank's ceil(numel/world)
// chunk of the rank-order sum) of the contributions every rank wrote at
// offset 0 of its staging buffer (a.peer_grads), with ready / done flags.
void p2p_collective(const FusedARArgs& a, DType dt, int mode, int root, void* out, int64_t numel, int ctas,
                    cudaStream_t s);
// One-shot low-latency variant for small buckets: every rank stores its
// gradients, each fp32 value paired with the step epoch in one 8-byte word,
// into every peer's LL buffer; receivers poll the words themselves (no
// flags, fences or barriers) and every rank updates the whole bucket.
// Requires fp32 gradients; peer_ll, my_ll, ll_off and ll_cap must be set.
void fused_allreduce_optimizer_ll(const FusedARArgs& a, DType value_dt, int ctas, cudaStream_t s);
// Two-shot push variant of fused_allreduce_optimizer (peer_recv, my_recv,
// recv_off, recv_slot, peer_cflags, my_cflags and cbucket must be set).
void fused_allreduce_optimizer_push(const FusedARArgs& a, DType grad_dt, DType value_dt, cudaStream_t s);

// NVLS two-shot: rank r's shard of the bucket is summed over all ranks by the
// NVSwitch (multimem.ld_reduce on mc_grads, fp32 gradients), updated by the
// optimizer on rank r, and the new parameters are written to every rank with
// one multicast store each (multimem.st on mc_values).  Ready / done flags as
// in fused_allreduce_optimizer.  Needs mc_grads and mc_values.
void fused_allreduce_optimizer_nvls(const FusedARArgs& a, DType value_dt, int ctas, cudaStream_t s);

// A device allocation that every rank of the node can address: cudaMalloc +
// cudaIpcGetMemHandle here, cudaIpcOpenMemHandle of the peers' handles there.
class SymmetricBuffer {
 public:
  SymmetricBuffer(int64_t bytes, int device);
  // A non-owning view of memory another allocator made symmetric (for
  // example PyTorch's symmetric memory): `ptrs[r]` is rank r's base address
  // as mapped on this device, `multicast` the NVLink multicast address of
  // the same buffer (0 if none).
  SymmetricBuffer(const std::vector<uint64_t>& ptrs, int rank, int64_t bytes, int device, uint64_t multicast);
  ~SymmetricBuffer();
  SymmetricBuffer(const SymmetricBuffer&) = delete;
  SymmetricBuffer& operator=(const SymmetricBuffer&) = delete;

  std::string handle() const;  // opaque 64-byte IPC handle
  // Map every peer's buffer; `handles[r]` is rank r's handle (own included).
  void open(const std::vector<std::string>& handles, int rank);
  void* local() const { return local_; }
  int64_t bytes() const { return bytes_; }
  // Device array of `world` base pointers (own buffer at index rank).
  void* const* device_ptrs() const { return dev_ptrs_; }
  const std::vector<void*>& host_ptrs() const { return ptrs_; }
  int device() const { return device_; }
  void* multicast() const { return multicast_; }

 private:
  int64_t bytes_;
  int device_;
  bool owned_ = true;
  void* multicast_ = nullptr;
  void* local_ = nullptr;
  std::vector<void*> ptrs_;
  std::vector<bool> opened_;
  void** dev_ptrs_ = nullptr;
};

// Failure-detection probe: waits (bounded by budget_ns) for *flag == epoch
// with the all-reduce kernels' wait; result[0] = 1 if seen, 0 on timeout
// (the timeout is also recorded in `err` as DLVK_ERR_PEER_TIMEOUT).
void wait_flag_probe(const uint32_t* flag, uint32_t epoch, uint64_t budget_ns, uint32_t* err, int* result,
                     cudaStream_t s);

}  // namespace dlvk
