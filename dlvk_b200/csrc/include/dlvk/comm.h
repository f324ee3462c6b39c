// Peer-memory communication: symmetric buffers mapped into every rank of a
// single-node job through CUDA IPC, and the launch arguments of the fused
// all-reduce + optimizer kernel (comm.cu).
#pragma once
#include <cuda_runtime.h>
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
};

void fused_allreduce_optimizer(const FusedARArgs& a, DType grad_dt, DType value_dt, int ctas, cudaStream_t s);
// Generic in-place sum (or mean) all-reduce of [start, end) of the symmetric
// buffer whose per-rank bases are a.peer_grads.
void p2p_allreduce(const FusedARArgs& a, DType dt, bool average, int ctas, cudaStream_t s);

// A device allocation that every rank of the node can address: cudaMalloc +
// cudaIpcGetMemHandle here, cudaIpcOpenMemHandle of the peers' handles there.
class SymmetricBuffer {
 public:
  SymmetricBuffer(int64_t bytes, int device);
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

 private:
  int64_t bytes_;
  int device_;
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
