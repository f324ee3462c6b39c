// SymmetricBuffer: device memory addressable by every rank of a single-node
// job.  Handles are exchanged by the caller (torch.distributed object
// all-gather); every rank maps every peer with cudaIpcOpenMemHandle, which on
// an NVSwitch system gives direct NVLink load/store access.
//
// This is the data path the reference's VulkanCommunicationBackend /
// RingAllReduce never had (src/deployment/multi_gpu_trainer.cpp:307-367 builds
// it over uninitialised devices; src/deployment/ring_all_reduce.cpp:208-256
// records no copy commands).
#include <cstring>
#include <stdexcept>

#include "dlvk/comm.h"

namespace dlvk {

SymmetricBuffer::SymmetricBuffer(int64_t bytes, int device) : bytes_(bytes), device_(device) {
  int prev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&prev));
  DLVK_CUDA_CHECK(cudaSetDevice(device));
  DLVK_CUDA_CHECK(cudaMalloc(&local_, (size_t)std::max<int64_t>(bytes, 256)));
  DLVK_CUDA_CHECK(cudaMemset(local_, 0, (size_t)std::max<int64_t>(bytes, 256)));
  DLVK_CUDA_CHECK(cudaSetDevice(prev));
}

SymmetricBuffer::SymmetricBuffer(const std::vector<uint64_t>& ptrs, int rank, int64_t bytes, int device,
                                 uint64_t multicast)
    : bytes_(bytes), device_(device), owned_(false) {
  DLVK_CHECK(rank >= 0 && rank < (int)ptrs.size(), "SymmetricBuffer: rank out of range");
  multicast_ = reinterpret_cast<void*>(multicast);
  local_ = reinterpret_cast<void*>(ptrs[rank]);
  ptrs_.resize(ptrs.size());
  for (size_t r = 0; r < ptrs.size(); ++r) ptrs_[r] = reinterpret_cast<void*>(ptrs[r]);
  opened_.assign(ptrs.size(), false);
  int prev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&prev));
  DLVK_CUDA_CHECK(cudaSetDevice(device_));
  DLVK_CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&dev_ptrs_), sizeof(void*) * ptrs_.size()));
  DLVK_CUDA_CHECK(cudaMemcpy(dev_ptrs_, ptrs_.data(), sizeof(void*) * ptrs_.size(), cudaMemcpyHostToDevice));
  DLVK_CUDA_CHECK(cudaSetDevice(prev));
}

SymmetricBuffer::~SymmetricBuffer() {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return;
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  if (!owned_) {  // the other allocator owns and unmaps the memory
    if (dev_ptrs_) cudaFree(dev_ptrs_);
    cudaSetDevice(prev);
    return;
  }
  for (size_t r = 0; r < ptrs_.size(); ++r)
    if (opened_[r] && ptrs_[r]) cudaIpcCloseMemHandle(ptrs_[r]);
  if (dev_ptrs_) cudaFree(dev_ptrs_);
  if (local_) cudaFree(local_);
  cudaSetDevice(prev);
}

std::string SymmetricBuffer::handle() const {
  cudaIpcMemHandle_t h;
  DLVK_CUDA_CHECK(cudaIpcGetMemHandle(&h, local_));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void SymmetricBuffer::open(const std::vector<std::string>& handles, int rank) {
  int prev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&prev));
  DLVK_CUDA_CHECK(cudaSetDevice(device_));
  const int world = (int)handles.size();
  ptrs_.assign(world, nullptr);
  opened_.assign(world, false);
  for (int r = 0; r < world; ++r) {
    if (r == rank) {
      ptrs_[r] = local_;
      continue;
    }
    if (handles[r].size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("SymmetricBuffer: bad IPC handle");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    DLVK_CUDA_CHECK(cudaIpcOpenMemHandle(&ptrs_[r], h, cudaIpcMemLazyEnablePeerAccess));
    opened_[r] = true;
  }
  DLVK_CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&dev_ptrs_), sizeof(void*) * world));
  DLVK_CUDA_CHECK(cudaMemcpy(dev_ptrs_, ptrs_.data(), sizeof(void*) * world, cudaMemcpyHostToDevice));
  DLVK_CUDA_CHECK(cudaSetDevice(prev));
}

}  // namespace dlvk
