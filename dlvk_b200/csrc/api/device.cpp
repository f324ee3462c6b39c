// C++ API: CudaDevice (the reference's VulkanDevice role, include/dlvk/core/
// vulkan_device.h) over the CUDA runtime.
#include <cuda_runtime.h>

#include "dlvk/common.h"
#include "dlvk/core/cuda_device.h"

namespace dlvk {

CudaDevice::CudaDevice(int index) : index_(index) {}

int CudaDevice::device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();  // no driver / no device: not an error for a CPU program
    return 0;
  }
  return n;
}

bool CudaDevice::initialize() {
  if (index_ < 0) {
    initialized_ = true;
    return true;
  }
  if (index_ >= device_count()) return false;
  if (cudaSetDevice(index_) != cudaSuccess || cudaFree(nullptr) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  initialized_ = true;
  return true;
}

c10::Device CudaDevice::device() const {
  return index_ < 0 ? c10::Device(c10::kCPU) : c10::Device(c10::kCUDA, (c10::DeviceIndex)index_);
}

std::string CudaDevice::name() const {
  if (index_ < 0) return "cpu";
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, index_) != cudaSuccess) {
    cudaGetLastError();
    return "cuda:" + std::to_string(index_);
  }
  return p.name;
}

std::shared_ptr<CudaDevice> CudaDevice::cpu() {
  static std::shared_ptr<CudaDevice> dev = [] {
    auto d = std::make_shared<CudaDevice>(-1);
    d->initialize();
    return d;
  }();
  return dev;
}

}  // namespace dlvk
