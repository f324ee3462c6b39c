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

namespace {
bool props(int index, cudaDeviceProp* p) {
  if (index < 0) return false;
  if (cudaGetDeviceProperties(p, index) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}
}  // namespace

std::string CudaDevice::get_device_type_string() const {
  cudaDeviceProp p;
  if (!props(index_, &p)) return "cpu";
  return "CUDA GPU sm_" + std::to_string(p.major) + std::to_string(p.minor) + ", " +
         std::to_string(p.multiProcessorCount) + " SMs";
}

std::string CudaDevice::get_vulkan_version_string() const {
  int v = 0;
  if (cudaRuntimeGetVersion(&v) != cudaSuccess) {
    cudaGetLastError();
    return "CUDA";
  }
  return "CUDA " + std::to_string(v / 1000) + "." + std::to_string((v % 1000) / 10);
}

uint32_t CudaDevice::get_max_workgroup_size() const {
  cudaDeviceProp p;
  return props(index_, &p) ? (uint32_t)p.maxThreadsPerBlock : 0u;
}

uint64_t CudaDevice::get_total_device_memory() const {
  cudaDeviceProp p;
  return props(index_, &p) ? (uint64_t)p.totalGlobalMem : 0u;
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
