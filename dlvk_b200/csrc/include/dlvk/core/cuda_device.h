// C++ API: the device a model or tensor lives on.
//
// Replaces the reference's VulkanDevice (include/dlvk/core/vulkan_device.h:
// instance, physical device, one compute queue) with a CUDA device index;
// streams and memory come from PyTorch's CUDA runtime (current stream,
// caching allocator), which the kernels launch on.  A device built with
// index -1 is the host CPU: every op then runs the plain ATen reference path
// that the Python package uses on CPU, so results match it bit for bit.
#pragma once
#include <c10/core/Device.h>

#include <cstdint>
#include <memory>
#include <string>

namespace dlvk {

class CudaDevice {
 public:
  // index >= 0: that CUDA device; -1: the host CPU.
  explicit CudaDevice(int index = 0);

  // Makes the device usable (selects it, creates its context).  Returns
  // false when a CUDA index was asked for and no such device exists.
  bool initialize();
  bool is_initialized() const { return initialized_; }

  bool is_cuda() const { return index_ >= 0; }
  int index() const { return index_; }
  c10::Device device() const;
  std::string name() const;

  // Device-info getters of the reference's vulkan_device.h:64-70, answered
  // from cudaGetDeviceProperties (the CPU device answers "cpu" / zeros):
  // get_device_type_string: "CUDA GPU sm_<major><minor>, <n> SMs" or "cpu";
  // get_vulkan_version_string: the CUDA runtime version ("CUDA 12.9");
  // get_max_workgroup_size: max threads per block;
  // get_max_memory_allocation / get_total_device_memory: total global memory
  // in bytes; get_memory_heap_count: 1 (one global memory).
  std::string get_device_name() const { return name(); }
  std::string get_device_type_string() const;
  std::string get_vulkan_version_string() const;
  uint32_t get_max_workgroup_size() const;
  uint64_t get_max_memory_allocation() const { return get_total_device_memory(); }
  uint32_t get_memory_heap_count() const { return is_cuda() ? 1u : 0u; }
  uint64_t get_total_device_memory() const;

  // Shared CPU device (for tests and CPU-only programs).
  static std::shared_ptr<CudaDevice> cpu();
  // Number of visible CUDA devices (0 on a host without a GPU).
  static int device_count();

 private:
  int index_;
  bool initialized_ = false;
};

// Source compatibility with code written against the reference.
using VulkanDevice = CudaDevice;

}  // namespace dlvk
