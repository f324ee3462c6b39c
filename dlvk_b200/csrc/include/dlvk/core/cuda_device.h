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
