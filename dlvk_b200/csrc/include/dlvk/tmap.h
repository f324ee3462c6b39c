// Host helpers for TMA tensor maps shared by the tensor-core kernels.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "dlvk/common.h"

namespace dlvk {
namespace tmap {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link dependency).
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    DLVK_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("dlvk: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// The encoder is a driver call and needs a current context on the calling
// thread; threads that only touched the runtime through PyTorch's autograd
// workers may not have one, so bind the primary context once per thread.
inline void bind_context() {
  thread_local int bound_dev = -1;
  int dev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&dev));
  if (bound_dev != dev) {
    DLVK_CUDA_CHECK(cudaSetDevice(dev));
    bound_dev = dev;
  }
}

// 2-D bf16 map over a row-major [rows, cols] matrix with row stride
// `ld` elements: box {64 columns (128 B), box_rows}, 128-byte swizzle.
inline CUtensorMap bf16_2d_sw128(const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("dlvk: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

inline int sm_count() {
  static int n[kMaxDevices] = {0};
  const int dev = current_device_slot();
  if (n[dev] == 0) DLVK_CUDA_CHECK(cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev));
  return n[dev];
}

}  // namespace tmap
}  // namespace dlvk
