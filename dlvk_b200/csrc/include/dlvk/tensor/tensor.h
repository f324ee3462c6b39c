// C++ API: dlvk::Tensor, a value handle over an at::Tensor.
//
// Keeps the reference's interface (include/dlvk/tensor/tensor.h:20-97):
// shape / size / dtype, upload_data / download_data, reshape, transpose, the
// element-wise and matrix ops returning std::shared_ptr<Tensor>, reductions
// over one axis or all elements (axis -1), activations and their backward
// passes.  CUDA tensors run the sm_100a kernels (the same launches as the
// Python package); CPU tensors run the ATen reference path.  Copies share
// storage (at::Tensor semantics); use clone() for a deep copy.
#pragma once
#include <ATen/ATen.h>

#include <memory>
#include <vector>

#include "dlvk/core/cuda_device.h"

namespace dlvk {

enum class DataType { FLOAT32, FLOAT16, INT32, INT8, BFLOAT16, INT64 };

at::ScalarType to_scalar_type(DataType dt);
DataType from_scalar_type(at::ScalarType st);

class Tensor {
 public:
  Tensor() = default;
  Tensor(const std::vector<size_t>& shape, DataType dtype, std::shared_ptr<CudaDevice> device);
  // Wraps an existing ATen tensor (no copy).
  explicit Tensor(at::Tensor t, std::shared_ptr<CudaDevice> device = nullptr);

  static Tensor zeros(std::shared_ptr<CudaDevice> device, const std::vector<size_t>& shape,
                      DataType dtype = DataType::FLOAT32);
  static Tensor from_vector(std::shared_ptr<CudaDevice> device, const std::vector<size_t>& shape,
                            const std::vector<float>& values);

  std::vector<size_t> shape() const;
  size_t size() const;
  size_t element_size() const;
  DataType dtype() const;
  std::shared_ptr<CudaDevice> device() const { return device_; }
  bool defined() const { return t_.defined(); }

  // Host <-> tensor copies of size() * element_size() bytes.
  void upload_data(const void* data);
  void download_data(void* data) const;
  std::vector<float> to_vector() const;

  std::shared_ptr<Tensor> reshape(const std::vector<size_t>& new_shape) const;
  // No axes: 2-D (or batched 2-D) transpose; else a permutation.
  std::shared_ptr<Tensor> transpose(const std::vector<size_t>& axes = {}) const;

  std::shared_ptr<Tensor> add(const Tensor& other) const;
  std::shared_ptr<Tensor> add_broadcast(const Tensor& bias) const;  // + bias over the last dimension
  std::shared_ptr<Tensor> subtract(const Tensor& other) const;
  std::shared_ptr<Tensor> multiply(const Tensor& other) const;
  std::shared_ptr<Tensor> multiply_scalar(float scalar) const;
  std::shared_ptr<Tensor> divide(const Tensor& other) const;
  std::shared_ptr<Tensor> matrix_multiply(const Tensor& other) const;

  // axis -1 (or a 1-D tensor): over all elements, result shape {1}.
  std::shared_ptr<Tensor> sum(int axis = -1) const;
  std::shared_ptr<Tensor> mean(int axis = -1) const;
  std::shared_ptr<Tensor> max(int axis = -1) const;
  std::shared_ptr<Tensor> min(int axis = -1) const;

  std::shared_ptr<Tensor> relu() const;
  std::shared_ptr<Tensor> sigmoid() const;
  std::shared_ptr<Tensor> tanh() const;
  std::shared_ptr<Tensor> softmax() const;

  std::shared_ptr<Tensor> relu_backward(const Tensor& grad_output) const;     // this = input
  std::shared_ptr<Tensor> sigmoid_backward(const Tensor& grad_output) const;  // this = output
  std::shared_ptr<Tensor> tanh_backward(const Tensor& grad_output) const;     // this = output

  Tensor clone() const;
  const at::Tensor& data() const { return t_; }
  at::Tensor& data() { return t_; }

 private:
  std::shared_ptr<Tensor> wrap(at::Tensor t) const;
  at::Tensor t_;
  std::shared_ptr<CudaDevice> device_;
};

}  // namespace dlvk
