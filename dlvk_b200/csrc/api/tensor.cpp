// C++ API: dlvk::Tensor (include/dlvk/tensor/tensor.h:20-97 of the
// reference) and TensorOpsStatic (include/dlvk/tensor/tensor_ops_static.h:
// 8-27).  The op choices restate the Python facade (dlvk_b200/tensor.py).
#include "dlvk/tensor/tensor.h"

#include <cstring>

#include "dispatch.h"
#include "dlvk/tensor/tensor_ops_static.h"

namespace dlvk {

at::ScalarType to_scalar_type(DataType dt) {
  switch (dt) {
    case DataType::FLOAT32: return at::kFloat;
    case DataType::FLOAT16: return at::kHalf;
    case DataType::INT32: return at::kInt;
    case DataType::INT8: return at::kChar;
    case DataType::BFLOAT16: return at::kBFloat16;
    case DataType::INT64: return at::kLong;
  }
  return at::kFloat;
}

DataType from_scalar_type(at::ScalarType st) {
  switch (st) {
    case at::kFloat: return DataType::FLOAT32;
    case at::kHalf: return DataType::FLOAT16;
    case at::kInt: return DataType::INT32;
    case at::kChar: return DataType::INT8;
    case at::kBFloat16: return DataType::BFLOAT16;
    case at::kLong: return DataType::INT64;
    default: TORCH_CHECK(false, "dlvk::Tensor: unsupported dtype ", st);
  }
}

namespace {
std::vector<int64_t> dims_of(const std::vector<size_t>& shape) { return std::vector<int64_t>(shape.begin(), shape.end()); }
std::shared_ptr<CudaDevice> device_or_cpu(std::shared_ptr<CudaDevice> d) { return d ? d : CudaDevice::cpu(); }
}  // namespace

Tensor::Tensor(const std::vector<size_t>& shape, DataType dtype, std::shared_ptr<CudaDevice> device)
    : device_(device_or_cpu(std::move(device))) {
  t_ = at::zeros(dims_of(shape), at::TensorOptions().dtype(to_scalar_type(dtype)).device(device_->device()));
}

Tensor::Tensor(at::Tensor t, std::shared_ptr<CudaDevice> device) : t_(std::move(t)) {
  if (device) {
    device_ = std::move(device);
  } else if (t_.defined() && t_.is_cuda()) {
    device_ = std::make_shared<CudaDevice>(t_.get_device());
    device_->initialize();
  } else {
    device_ = CudaDevice::cpu();
  }
}

Tensor Tensor::zeros(std::shared_ptr<CudaDevice> device, const std::vector<size_t>& shape, DataType dtype) {
  return Tensor(shape, dtype, std::move(device));
}

Tensor Tensor::from_vector(std::shared_ptr<CudaDevice> device, const std::vector<size_t>& shape,
                           const std::vector<float>& values) {
  Tensor t(shape, DataType::FLOAT32, std::move(device));
  TORCH_CHECK(values.size() == t.size(), "dlvk::Tensor::from_vector: ", values.size(), " values for ", t.size(),
              " elements");
  t.upload_data(values.data());
  return t;
}

std::vector<size_t> Tensor::shape() const {
  std::vector<size_t> s;
  for (auto d : t_.sizes()) s.push_back((size_t)d);
  return s;
}
size_t Tensor::size() const { return (size_t)t_.numel(); }
size_t Tensor::element_size() const { return (size_t)t_.element_size(); }
DataType Tensor::dtype() const { return from_scalar_type(t_.scalar_type()); }

void Tensor::upload_data(const void* data) {
  at::Tensor host = at::from_blob(const_cast<void*>(data), t_.sizes(), t_.options().device(c10::kCPU));
  t_.copy_(host);
}

void Tensor::download_data(void* data) const {
  at::Tensor host = t_.contiguous().to(c10::kCPU);
  std::memcpy(data, host.data_ptr(), host.numel() * host.element_size());
}

std::vector<float> Tensor::to_vector() const {
  at::Tensor host = t_.to(c10::kCPU, at::kFloat).contiguous();
  return std::vector<float>(host.data_ptr<float>(), host.data_ptr<float>() + host.numel());
}

std::shared_ptr<Tensor> Tensor::wrap(at::Tensor t) const { return std::make_shared<Tensor>(std::move(t), device_); }

std::shared_ptr<Tensor> Tensor::reshape(const std::vector<size_t>& new_shape) const {
  return wrap(t_.reshape(dims_of(new_shape)));
}

std::shared_ptr<Tensor> Tensor::transpose(const std::vector<size_t>& axes) const {
  if (!axes.empty()) return wrap(t_.permute(dims_of(axes)).contiguous());
  return wrap(api::transpose(t_));
}

std::shared_ptr<Tensor> Tensor::add(const Tensor& o) const { return wrap(api::binary(t_, o.t_, BIN_ADD)); }
std::shared_ptr<Tensor> Tensor::add_broadcast(const Tensor& b) const { return wrap(api::bias_act(t_, b.t_)); }
std::shared_ptr<Tensor> Tensor::subtract(const Tensor& o) const { return wrap(api::binary(t_, o.t_, BIN_SUB)); }
std::shared_ptr<Tensor> Tensor::multiply(const Tensor& o) const { return wrap(api::binary(t_, o.t_, BIN_MUL)); }
std::shared_ptr<Tensor> Tensor::multiply_scalar(float s) const { return wrap(api::unary(t_, UN_SCALE, (double)s)); }
std::shared_ptr<Tensor> Tensor::divide(const Tensor& o) const { return wrap(api::binary(t_, o.t_, BIN_DIV)); }
std::shared_ptr<Tensor> Tensor::matrix_multiply(const Tensor& o) const { return wrap(api::gemm(t_, o.t_)); }

namespace {
at::Tensor reduce_axis(const at::Tensor& t, int op, int axis) {
  if (axis == -1 || t.dim() == 1) return api::reduce(t, op).reshape({1});
  if (axis == 0 && t.dim() == 2 && op == RED_SUM) return api::colsum(t);
  at::Tensor f = t.to(at::kFloat);
  if (op == RED_SUM) return f.sum(axis);
  if (op == RED_MAX) return f.amax(axis);
  return f.amin(axis);
}
}  // namespace

std::shared_ptr<Tensor> Tensor::sum(int axis) const { return wrap(reduce_axis(t_, RED_SUM, axis)); }
std::shared_ptr<Tensor> Tensor::mean(int axis) const {
  const double n = (axis == -1 || t_.dim() == 1) ? (double)t_.numel() : (double)t_.size(axis);
  return wrap(api::unary(reduce_axis(t_, RED_SUM, axis), UN_SCALE, 1.0 / n));
}
std::shared_ptr<Tensor> Tensor::max(int axis) const { return wrap(reduce_axis(t_, RED_MAX, axis)); }
std::shared_ptr<Tensor> Tensor::min(int axis) const { return wrap(reduce_axis(t_, RED_MIN, axis)); }

std::shared_ptr<Tensor> Tensor::relu() const { return wrap(api::unary(t_, UN_RELU)); }
std::shared_ptr<Tensor> Tensor::sigmoid() const { return wrap(api::unary(t_, UN_SIGMOID)); }
std::shared_ptr<Tensor> Tensor::tanh() const { return wrap(api::unary(t_, UN_TANH)); }
std::shared_ptr<Tensor> Tensor::softmax() const { return wrap(api::softmax(t_)); }
std::shared_ptr<Tensor> Tensor::relu_backward(const Tensor& g) const {
  return wrap(api::binary(g.t_, t_, BIN_RELU_BWD));
}
std::shared_ptr<Tensor> Tensor::sigmoid_backward(const Tensor& g) const {
  return wrap(api::binary(g.t_, t_, BIN_SIGMOID_BWD));
}
std::shared_ptr<Tensor> Tensor::tanh_backward(const Tensor& g) const {
  return wrap(api::binary(g.t_, t_, BIN_TANH_BWD));
}

Tensor Tensor::clone() const { return Tensor(t_.clone(), device_); }

// ---------------------------------------------------------------- TensorOpsStatic
namespace {
bool fits(const Tensor& r, const at::Tensor& v) {
  return r.defined() && r.data().numel() == v.numel() && r.data().device() == v.device();
}
template <typename F>
bool into(Tensor& result, F&& f) {
  try {
    at::Tensor v = f();
    if (!fits(result, v)) return false;
    result.data().copy_(v.reshape(result.data().sizes()));
    return true;
  } catch (const std::exception&) {
    return false;
  }
}
}  // namespace

bool TensorOpsStatic::relu(const Tensor& in, Tensor& r) { return into(r, [&] { return in.relu()->data(); }); }
bool TensorOpsStatic::sigmoid(const Tensor& in, Tensor& r) { return into(r, [&] { return in.sigmoid()->data(); }); }
bool TensorOpsStatic::tanh_activation(const Tensor& in, Tensor& r) {
  return into(r, [&] { return in.tanh()->data(); });
}
bool TensorOpsStatic::softmax(const Tensor& in, Tensor& r) { return into(r, [&] { return in.softmax()->data(); }); }
bool TensorOpsStatic::matrix_multiply(const Tensor& a, const Tensor& b, Tensor& r) {
  return into(r, [&] { return a.matrix_multiply(b)->data(); });
}
bool TensorOpsStatic::relu_backward(const Tensor& in, const Tensor& g, Tensor& r) {
  return into(r, [&] { return in.relu_backward(g)->data(); });
}
bool TensorOpsStatic::sigmoid_backward(const Tensor& out, const Tensor& g, Tensor& r) {
  return into(r, [&] { return out.sigmoid_backward(g)->data(); });
}
bool TensorOpsStatic::tanh_backward(const Tensor& out, const Tensor& g, Tensor& r) {
  return into(r, [&] { return out.tanh_backward(g)->data(); });
}
bool TensorOpsStatic::copy(const Tensor& src, Tensor& dst) { return into(dst, [&] { return src.data(); }); }
bool TensorOpsStatic::fill(Tensor& t, float value) {
  if (!t.defined()) return false;
  t.data().fill_(value);
  return true;
}

}  // namespace dlvk
