// Shared helpers for the PyTorch binding translation units.
#pragma once
#include <torch/extension.h>

#include "dlvk/common.h"

namespace dlvk {
namespace bind {

DType to_dtype(const at::Tensor& t);
void check_cuda(const at::Tensor& t, const char* name);
cudaStream_t stream();

void register_ops(py::module& m);
void register_runtime(py::module& m);
void register_nn(py::module& m);
void register_comm(py::module& m);

}  // namespace bind
}  // namespace dlvk
