// Shared helpers for the PyTorch binding translation units.
#pragma once
#include <torch/extension.h>

#include "dlvk/aten_ops.h"
#include "dlvk/common.h"

namespace dlvk {
namespace bind {

// Tensor helpers of the ATen op layer (dlvk/aten_ops.h).
using ::dlvk::aten::check_cuda;
using ::dlvk::aten::stream;
using ::dlvk::aten::to_dtype;

void register_ops(py::module& m);
void register_runtime(py::module& m);
void register_nn(py::module& m);
void register_comm(py::module& m);

}  // namespace bind
}  // namespace dlvk
