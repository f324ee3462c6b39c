// Python module definition: dlvk_b200._C
#include "bind_common.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dlvk_b200 native extension: sm_100a kernels and the C++ runtime";
  dlvk::bind::register_ops(m);
  dlvk::bind::register_runtime(m);
  dlvk::bind::register_nn(m);
  dlvk::bind::register_comm(m);
}
