// Registration hooks for binding groups that are filled in by other files.
#include "bind_common.h"

namespace dlvk {
namespace bind {


void register_comm(py::module&) {}
}  // namespace bind
}  // namespace dlvk
