// Symmetric-memory communication runtime and fused collective kernels over
// NVLink 5 / NVSwitch (peer loads/stores with bounded flag waits).
#pragma once

#include <pybind11/pybind11.h>

namespace uhfs {
void bind_comm(pybind11::module_& m);
}  // namespace uhfs
