// Python bindings of the communication runtime (comm.cu).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "comm.h"

namespace uhfs {
void bind_comm(pybind11::module_& m) { (void)m; }
}  // namespace uhfs
