// Python bindings of the communication runtime (comm.cu) and a minimal DLPack
// exporter so regions of the symmetric heap become torch tensors without a
// copy (torch.from_dlpack on the returned capsule).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdlib>
#include <stdexcept>

#include "comm.h"
#include "comm_api.h"

namespace py = pybind11;

namespace uhfs {

namespace {

// DLPack ABI (open standard, v0.x layout).
struct DLDevice {
  int32_t device_type;  // 2 = kDLCUDA
  int32_t device_id;
};
struct DLDataType {
  uint8_t code;  // 0 int, 1 uint, 2 float, 4 bfloat
  uint8_t bits;
  uint16_t lanes;
};
struct DLTensor {
  void* data;
  DLDevice device;
  int32_t ndim;
  DLDataType dtype;
  int64_t* shape;
  int64_t* strides;
  uint64_t byte_offset;
};
struct DLManagedTensor {
  DLTensor dl_tensor;
  void* manager_ctx;
  void (*deleter)(DLManagedTensor*);
};

void dl_deleter(DLManagedTensor* t) {
  std::free(t->dl_tensor.shape);
  delete t;
}

void capsule_destructor(PyObject* cap) {
  // Only free if torch did not consume it (consumed capsules are renamed).
  if (PyCapsule_IsValid(cap, "dltensor")) {
    auto* t = static_cast<DLManagedTensor*>(PyCapsule_GetPointer(cap, "dltensor"));
    if (t != nullptr && t->deleter != nullptr) t->deleter(t);
  }
}

py::capsule make_capsule(uintptr_t ptr, int device, int64_t numel, const std::string& dtype) {
  auto* t = new DLManagedTensor();
  t->dl_tensor.data = reinterpret_cast<void*>(ptr);
  t->dl_tensor.device = DLDevice{2, device};
  t->dl_tensor.ndim = 1;
  if (dtype == "float32") t->dl_tensor.dtype = DLDataType{2, 32, 1};
  else if (dtype == "bfloat16") t->dl_tensor.dtype = DLDataType{4, 16, 1};
  else if (dtype == "int32") t->dl_tensor.dtype = DLDataType{0, 32, 1};
  else if (dtype == "uint8") t->dl_tensor.dtype = DLDataType{1, 8, 1};
  else {
    delete t;
    throw std::invalid_argument("unsupported dlpack dtype " + dtype);
  }
  t->dl_tensor.shape = static_cast<int64_t*>(std::malloc(sizeof(int64_t)));
  t->dl_tensor.shape[0] = numel;
  t->dl_tensor.strides = nullptr;
  t->dl_tensor.byte_offset = 0;
  t->manager_ctx = nullptr;
  t->deleter = dl_deleter;
  return py::capsule(t, "dltensor", capsule_destructor);
}

cudaStream_t S(uintptr_t s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

void bind_comm(py::module_& m) {
  py::class_<SymmetricHeap>(m, "SymmetricHeap")
      .def(py::init<int, int, size_t>(), py::arg("rank"), py::arg("world"), py::arg("data_bytes"))
      .def("ipc_handle", [](const SymmetricHeap& h) { return py::bytes(h.ipc_handle()); })
      .def("open", [](SymmetricHeap& h, const std::vector<py::bytes>& hs) {
        std::vector<std::string> v;
        for (auto& b : hs) v.push_back(std::string(b));
        h.open(v);
      })
      .def("close", &SymmetricHeap::close)
      .def_property_readonly("rank", &SymmetricHeap::rank)
      .def_property_readonly("world", &SymmetricHeap::world)
      .def_property_readonly("data_bytes", &SymmetricHeap::data_bytes)
      .def("data_ptr", &SymmetricHeap::data_ptr)
      .def("signal_ptr", &SymmetricHeap::signal_ptr)
      .def("dlpack", [](const SymmetricHeap& h, long long off_bytes, int64_t numel, const std::string& dtype) {
        return make_capsule(h.data_ptr(h.rank()) + off_bytes, h.device(), numel, dtype);
      });
  m.def("comm_allreduce_f32", [](const SymmetricHeap& h, long long off, long long n, float scale, int blocks,
                                 uintptr_t s) { comm_allreduce_f32(h, off, n, scale, blocks, S(s)); });
  m.def("comm_allreduce_f32_nvls", [](const SymmetricHeap& h, uintptr_t mc, long long off, long long n, float scale,
                                      int blocks, uintptr_t s) {
    comm_allreduce_f32_nvls(h, mc, off, n, scale, blocks, S(s));
  });
  m.def("comm_rs_adamw_ag",
        [](const SymmetricHeap& g, long long goff, const SymmetricHeap& p, long long poff, long long lo, long long n,
           uintptr_t master, uintptr_t mm, uintptr_t vv, float lr, float b1, float b2, float eps, float wd,
           float gscale, bool decoupled, uintptr_t step_ptr, int blocks, uintptr_t s) {
          comm_rs_adamw_ag(g, goff, p, poff, lo, n, master, mm, vv, lr, b1, b2, eps, wd, gscale, decoupled,
                           step_ptr, blocks, S(s));
        });
  m.def("comm_allgather", [](const SymmetricHeap& h, long long off, long long shard_bytes, int blocks, uintptr_t s) {
    comm_allgather(h, off, shard_bytes, blocks, S(s));
  });
  m.def("comm_allreduce_bf16", [](const SymmetricHeap& h, long long off, long long n, float scale, int blocks,
                                  uintptr_t s) { comm_allreduce_bf16(h, off, n, scale, blocks, S(s)); });
  m.def("comm_allreduce_f32_wire_bf16", [](const SymmetricHeap& h, long long off, long long wire_off, long long n,
                                           float scale, int blocks, uintptr_t s) {
    comm_allreduce_f32_wire_bf16(h, off, wire_off, n, scale, blocks, S(s));
  });
  m.def("comm_reduce_scatter", [](const SymmetricHeap& h, long long in_off, long long out_off, long long n, bool bf16,
                                  float scale, int blocks, uintptr_t s) {
    comm_reduce_scatter(h, in_off, out_off, n, bf16, scale, blocks, S(s));
  });
  m.def("comm_gather_segments", [](const SymmetricHeap& h, long long dst_off, uintptr_t shard,
                                   const std::vector<std::array<long long, 3>>& segs, int blocks, uintptr_t s) {
    comm_gather_segments(h, dst_off, shard, segs, blocks, S(s));
  });
  m.def("comm_rs_adamw_segments",
        [](const SymmetricHeap& g, long long goff, const std::vector<std::array<long long, 3>>& segs, uintptr_t master,
           uintptr_t mm, uintptr_t vv, uintptr_t shard16, float lr, float b1, float b2, float eps, float wd,
           float gscale, bool decoupled, uintptr_t step_ptr, int blocks, uintptr_t s) {
          comm_rs_adamw_segments(g, goff, segs, master, mm, vv, shard16, lr, b1, b2, eps, wd, gscale, decoupled,
                                 step_ptr, blocks, S(s));
        });
  m.def("comm_barrier", [](const SymmetricHeap& h, uintptr_t s) { comm_barrier(h, S(s)); });
  m.def("comm_wait_probe", [](const SymmetricHeap& h, unsigned int want, unsigned long long bound_ns, uintptr_t s) {
    comm_wait_probe(h, want, bound_ns, S(s));
  });
}

}  // namespace uhfs
