// fgt_native.cpp — the Python extension `fugatensor_b200._native`: prepared
// programs of the C ABI (include/fgt.h) for the engine's cache-hit dispatch.
//
// Shape of the reference's native session API for this path:
// Session.prepare_program(..., graph) returns a PreparedProgram whose run
// enqueues the whole plan, replayed as one CUDA graph
// (cpp/ask_runtime.cpp:789-843; Python side src/fugatensor/_ask/executable.py:120-152),
// and the cache-hit dispatch calls it natively (cpp/lazy.cpp:946-948).
// Here prepare_program(spec_handle, graph) wraps fgt_program_create and
// Program.run wraps fgt_program_run with the GIL released; buffers cross as
// integer device addresses. Statuses are returned as integers (the Python
// layer reads fgt_last_error() on the same thread and raises).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "fgt.h"

namespace py = pybind11;

namespace {

class Program {
 public:
  Program(uintptr_t spec, bool graph) {
    const fgt_status st = fgt_program_create(reinterpret_cast<const fgt_spec*>(spec), graph ? 1 : 0, &p_);
    if (st != FGT_OK) throw std::runtime_error(std::string("fgt_program_create: ") + fgt_last_error());
    graph_ = graph;
  }
  ~Program() { fgt_program_destroy(p_); }
  Program(const Program&) = delete;
  Program& operator=(const Program&) = delete;

  int run(const std::vector<uintptr_t>& inputs, const std::vector<uintptr_t>& outputs, uintptr_t workspace,
          size_t workspace_bytes, uintptr_t stream) {
    fgt_status st;
    {
      py::gil_scoped_release release;
      st = fgt_program_run(p_, reinterpret_cast<const void* const*>(inputs.data()),
                           reinterpret_cast<void* const*>(outputs.data()), reinterpret_cast<void*>(workspace),
                           workspace_bytes, reinterpret_cast<void*>(stream));
    }
    return (int)st;
  }
  int kernel_count() const { return fgt_program_kernel_count(p_); }
  bool graph() const { return graph_; }

 private:
  fgt_program* p_ = nullptr;
  bool graph_ = true;
};

}  // namespace

PYBIND11_MODULE(_native, m) {
  m.doc() = "prepared programs of the fgt C ABI (CUDA graph replay of a partition's kernels)";
  m.def("abi_version", &fgt_abi_version);
  py::class_<Program>(m, "Program")
      .def_property_readonly("kernel_count", &Program::kernel_count)
      .def_property_readonly("graph", &Program::graph)
      .def("run", &Program::run, py::arg("inputs"), py::arg("outputs"), py::arg("workspace"),
           py::arg("workspace_bytes"), py::arg("stream"));
  m.def(
      "prepare_program",
      [](uintptr_t spec, bool graph) { return new Program(spec, graph); }, py::arg("spec"), py::arg("graph") = true,
      py::return_value_policy::take_ownership);
}
