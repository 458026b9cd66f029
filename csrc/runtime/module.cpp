// Module openmini_v1_b200._rt: host-side C++ runtime (no CUDA).
#include <pybind11/pybind11.h>

namespace py = pybind11;

void bind_block_manager(py::module_& m);
void bind_ipc(py::module_& m);
void bind_gguf(py::module_& m);

PYBIND11_MODULE(_rt, m) {
  m.doc() = "openmini_v1_b200 native runtime: block manager, IPC framing, GGUF index";
  bind_block_manager(m);
  bind_ipc(m);
  bind_gguf(m);
}
