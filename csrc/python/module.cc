// The `furiosa_opt_engine._native` extension: the engine's Python surface and its raw kernel
// launchers (`_native.ops`).
#include <pybind11/pybind11.h>

namespace py = pybind11;

void bind_ops(py::module_& m);
void bind_engine(py::module_& m);
void bind_encoder(py::module_& m);
void bind_emulate(py::module_& m);

PYBIND11_MODULE(_native, m) {
  m.doc() = "Native engine of furiosa_opt_engine for NVIDIA Blackwell (sm_100a).";
  py::module_ ops = m.def_submodule("ops", "Raw kernel launchers (device addresses and streams).");
  bind_ops(ops);
  bind_engine(m);
  bind_encoder(m);
  bind_emulate(m);
}
