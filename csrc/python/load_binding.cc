// Checkpoints and load options (filled in by the checkpoint layer).
#include <pybind11/pybind11.h>
namespace py = pybind11;
void bind_checkpoint_and_load(py::module_& m) { (void)m; }
