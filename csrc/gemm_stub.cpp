#include <torch/extension.h>
namespace py = pybind11;
void register_gemm(py::module_& m) { (void)m; }
