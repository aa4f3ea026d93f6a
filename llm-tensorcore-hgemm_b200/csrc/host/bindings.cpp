// pybind11 module llm_hgemm._C: the four functions of the reference module
// (reference csrc/bindings.cpp:6-14, same defaults) plus introspection and
// the FP32-output entry used by the tensor-parallel MLP.
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "hgemm.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "B200 (sm_100a) tcgen05 HGEMM backends";
    m.def("hgemm", &hgemm, py::arg("a"), py::arg("b"), py::arg("implementation") = "auto",
          py::arg("epilogue") = "none", py::arg("bias") = py::none(), py::arg("residual") = py::none());
    m.def("hgemm_out", &hgemm_out, py::arg("a"), py::arg("b"), py::arg("out"),
          py::arg("implementation"), py::arg("epilogue") = "none", py::arg("bias") = py::none(),
          py::arg("residual") = py::none());
    m.def("has_cutlass", &has_cutlass);
    m.def("backend_info", &backend_info, py::arg("implementation"), py::arg("m") = 0, py::arg("n") = 0,
          py::arg("k") = 0);
    m.def("hgemm_out_f32", &hgemm_out_f32, py::arg("a"), py::arg("b"), py::arg("out"),
          py::arg("implementation") = "auto");
    m.def("implementations", &implementations);
    m.def("resolve", &resolve, py::arg("a"), py::arg("b"), py::arg("implementation") = "auto");
}
