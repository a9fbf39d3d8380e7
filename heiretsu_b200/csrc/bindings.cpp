// Python bindings of the heiretsu_b200 native extension (module `_C`).
#include <torch/extension.h>

#include "ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "heiretsu_b200 sm_100a kernels and runtime";
  m.def("read_and_clear_status", &hb::read_and_clear_status, "Read and clear the device status word");
  m.def("gemm", &hb::gemm, "tcgen05 GEMM with fused epilogue", py::arg("a"), py::arg("b"), py::arg("c"),
        py::arg("N"), py::arg("epi"), py::arg("a_mn"), py::arg("b_mn"), py::arg("bias") = py::none(),
        py::arg("aux") = py::none(), py::arg("resid") = py::none(), py::arg("block_n") = 128);
}
