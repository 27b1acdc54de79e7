// Python bindings of the sm_100a kernels: module rs_nanogpt_b200._C.
#include <torch/extension.h>

#include "status.h"

namespace nk {
void gemm(torch::Tensor A, bool a_mn_major, torch::Tensor B, bool b_mn_major, torch::Tensor C, int64_t mode,
          double alpha, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> aux_out, int64_t splits,
          int64_t block_n);
}  // namespace nk

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels (tcgen05 GEMM, attention, norms, loss, optimizer, comm)";
  m.def("gemm", &nk::gemm, "tcgen05 bf16 GEMM with fused epilogues", py::arg("A"), py::arg("a_mn_major"),
        py::arg("B"), py::arg("b_mn_major"), py::arg("C"), py::arg("mode"), py::arg("alpha"), py::arg("aux"),
        py::arg("aux_out"), py::arg("splits"), py::arg("block_n"));
  m.def("kernel_status", &nk::kernel_status, "device error word of the kernels (0 = ok)", py::arg("reset") = true);
}
