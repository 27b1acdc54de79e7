// Python bindings of the bounds-checked debug build: module
// rs_nanogpt_b200._C_bounds. It carries the tile-indexed tcgen05 kernels
// (GEMM, flash-attention forward and backward) compiled with
// NANOGPT_DEBUG_BOUNDS: an out-of-range or misaligned TMA coordinate, bulk-copy
// offset or row index records error code 5 in this module's own error word
// (read with kernel_status) and the access is skipped. This stands in for
// compute-sanitizer, which is not available on the GPU pool.
#include <torch/extension.h>

#include "../status.h"

namespace nk {
void gemm(torch::Tensor A, bool a_mn_major, torch::Tensor B, bool b_mn_major, torch::Tensor C, int64_t mode,
          double alpha, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> aux_out, int64_t splits,
          int64_t block_n);
void flash_fwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H);
void flash_bwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dsum,
                  torch::Tensor dq_acc, torch::Tensor dqkv, int64_t B, int64_t T, int64_t H,
                  c10::optional<torch::Tensor> rope_rstd, c10::optional<torch::Tensor> rope_cos,
                  c10::optional<torch::Tensor> rope_sin, bool prepared);
void gemm_qkv_rope(torch::Tensor x, torch::Tensor w, torch::Tensor qkv, torch::Tensor rstd, torch::Tensor cos_t,
                   torch::Tensor sin_t, int64_t T, int64_t H, double eps);
}  // namespace nk

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "bounds-checked debug build of the tcgen05 GEMM and flash-attention kernels";
  m.def("kernel_status", &nk::kernel_status, py::arg("reset") = true);
  m.def("gemm", &nk::gemm);
  m.def("gemm_qkv_rope", &nk::gemm_qkv_rope);
  m.def("flash_fwd_tc", &nk::flash_fwd_tc);
  m.def("flash_bwd_tc", &nk::flash_bwd_tc, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"),
        py::arg("dsum"), py::arg("dq_acc"), py::arg("dqkv"), py::arg("B"), py::arg("T"), py::arg("H"),
        py::arg("rope_rstd") = py::none(), py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none(),
        py::arg("prepared") = false);
}
