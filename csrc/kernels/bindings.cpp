// Python bindings of the sm_100a kernels: module rs_nanogpt_b200._C.
#include <torch/extension.h>

#include "status.h"

namespace nk {
void gemm(torch::Tensor A, bool a_mn_major, torch::Tensor B, bool b_mn_major, torch::Tensor C, int64_t mode,
          double alpha, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> aux_out, int64_t splits,
          int64_t block_n);
void rmsnorm_fwd(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> rstd, double eps);
void rmsnorm_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor rstd, torch::Tensor dx, bool accum);
void rope_qknorm_fwd(torch::Tensor qkv, torch::Tensor rstd, torch::Tensor cos_t, torch::Tensor sin_t, int64_t T,
                     int64_t t0, int64_t H, double eps);
void rope_qknorm_bwd(torch::Tensor qkv, torch::Tensor dqkv, torch::Tensor rstd, torch::Tensor cos_t,
                     torch::Tensor sin_t, int64_t T, int64_t H);
void embedding_fwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor out);
void embedding_bwd(torch::Tensor idx, torch::Tensor dx, torch::Tensor grad);
void softmax_xent(torch::Tensor logits, torch::Tensor targets, c10::optional<torch::Tensor> nll, double grad_scale,
                  bool write_grad);
void xent_from_stats(torch::Tensor logits, torch::Tensor stats, torch::Tensor targets,
                     c10::optional<torch::Tensor> nll, double grad_scale, bool write_grad);
void gemm_logits_stats(torch::Tensor x, torch::Tensor w, torch::Tensor logits, torch::Tensor stats);
void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> work,
                double lr, double b1, double b2, double eps, double wd, int64_t step, double grad_scale);
void sumsq(torch::Tensor x, torch::Tensor out);
void flash_fwd(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H);
void flash_bwd(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dsum,
               torch::Tensor dqkv, int64_t B, int64_t T, int64_t H);
void ddp_barrier(int64_t pads_dev, int64_t rank, int64_t world, int64_t epoch);
void ddp_rs_adam_ag(int64_t grads_dev, int64_t works_dev, int64_t world, torch::Tensor master, torch::Tensor m,
                    torch::Tensor v, int64_t shard_lo, int64_t shard_hi, torch::Tensor groups, double grad_scale,
                    c10::optional<torch::Tensor> sumsq, int64_t mv_base, int64_t mc_grad, int64_t mc_work,
                    int64_t max_ctas);
void flash_fwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t T, int64_t H);
bool flash_fwd_tc_supported(int64_t T, int64_t HD);
void flash_bwd_tc(torch::Tensor qkv, torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dsum,
                  torch::Tensor dq_acc, torch::Tensor dqkv, int64_t B, int64_t T, int64_t H,
                  c10::optional<torch::Tensor> rope_rstd, c10::optional<torch::Tensor> rope_cos,
                  c10::optional<torch::Tensor> rope_sin, bool prepared);
void flash_bwd_prep(torch::Tensor out, torch::Tensor dout, torch::Tensor dsum, torch::Tensor dq_acc, int64_t B,
                    int64_t T, int64_t H);
bool flash_bwd_tc_supported(int64_t T, int64_t HD);
torch::Tensor flash_bwd_trace();
void gemm_qkv_rope(torch::Tensor x, torch::Tensor w, torch::Tensor qkv, torch::Tensor rstd, torch::Tensor cos_t,
                   torch::Tensor sin_t, int64_t T, int64_t H, double eps);
void kv_rope_append(torch::Tensor qkv, torch::Tensor k_cache, torch::Tensor v_cache, c10::optional<torch::Tensor> pos,
                    c10::optional<torch::Tensor> lens, int64_t rows_per_seq, int64_t H, torch::Tensor cos_t,
                    torch::Tensor sin_t, bool do_rope, double eps);
void decode_attention(torch::Tensor qkv, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor pos,
                      torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, int64_t chunk);
void sample_tokens(torch::Tensor logits, double temperature, int64_t top_k, torch::Tensor uniforms,
                   torch::Tensor gen_count, torch::Tensor out_tokens, torch::Tensor next_in, torch::Tensor pos,
                   bool advance_pos);
void skinny_finish(torch::Tensor acc, torch::Tensor out, int64_t mode, c10::optional<torch::Tensor> aux,
                   c10::optional<torch::Tensor> aux_out, c10::optional<torch::Tensor> norm_out, double eps);
void qkv_decode_finish(torch::Tensor acc, torch::Tensor qkv, torch::Tensor k_cache, torch::Tensor v_cache,
                       torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t, int64_t H, double eps);
void gemm_skinny_acc(torch::Tensor w, torch::Tensor x, torch::Tensor acc, int64_t splits);
void set_pdl(bool on);
torch::Tensor gemm_trace();
}  // namespace nk

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels (tcgen05 GEMM, attention, norms, loss, optimizer, comm)";
  m.def("gemm", &nk::gemm, "tcgen05 bf16 GEMM with fused epilogues", py::arg("A"), py::arg("a_mn_major"),
        py::arg("B"), py::arg("b_mn_major"), py::arg("C"), py::arg("mode"), py::arg("alpha"), py::arg("aux"),
        py::arg("aux_out"), py::arg("splits"), py::arg("block_n"));
  m.def("gemm_qkv_rope", &nk::gemm_qkv_rope);
  m.def("kernel_status", &nk::kernel_status, "device error word of the kernels (0 = ok)", py::arg("reset") = true);
  m.def("rmsnorm_fwd", &nk::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &nk::rmsnorm_bwd);
  m.def("rope_qknorm_fwd", &nk::rope_qknorm_fwd);
  m.def("rope_qknorm_bwd", &nk::rope_qknorm_bwd);
  m.def("embedding_fwd", &nk::embedding_fwd);
  m.def("embedding_bwd", &nk::embedding_bwd);
  m.def("softmax_xent", &nk::softmax_xent);
  m.def("xent_from_stats", &nk::xent_from_stats);
  m.def("gemm_logits_stats", &nk::gemm_logits_stats);
  m.def("adamw_step", &nk::adamw_step);
  m.def("sumsq", &nk::sumsq);
  m.def("flash_fwd", &nk::flash_fwd);
  m.def("flash_bwd", &nk::flash_bwd);
  m.def("flash_fwd_tc", &nk::flash_fwd_tc);
  m.def("flash_bwd_tc", &nk::flash_bwd_tc, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"),
        py::arg("dsum"), py::arg("dq_acc"), py::arg("dqkv"), py::arg("B"), py::arg("T"), py::arg("H"),
        py::arg("rope_rstd") = py::none(), py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none(),
        py::arg("prepared") = false);
  m.def("flash_bwd_prep", &nk::flash_bwd_prep);
  m.def("flash_bwd_tc_supported", &nk::flash_bwd_tc_supported);
  m.def("flash_bwd_trace", &nk::flash_bwd_trace, "timeline of the first CTA of the last traced backward (measurement)");
  m.def("flash_fwd_tc_supported", &nk::flash_fwd_tc_supported);
  m.def("ddp_barrier", &nk::ddp_barrier);
  m.def("ddp_rs_adam_ag", &nk::ddp_rs_adam_ag, py::arg("grads_dev"), py::arg("works_dev"), py::arg("world"),
        py::arg("master"), py::arg("m"), py::arg("v"), py::arg("shard_lo"), py::arg("shard_hi"), py::arg("groups"),
        py::arg("grad_scale"), py::arg("sumsq"), py::arg("mv_base") = 0, py::arg("mc_grad") = 0,
        py::arg("mc_work") = 0, py::arg("max_ctas") = 0);
  m.def("kv_rope_append", &nk::kv_rope_append);
  m.def("decode_attention", &nk::decode_attention);
  m.def("sample_tokens", &nk::sample_tokens);
  m.def("skinny_finish", &nk::skinny_finish);
  m.def("qkv_decode_finish", &nk::qkv_decode_finish);
  m.def("gemm_skinny_acc", &nk::gemm_skinny_acc);
  m.def("gemm_trace", &nk::gemm_trace, "MMA-warp wait accounting of the last traced GEMM (measurement)");
  m.def("set_pdl", &nk::set_pdl, "programmatic dependent launch for the decode-chain kernels");
}
