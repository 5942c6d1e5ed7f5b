// Python bindings for the tinytron_b200 CUDA extension (sm_100a only).
#include <torch/extension.h>

namespace tt {
void gemm_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool a_mn, bool b_mn, bool accumulate, double alpha,
             c10::optional<torch::Tensor> alpha_t, int64_t bn);
void gemm_swiglu_op(torch::Tensor x, torch::Tensor w_gu, torch::Tensor out, c10::optional<torch::Tensor> gu_out);
void gemm_dswiglu_op(torch::Tensor dy, torch::Tensor w_down, torch::Tensor gu, torch::Tensor dgu, double alpha);
int64_t status_read(int64_t device);
void status_clear(int64_t device);
void add_rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> delta, torch::Tensor w,
                     c10::optional<torch::Tensor> x_out, torch::Tensor h, torch::Tensor rstd, double eps);
void rmsnorm_bwd(torch::Tensor gh, torch::Tensor x, torch::Tensor rstd, torch::Tensor w,
                 c10::optional<torch::Tensor> g_res, c10::optional<torch::Tensor> gx,
                 c10::optional<torch::Tensor> g_delta, torch::Tensor dw, bool accumulate_dw, torch::Tensor scratch);
int64_t rmsnorm_bwd_scratch_numel(int64_t M, int64_t D);
void rope_inplace(torch::Tensor qkv, torch::Tensor cos_t, torch::Tensor sin_t, int64_t T, int64_t pos_offset,
                  int64_t n_heads, int64_t head_dim, bool inverse);
void cross_entropy_fwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss,
                       c10::optional<torch::Tensor> lse, int64_t ignore_index, bool write_grad);
void embedding_fwd(torch::Tensor idx, torch::Tensor table, torch::Tensor out);
void embedding_bwd(torch::Tensor idx, torch::Tensor g, torch::Tensor gtable);
void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
                double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                c10::optional<torch::Tensor> grad_scale);
void sumsq(torch::Tensor x, torch::Tensor out, torch::Tensor scratch, bool accumulate);
void clip_coef(torch::Tensor sumsq_t, torch::Tensor norm_out, torch::Tensor coef_out, double max_norm);
void attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t q_col0, int64_t k_col0, int64_t v_col0,
              int64_t B, int64_t T, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor o,
              c10::optional<torch::Tensor> lse, double scale, bool causal, int64_t causal_offset);
void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
              int64_t q_col0, int64_t k_col0, int64_t v_col0, torch::Tensor lse, int64_t B, int64_t T, int64_t Hq,
              int64_t Hkv, int64_t D, torch::Tensor dq, int64_t dq_col0, torch::Tensor dk, int64_t dk_col0,
              torch::Tensor dv, int64_t dv_col0, torch::Tensor dq_acc, torch::Tensor delta, double scale,
              bool causal);
}  // namespace tt

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tinytron_b200 sm_100a kernels";
  m.def("gemm", &tt::gemm_op, "C (+)= alpha * op(A) op(B)^T on tcgen05", py::arg("a"), py::arg("b"), py::arg("c"),
        py::arg("a_mn") = false, py::arg("b_mn") = false, py::arg("accumulate") = false, py::arg("alpha") = 1.0,
        py::arg("alpha_t") = py::none(), py::arg("bn") = 0);
  m.def("gemm_swiglu", &tt::gemm_swiglu_op, "silu(x Wg^T) * (x Wu^T) with fused gate|up weight", py::arg("x"),
        py::arg("w_gu"), py::arg("out"), py::arg("gu_out") = py::none());
  m.def("gemm_dswiglu", &tt::gemm_dswiglu_op, "SwiGLU backward fused into the down-proj dgrad", py::arg("dy"),
        py::arg("w_down"), py::arg("gu"), py::arg("dgu"), py::arg("alpha") = 1.0);
  m.def("status_read", &tt::status_read, "read the device status word");
  m.def("status_clear", &tt::status_clear, "clear the device status word");
  m.def("add_rmsnorm_fwd", &tt::add_rmsnorm_fwd, "x_out = x + delta; h = bf16(w * rmsnorm(x_out))");
  m.def("rmsnorm_bwd", &tt::rmsnorm_bwd, "RMSNorm backward (+ residual grad), deterministic dw");
  m.def("rmsnorm_bwd_scratch_numel", &tt::rmsnorm_bwd_scratch_numel);
  m.def("rope_inplace", &tt::rope_inplace, "HF half-split RoPE in place on the packed qkv buffer");
  m.def("cross_entropy_fwd", &tt::cross_entropy_fwd, "per-row CE loss/LSE; optional in-place grad");
  m.def("embedding_fwd", &tt::embedding_fwd);
  m.def("embedding_bwd", &tt::embedding_bwd);
  m.def("adamw_step", &tt::adamw_step, "fused AdamW over flat fp32 buffers (+ bf16 shadow)");
  m.def("sumsq", &tt::sumsq);
  m.def("clip_coef", &tt::clip_coef);
  m.def("attn_fwd", &tt::attn_fwd, "flash attention forward (tcgen05, GQA-native)");
  m.def("attn_bwd", &tt::attn_bwd, "flash attention backward (tcgen05, GQA-native, dQ via fp32 atomics)");
}
