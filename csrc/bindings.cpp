// Python bindings for the tinytron_b200 CUDA extension (sm_100a only).
#include <torch/extension.h>

namespace tt {
void gemm_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool a_mn, bool b_mn, bool accumulate, double alpha,
             c10::optional<torch::Tensor> alpha_t, int64_t bn);
void gemm_axpby_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool b_mn, double alpha,
                   c10::optional<torch::Tensor> addend, double beta, bool symmetric, int64_t batch);
void gemm_set_pair_mode(int64_t mode);
int64_t gemm_pair_mode();
void gemm_swiglu_op(torch::Tensor x, torch::Tensor w_gu, torch::Tensor out, c10::optional<torch::Tensor> gu_out);
void gemm_dswiglu_op(torch::Tensor dy, torch::Tensor w_down, torch::Tensor gu, torch::Tensor dgu, double alpha);
void moe_gemm_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_off, int64_t n_groups,
                 bool b_mn, int64_t b_grp_rows, int64_t b_split_k, int64_t b_off2, bool pair,
                 c10::optional<torch::Tensor> row_ptr);
void moe_gemm_swiglu_op(torch::Tensor x, torch::Tensor w_gu, torch::Tensor out, torch::Tensor gu_out,
                        torch::Tensor grp_off, int64_t n_groups, bool pair);
void moe_gemm_dswiglu_op(torch::Tensor dy, torch::Tensor w_down, torch::Tensor gu, torch::Tensor dgu,
                         torch::Tensor grp_off, int64_t n_groups, bool pair);
void moe_topk_softmax_op(torch::Tensor logits, int64_t k, torch::Tensor w, torch::Tensor sel);
void skinny_linear_op(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t publish_gid, int64_t slot_off,
                      int64_t slot_bytes);
void moe_skinny_swiglu_op(torch::Tensor xr, torch::Tensor w_gu, torch::Tensor grp_off, int64_t E, torch::Tensor act);
void moe_skinny_down_combine_op(torch::Tensor act, torch::Tensor wd, torch::Tensor grp_off, int64_t E,
                                torch::Tensor slot, c10::optional<torch::Tensor> w, int64_t k, torch::Tensor out,
                                c10::optional<torch::Tensor> row_limit, int64_t publish_gid, int64_t slot_off,
                                int64_t slot_bytes);
void moe_topk_softmax_bwd_op(torch::Tensor dw, torch::Tensor w, torch::Tensor sel, torch::Tensor dlogits);
int64_t moe_row_capacity(int64_t P, int64_t E, int64_t align);
void moe_layout_op(torch::Tensor sel, int64_t E, torch::Tensor grp_off, torch::Tensor slot, torch::Tensor row_pair,
                   int64_t align, int64_t remap_lo);
void moe_gather_rows_op(torch::Tensor x, torch::Tensor row_pair, torch::Tensor grp_off, int64_t k, torch::Tensor out);
void moe_combine_op(torch::Tensor y_rows, torch::Tensor slot, c10::optional<torch::Tensor> w, int64_t k,
                    torch::Tensor out, c10::optional<torch::Tensor> row_limit);
void moe_combine_bwd_op(torch::Tensor dout, torch::Tensor y_rows, torch::Tensor row_pair, torch::Tensor w,
                        torch::Tensor grp_off, int64_t k, torch::Tensor dy_rows, torch::Tensor dw);
void moe_gemm_wgrad_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_off, int64_t n_groups,
                       bool accumulate, bool pair);
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
int64_t attn_bwd_scratch_numel(int64_t B, int64_t Hq, int64_t T);
void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
              int64_t q_col0, int64_t k_col0, int64_t v_col0, torch::Tensor lse, int64_t B, int64_t T, int64_t Hq,
              int64_t Hkv, int64_t D, torch::Tensor dq, int64_t dq_col0, torch::Tensor dk, int64_t dk_col0,
              torch::Tensor dv, int64_t dv_col0, torch::Tensor dq_acc, torch::Tensor scratch, double scale,
              bool causal);
void exp2_poly_op(torch::Tensor x, torch::Tensor y);
void decode_rope_append(torch::Tensor qkv, int64_t B, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                        c10::optional<torch::Tensor> pos_dev, int64_t pos_host, torch::Tensor cos_t,
                        torch::Tensor sin_t, torch::Tensor q_out, torch::Tensor k_pages, torch::Tensor v_pages,
                        torch::Tensor page_table);
int64_t decode_num_splits(int64_t max_len);
void sample_tokens(torch::Tensor logits, double temperature, int64_t top_k, double top_p, int64_t seed,
                   int64_t offset, torch::Tensor tokens, c10::optional<torch::Tensor> logprob,
                   c10::optional<torch::Tensor> rng);
void decode_advance(torch::Tensor nxt, torch::Tensor tokens, int64_t P, torch::Tensor tok_in, torch::Tensor rng,
                    c10::optional<torch::Tensor> lp, c10::optional<torch::Tensor> lp_all);
void decode_attention(torch::Tensor q, torch::Tensor k_pages, torch::Tensor v_pages, torch::Tensor page_table,
                      c10::optional<torch::Tensor> len_dev, int64_t len_host, int64_t splits, double scale,
                      torch::Tensor o_part, torch::Tensor ml_part, torch::Tensor out);
void ep_allgather_counts(int64_t gid, torch::Tensor counts, int64_t dst_off);
void ep_scatter(int64_t gid, torch::Tensor x, int64_t k, torch::Tensor tgt, torch::Tensor dst, int64_t recv_off,
                int64_t cap, c10::optional<torch::Tensor> w, c10::optional<torch::Tensor> y_pairs,
                c10::optional<torch::Tensor> dw, int64_t ret_off, int64_t back_off);
void ep_local_combine(int64_t gid, int64_t y_off, int64_t k, c10::optional<torch::Tensor> w, torch::Tensor out,
                      c10::optional<torch::Tensor> y_save);
void ep_resolve_rows(int64_t gid, int64_t ret_off, int64_t rows, int64_t H, torch::Tensor row_ptr);
void ep_pull_combine(int64_t gid, int64_t y_off, int64_t cap, torch::Tensor tgt, torch::Tensor dst, int64_t k,
                     c10::optional<torch::Tensor> w, torch::Tensor out, c10::optional<torch::Tensor> y_save);
void ep_zero_pad(torch::Tensor buf, torch::Tensor seg_off, torch::Tensor seg_cnt);
void ep_plan_rows(torch::Tensor sel, torch::Tensor slot, torch::Tensor delta, int64_t E_l, torch::Tensor dst,
                  torch::Tensor tgt);
namespace comm {
int64_t comm_create(int64_t device, int64_t bytes);
torch::Tensor comm_ipc_handle(int64_t gid);
void comm_open(int64_t gid, int64_t rank, int64_t world, torch::Tensor handles);
void comm_open_emulated(std::vector<int64_t> gids, bool waits);
void comm_set_timeout(double seconds);
torch::Tensor comm_view(int64_t gid, int64_t offset_bytes, std::vector<int64_t> shape, int64_t dtype_code);
int64_t comm_user_offset();
int64_t comm_heap_base(int64_t gid);
void comm_barrier(int64_t gid, bool signal);
void comm_all_reduce(int64_t gid, int64_t in_offset, torch::Tensor out, c10::optional<torch::Tensor> residual);
void comm_reduce_scatter_sumsq(int64_t gid, int64_t grad_offset, int64_t lo, int64_t hi, int64_t split, double scale);
void comm_reduce_scatter_bucket(int64_t gid, int64_t grad_offset, int64_t lo, int64_t hi, int64_t split,
                                double scale, torch::Tensor sq_local, int64_t max_blocks);
int64_t comm_publish_sumsq(int64_t gid, torch::Tensor sq);
void comm_adamw_allgather(int64_t gid, int64_t data_offset, int64_t grad_offset, c10::optional<torch::Tensor> p16,
                          torch::Tensor m, torch::Tensor v, int64_t lo, int64_t hi, double lr, double beta1,
                          double beta2, double eps, double wd, int64_t step, double max_norm,
                          c10::optional<torch::Tensor> extra_sq, c10::optional<torch::Tensor> norm_out, int64_t pads_epoch);
void comm_shadow_refresh(int64_t gid, int64_t data_offset, torch::Tensor p16, int64_t lo, int64_t hi);
void comm_all_to_all(int64_t gid, int64_t slot_offset, torch::Tensor out);
int64_t comm_epoch(int64_t gid);
void ul_pack(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor src, int64_t B, int64_t T,
             std::vector<int64_t> rows, int64_t W, int64_t s1, int64_t s2, std::vector<int64_t> b0,
             std::vector<int64_t> b1, std::vector<int64_t> b2);
void ul_exchange(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor out, int64_t B, int64_t T,
                 std::vector<int64_t> rows, int64_t dcol_c, int64_t W);
void ul_exchange_qkv_grad(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor dqkv, int64_t B,
                          int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t hq_l, int64_t hkv_l,
                          std::vector<int64_t> kv0);
void comm_replay_publish(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor in);
void comm_replay_reduce(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor out,
                        c10::optional<torch::Tensor> residual, int64_t root);
void comm_destroy(int64_t gid);
}  // namespace comm
}  // namespace tt

namespace {
// Kernel ops dereference every tensor operand on the launching device, so each must be a
// CUDA tensor, all on one device, or pinned host memory (which the device reads directly).
// A pageable host tensor or a second device is rejected here instead of faulting in a kernel.
struct OperandDevices {
  const char* op;
  int device = -1;
  void operator()(const torch::Tensor& t) {
    if (!t.defined()) return;
    if (!t.is_cuda()) {
      TORCH_CHECK(t.is_pinned(), op, ": tensor operands must be CUDA tensors (or pinned host memory)");
      return;
    }
    if (device < 0) device = t.get_device();
    TORCH_CHECK(t.get_device() == device, op, ": tensor operands on different CUDA devices");
  }
  void operator()(const c10::optional<torch::Tensor>& t) {
    if (t.has_value()) (*this)(*t);
  }
  template <typename T>
  void operator()(const T&) {}
};

template <typename R, typename... A>
auto checked(const char* op, R (*fn)(A...)) {
  return [op, fn](A... a) -> R {
    OperandDevices check{op};
    (check(a), ...);
    return fn(std::forward<A>(a)...);
  };
}
}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tinytron_b200 sm_100a kernels";
  m.def("gemm", checked("gemm", &tt::gemm_op), "C (+)= alpha * op(A) op(B)^T on tcgen05", py::arg("a"), py::arg("b"), py::arg("c"),
        py::arg("a_mn") = false, py::arg("b_mn") = false, py::arg("accumulate") = false, py::arg("alpha") = 1.0,
        py::arg("alpha_t") = py::none(), py::arg("bn") = 0);
  m.def("gemm_axpby", checked("gemm_axpby", &tt::gemm_axpby_op), "C = alpha * A op(B)^T + beta * addend (bf16); symmetric: upper tiles mirrored",
        py::arg("a"), py::arg("b"), py::arg("c"), py::arg("b_mn") = false, py::arg("alpha") = 1.0,
        py::arg("addend") = py::none(), py::arg("beta") = 0.0, py::arg("symmetric") = false,
        py::arg("batch") = 1);
  m.def("skinny_linear", checked("skinny_linear", &tt::skinny_linear_op),
        "y[M, N] = x[M, K] w[N, K]^T for M <= 32: weight-streaming split-K tcgen05 GEMM (decode); publish_gid >= 0: "
        "y goes to that heap's all-reduce slot (published to the peers) instead of out",
        py::arg("x"), py::arg("w"), py::arg("out"), py::arg("publish_gid") = -1, py::arg("slot_off") = 0,
        py::arg("slot_bytes") = 0);
  m.def("moe_skinny_swiglu", checked("moe_skinny_swiglu", &tt::moe_skinny_swiglu_op),
        "decode experts: act = silu(x Wg_e^T) * (x Wu_e^T) over unpadded expert segments", py::arg("xr"),
        py::arg("w_gu"), py::arg("grp_off"), py::arg("E"), py::arg("act"));
  m.def("moe_skinny_down_combine", checked("moe_skinny_down_combine", &tt::moe_skinny_down_combine_op),
        "decode experts: out[n] = sum_j w[n,j] act_{slot[n,j]} Wd_e^T (pairs at or past *row_limit skipped)",
        py::arg("act"), py::arg("wd"), py::arg("grp_off"), py::arg("E"), py::arg("slot"), py::arg("w"), py::arg("k"),
        py::arg("out"), py::arg("row_limit") = py::none(), py::arg("publish_gid") = -1, py::arg("slot_off") = 0,
        py::arg("slot_bytes") = 0);
  m.def("gemm_set_pair_mode", checked("gemm_set_pair_mode", &tt::gemm_set_pair_mode), "CTA-pair GEMM: 0 never, 1 when faster, 2 always");
  m.def("gemm_pair_mode", &tt::gemm_pair_mode);
  m.def("moe_gemm", checked("moe_gemm", &tt::moe_gemm_op), "grouped GEMM over expert row segments (bf16 out)", py::arg("a"),
        py::arg("b"), py::arg("c"), py::arg("grp_off"), py::arg("n_groups"), py::arg("b_mn"), py::arg("b_grp_rows"),
        py::arg("b_split_k") = 0, py::arg("b_off2") = 0, py::arg("pair") = false, py::arg("row_ptr") = py::none());
  m.def("moe_gemm_swiglu", checked("moe_gemm_swiglu", &tt::moe_gemm_swiglu_op), "grouped gate|up GEMM with SwiGLU epilogue", py::arg("x"),
        py::arg("w_gu"), py::arg("out"), py::arg("gu_out"), py::arg("grp_off"), py::arg("n_groups"),
        py::arg("pair") = false);
  m.def("moe_gemm_dswiglu", checked("moe_gemm_dswiglu", &tt::moe_gemm_dswiglu_op), "grouped down-proj dgrad with SwiGLU backward epilogue",
        py::arg("dy"), py::arg("w_down"), py::arg("gu"), py::arg("dgu"), py::arg("grp_off"), py::arg("n_groups"),
        py::arg("pair") = false);
  m.def("moe_gemm_wgrad", checked("moe_gemm_wgrad", &tt::moe_gemm_wgrad_op), "per-expert weight gradient over token segments (fp32)",
        py::arg("a"), py::arg("b"), py::arg("c"), py::arg("grp_off"), py::arg("n_groups"), py::arg("accumulate"),
        py::arg("pair") = false);
  m.def("moe_topk_softmax", checked("moe_topk_softmax", &tt::moe_topk_softmax_op), "router top-k + softmax over the selected logits");
  m.def("moe_topk_softmax_bwd", checked("moe_topk_softmax_bwd", &tt::moe_topk_softmax_bwd_op), "backward of moe_topk_softmax");
  m.def("moe_row_capacity", checked("moe_row_capacity", &tt::moe_row_capacity), "padded expert-row capacity for P pairs and E experts",
        py::arg("P"), py::arg("E"), py::arg("align") = 128);
  m.def("moe_layout", checked("moe_layout", &tt::moe_layout_op),
        "expert segments (1-, 128- or 256-row aligned, stable) for the grouped GEMMs; remap_lo >= 0: ids "
        "sel - remap_lo in [0, E - 1) are local experts, all others go to group E - 1",
        py::arg("sel"), py::arg("E"), py::arg("grp_off"), py::arg("slot"), py::arg("row_pair"), py::arg("align") = 128,
        py::arg("remap_lo") = -1);
  m.def("moe_gather_rows", checked("moe_gather_rows", &tt::moe_gather_rows_op), "x_rows[r] = x[token of row r], zero pad rows");
  m.def("moe_combine", checked("moe_combine", &tt::moe_combine_op), "out[t] = sum_j w[t,j] y_rows[slot[t,j]] (slots below row_limit)",
        py::arg("y_rows"), py::arg("slot"), py::arg("w"), py::arg("k"), py::arg("out"),
        py::arg("row_limit") = py::none());
  m.def("moe_combine_bwd", checked("moe_combine_bwd", &tt::moe_combine_bwd_op), "backward of moe_combine (dy_rows, dw)");
  m.def("gemm_swiglu", checked("gemm_swiglu", &tt::gemm_swiglu_op), "silu(x Wg^T) * (x Wu^T) with fused gate|up weight", py::arg("x"),
        py::arg("w_gu"), py::arg("out"), py::arg("gu_out") = py::none());
  m.def("gemm_dswiglu", checked("gemm_dswiglu", &tt::gemm_dswiglu_op), "SwiGLU backward fused into the down-proj dgrad", py::arg("dy"),
        py::arg("w_down"), py::arg("gu"), py::arg("dgu"), py::arg("alpha") = 1.0);
  m.def("status_read", checked("status_read", &tt::status_read), "read the device status word");
  m.def("status_clear", checked("status_clear", &tt::status_clear), "clear the device status word");
  m.def("add_rmsnorm_fwd", checked("add_rmsnorm_fwd", &tt::add_rmsnorm_fwd), "x_out = x + delta; h = bf16(w * rmsnorm(x_out))");
  m.def("rmsnorm_bwd", checked("rmsnorm_bwd", &tt::rmsnorm_bwd), "RMSNorm backward (+ residual grad), deterministic dw");
  m.def("rmsnorm_bwd_scratch_numel", &tt::rmsnorm_bwd_scratch_numel);
  m.def("rope_inplace", checked("rope_inplace", &tt::rope_inplace), "HF half-split RoPE in place on the packed qkv buffer");
  m.def("cross_entropy_fwd", checked("cross_entropy_fwd", &tt::cross_entropy_fwd), "per-row CE loss/LSE; optional in-place grad");
  m.def("embedding_fwd", checked("embedding_fwd", &tt::embedding_fwd));
  m.def("embedding_bwd", checked("embedding_bwd", &tt::embedding_bwd));
  m.def("adamw_step", checked("adamw_step", &tt::adamw_step), "fused AdamW over flat fp32 buffers (+ bf16 shadow)");
  m.def("sumsq", checked("sumsq", &tt::sumsq));
  m.def("clip_coef", checked("clip_coef", &tt::clip_coef));
  m.def("exp2_poly", checked("exp2_poly", &tt::exp2_poly_op), "2^x via the FMA-pipe polynomial (test hook)");
  m.def("attn_fwd", checked("attn_fwd", &tt::attn_fwd), "flash attention forward (tcgen05, GQA-native)");
  m.def("attn_bwd_scratch_numel", checked("attn_bwd_scratch_numel", &tt::attn_bwd_scratch_numel), "fp32 scratch elements attn_bwd needs");
  m.def("attn_bwd", checked("attn_bwd", &tt::attn_bwd), "flash attention backward (tcgen05, GQA-native, dQ via fp32 atomics)");
  m.def("decode_rope_append", checked("decode_rope_append", &tt::decode_rope_append), "RoPE on q/k + paged KV-cache append (device position)");
  m.def("sample_tokens", checked("sample_tokens", &tt::sample_tokens), "temperature/top-k/top-p sampling in one kernel (Philox draw)",
        py::arg("logits"), py::arg("temperature"), py::arg("top_k"), py::arg("top_p"), py::arg("seed"),
        py::arg("offset"), py::arg("tokens"), py::arg("logprob") = py::none(), py::arg("rng") = py::none());
  m.def("decode_advance", checked("decode_advance", &tt::decode_advance),
        "decode step bookkeeping on the device: tokens[:, P + step] = nxt, token input = nxt, log-prob column "
        "step, step += 1 (step = rng[1])",
        py::arg("nxt"), py::arg("tokens"), py::arg("P"), py::arg("tok_in"), py::arg("rng"), py::arg("lp") = py::none(),
        py::arg("lp_all") = py::none());
  m.def("decode_num_splits", checked("decode_num_splits", &tt::decode_num_splits), "split-KV CTAs per (sequence, kv head) for a max length");
  m.def("decode_attention", checked("decode_attention", &tt::decode_attention), "split-KV paged decode attention (GQA-native) + combine");
  m.def("ep_allgather_counts", checked("ep_allgather_counts", &tt::ep_allgather_counts), "EP: all-gather per-expert counts into the heap");
  m.def("ep_scatter", checked("ep_scatter", &tt::ep_scatter), "EP dispatch: pair rows to their owners' receive buffers (peer stores)",
        py::arg("gid"), py::arg("x"), py::arg("k"), py::arg("tgt"), py::arg("dst"), py::arg("recv_off"),
        py::arg("cap"), py::arg("w") = py::none(), py::arg("y_pairs") = py::none(), py::arg("dw") = py::none(),
        py::arg("ret_off") = -1, py::arg("back_off") = 0);
  m.def("ep_local_combine", checked("ep_local_combine", &tt::ep_local_combine),
        "EP combine after a pushed exchange: weighted sum of this rank's own return buffer", py::arg("gid"),
        py::arg("y_off"), py::arg("k"), py::arg("w"), py::arg("out"), py::arg("y_save") = py::none());
  m.def("ep_resolve_rows", checked("ep_resolve_rows", &tt::ep_resolve_rows),
        "EP: recorded return slots of received rows -> peer addresses for the GEMM epilogue", py::arg("gid"),
        py::arg("ret_off"), py::arg("rows"), py::arg("H"), py::arg("row_ptr"));
  m.def("ep_pull_combine", checked("ep_pull_combine", &tt::ep_pull_combine), "EP combine: weighted sum of owners' rows (peer loads)",
        py::arg("gid"), py::arg("y_off"), py::arg("cap"), py::arg("tgt"), py::arg("dst"), py::arg("k"),
        py::arg("w"), py::arg("out"), py::arg("y_save") = py::none());
  m.def("ep_zero_pad", checked("ep_zero_pad", &tt::ep_zero_pad), "zero the padding rows of expert segments");
  m.def("ep_plan_rows", checked("ep_plan_rows", &tt::ep_plan_rows),
        "EP pair destinations: dst = slot + delta[e], tgt = e / E_l (slot: position in the stable expert order)");
  // tt_comm: symmetric heap over CUDA IPC + device-initiated collectives (csrc/runtime/comm.cu)
  m.def("comm_create", checked("comm_create", &tt::comm::comm_create), "allocate a symmetric heap on a device; returns a group id");
  m.def("comm_ipc_handle", checked("comm_ipc_handle", &tt::comm::comm_ipc_handle), "64-byte CUDA IPC handle of the group's heap");
  m.def("comm_open", &tt::comm::comm_open, "map every peer's heap (handles uint8 [world, 64])");
  m.def("comm_open_emulated", checked("comm_open_emulated", &tt::comm::comm_open_emulated), "single-GPU test mode: groups act as ranks",
        py::arg("gids"), py::arg("waits") = false);
  m.def("comm_set_timeout", checked("comm_set_timeout", &tt::comm::comm_set_timeout), "bound (seconds) on every device-side wait");
  m.def("comm_view", checked("comm_view", &tt::comm::comm_view), "tensor view into the local heap");
  m.def("comm_user_offset", checked("comm_user_offset", &tt::comm::comm_user_offset), "first byte of the heap's user region");
  m.def("comm_heap_base", checked("comm_heap_base", &tt::comm::comm_heap_base), "device address of the local heap");
  m.def("comm_barrier", checked("comm_barrier", &tt::comm::comm_barrier), "device-side barrier over the group (bounded wait)",
        py::arg("gid"), py::arg("signal") = true);
  m.def("comm_all_reduce", checked("comm_all_reduce", &tt::comm::comm_all_reduce), "one-shot all-reduce of a heap region (+ residual)",
        py::arg("gid"), py::arg("in_offset"), py::arg("out"), py::arg("residual") = py::none());
  m.def("ul_pack", checked("ul_pack", &tt::comm::ul_pack), "Ulysses: gather this rank's outgoing chunks into its send slot and signal");
  m.def("ul_exchange", checked("ul_exchange", &tt::comm::ul_exchange), "Ulysses: wait, load chunk `me` of every peer into out (remapped)");
  m.def("ul_exchange_qkv_grad", checked("ul_exchange_qkv_grad", &tt::comm::ul_exchange_qkv_grad),
        "Ulysses backward of the q|k|v direction: d(q|k|v) summed over ranks sharing a kv head");
  m.def("comm_replay_publish", checked("comm_replay_publish", &tt::comm::comm_replay_publish),
        "graph-safe collective, step 1: copy the input into this rank's slot and signal (device epoch)");
  m.def("comm_replay_reduce", checked("comm_replay_reduce", &tt::comm::comm_replay_reduce),
        "graph-safe collective, step 2: wait, sum the ranks' slots (root >= 0: copy the root's) (+ residual)",
        py::arg("gid"), py::arg("slot_offset"), py::arg("slot_bytes"), py::arg("out"), py::arg("residual") = py::none(),
        py::arg("root") = -1);
  m.def("comm_reduce_scatter_sumsq", checked("comm_reduce_scatter_sumsq", &tt::comm::comm_reduce_scatter_sumsq),
        "ZeRO-1 fp32 gradient reduce-scatter in place + published sums of squares");
  m.def("comm_adamw_allgather", checked("comm_adamw_allgather", &tt::comm::comm_adamw_allgather),
        "ZeRO-1 clip + AdamW on the owned shard + fp32 all-gather by peer stores", py::arg("gid"),
        py::arg("data_offset"), py::arg("grad_offset"), py::arg("p16"), py::arg("m"), py::arg("v"), py::arg("lo"),
        py::arg("hi"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"),
        py::arg("step"), py::arg("max_norm"), py::arg("extra_sq") = py::none(), py::arg("norm_out") = py::none(),
        py::arg("pads_epoch") = -1);
  m.def("comm_reduce_scatter_bucket", checked("comm_reduce_scatter_bucket", &tt::comm::comm_reduce_scatter_bucket),
        "one bucket of a reduce-scatter overlapped with the backward (sums of squares kept local)");
  m.def("comm_publish_sumsq", checked("comm_publish_sumsq", &tt::comm::comm_publish_sumsq),
        "publish the per-bucket sums of squares to every peer's pad; returns the epoch to wait for");
  m.def("comm_shadow_refresh", checked("comm_shadow_refresh", &tt::comm::comm_shadow_refresh), "wait for the all-gather; refresh bf16 shadow");
  m.def("comm_all_to_all", checked("comm_all_to_all", &tt::comm::comm_all_to_all), "equal-split all-to-all of a heap slot by peer loads");
  m.def("comm_epoch", &tt::comm::comm_epoch);
  m.def("comm_destroy", &tt::comm::comm_destroy);
}
