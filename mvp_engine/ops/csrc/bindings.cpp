// Python bindings of the sm_100a kernels (module mvp_engine._C).
#include <torch/extension.h>

void gemm_sm100(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                bool accumulate, int64_t status_ptr);

std::vector<torch::Tensor> rmsnorm_fwd(const torch::Tensor& x, const c10::optional<torch::Tensor>& res,
                                       const torch::Tensor& w, double eps);
std::vector<torch::Tensor> rmsnorm_bwd(const torch::Tensor& dy, const torch::Tensor& h, const torch::Tensor& rstd,
                                       const torch::Tensor& w, const c10::optional<torch::Tensor>& dres, bool need_dw,
                                       const c10::optional<torch::Tensor>& dw_acc);
std::vector<torch::Tensor> qk_norm_rope_fwd(const torch::Tensor& qkv, int64_t Hq, int64_t Hkv,
                                            const torch::Tensor& wq, const torch::Tensor& wk,
                                            const torch::Tensor& pos, const torch::Tensor& axis_of,
                                            const torch::Tensor& cos_tab, const torch::Tensor& sin_tab, double eps);
std::vector<torch::Tensor> qk_norm_rope_bwd(const torch::Tensor& dq, const torch::Tensor& dk,
                                            const torch::Tensor& qkv, torch::Tensor& dqkv, int64_t Hq, int64_t Hkv,
                                            const torch::Tensor& wq, const torch::Tensor& wk,
                                            const torch::Tensor& pos, const torch::Tensor& axis_of,
                                            const torch::Tensor& cos_tab, const torch::Tensor& sin_tab,
                                            const torch::Tensor& rstd,
                                            const c10::optional<std::vector<int64_t>>& route,
                                            const c10::optional<torch::Tensor>& dwq_acc,
                                            const c10::optional<torch::Tensor>& dwk_acc);
torch::Tensor swiglu_fwd(const torch::Tensor& gu);
torch::Tensor swiglu_bwd(const torch::Tensor& gu, const torch::Tensor& dout);

std::vector<torch::Tensor> ce_fwd(const torch::Tensor& logits, const torch::Tensor& labels);
void ce_bwd_(torch::Tensor& logits, const torch::Tensor& labels, const torch::Tensor& lse, const torch::Tensor& g);
void adamw_step_(torch::Tensor& p, const torch::Tensor& g, torch::Tensor& m, torch::Tensor& v,
                 const c10::optional<torch::Tensor>& p_bf16, double lr, double beta1, double beta2, double eps,
                 double wd, int64_t step, double grad_scale, const c10::optional<torch::Tensor>& norm_sq,
                 double max_norm);
torch::Tensor sumsq(const torch::Tensor& x);
torch::Tensor embedding_fwd(const torch::Tensor& w, const torch::Tensor& ids, int64_t status_ptr);
void embedding_bwd_(torch::Tensor& dw, const torch::Tensor& dout, const torch::Tensor& ids);

std::vector<torch::Tensor> flash_attn_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                                          const torch::Tensor& cu_seqlens, double softmax_scale, bool causal,
                                          int64_t status_ptr, const c10::optional<torch::Tensor>& cu_seqlens_k,
                                          const c10::optional<std::vector<int64_t>>& pull,
                                          const c10::optional<std::vector<int64_t>>& route);

std::vector<torch::Tensor> flash_attn_bwd(const torch::Tensor& dout, const torch::Tensor& q, const torch::Tensor& k,
                                          const torch::Tensor& v, const torch::Tensor& out, const torch::Tensor& lse,
                                          const torch::Tensor& cu_seqlens, double softmax_scale, bool causal,
                                          int64_t status_ptr, const c10::optional<torch::Tensor>& dk_out,
                                          const c10::optional<torch::Tensor>& dv_out,
                                          const c10::optional<torch::Tensor>& cu_seqlens_k,
                                          const c10::optional<std::vector<int64_t>>& pull,
                                          const c10::optional<torch::Tensor>& dq_accum,
                                          const c10::optional<std::vector<int64_t>>& dkv_f32,
                                          const c10::optional<std::vector<int64_t>>& route);

void peer_reduce_scatter(const std::vector<int64_t>& peer_bufs, const std::vector<int64_t>& peer_slots,
                         int64_t my_slots, int64_t rank, int64_t offset, int64_t shard, int64_t seq, double scale,
                         torch::Tensor& out, const c10::optional<torch::Tensor>& sumsq, int64_t status_ptr,
                         int64_t timeout_ns);
void peer_barrier(const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                  int64_t status_ptr, int64_t timeout_ns);

void peer_push_rows(const torch::Tensor& src, const std::vector<int64_t>& dsts, int64_t dst_row0,
                    const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                    int64_t status_ptr, int64_t timeout_ns);
void peer_wait_all(const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                   int64_t status_ptr, int64_t timeout_ns);
void peer_slot_reduce(const torch::Tensor& slots, torch::Tensor& out, const std::vector<int64_t>& peer_slots,
                      int64_t my_slots, int64_t rank, int64_t seq, int64_t status_ptr, int64_t timeout_ns);
void peer_publish(const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                  int64_t status_ptr, int64_t timeout_ns);
void peer_gather_shards(const std::vector<int64_t>& peer_bufs, const std::vector<int64_t>& peer_flags,
                        int64_t offset, int64_t shard, int64_t epoch, torch::Tensor& out, int64_t status_ptr,
                        int64_t timeout_ns);
void publish_epoch(int64_t flag_ptr, int64_t epoch);
void gemm_pair_gather(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                      bool accumulate, int64_t status_ptr, const std::vector<int64_t>& peer_bufs,
                      const std::vector<int64_t>& peer_flags, int64_t offset, int64_t shard, int64_t epoch,
                      torch::Tensor& slot, int64_t copy_ctas, int64_t timeout_ns);
void peer_slot_sum_f32(const torch::Tensor& slots, torch::Tensor& out, const std::vector<int64_t>& peer_slots,
                       int64_t my_slots, int64_t rank, int64_t seq, int64_t status_ptr, int64_t timeout_ns);
void gemm_ulysses(const torch::Tensor& a, const torch::Tensor& b, bool b_mn, const std::vector<int64_t>& dst,
                  int64_t ld, int64_t rank, int64_t chunk, int64_t head_dim, const std::vector<int64_t>& secs,
                  int64_t status_ptr);
void gemm_pair_tp(const torch::Tensor& a, const torch::Tensor& b, bool b_mn, const c10::optional<torch::Tensor>& c,
                  int64_t ldc, int64_t a_slots, int64_t a_seq, int64_t a_rows, int64_t a_first_row,
                  const std::vector<int64_t>& dst, int64_t dst_rows, int64_t dst_row0, int64_t status_ptr,
                  int64_t wait_ns);

std::vector<torch::Tensor> layernorm_fwd(const torch::Tensor& x, const torch::Tensor& w, const torch::Tensor& b,
                                         double eps);
std::vector<torch::Tensor> layernorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& mean,
                                         const torch::Tensor& rstd, const torch::Tensor& w,
                                         const c10::optional<torch::Tensor>& dw_acc,
                                         const c10::optional<torch::Tensor>& db_acc);
torch::Tensor bias_gelu_fwd(const torch::Tensor& x, const torch::Tensor& b, bool tanh_form);
std::vector<torch::Tensor> bias_gelu_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& b,
                                         bool tanh_form, const c10::optional<torch::Tensor>& db_acc);
std::vector<torch::Tensor> vision_rope_fwd(const torch::Tensor& qkv, int64_t nh, const torch::Tensor& cosv,
                                           const torch::Tensor& sinv, int64_t DP,
                                           const c10::optional<torch::Tensor>& bias);
torch::Tensor bias_residual_fwd(const torch::Tensor& y, const torch::Tensor& b, const torch::Tensor& x);
torch::Tensor bias_grad(const torch::Tensor& g, const c10::optional<torch::Tensor>& acc);
torch::Tensor vision_rope_bwd(const torch::Tensor& dq, const torch::Tensor& dk, const torch::Tensor& dv,
                              const torch::Tensor& cosv, const torch::Tensor& sinv, int64_t D);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mvp_engine sm_100a kernels";
  m.def("gemm", &gemm_sm100, "tcgen05 bf16 GEMM C (+)= A * B^T with K- or MN-major operands");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd, py::arg("dy"), py::arg("h"), py::arg("rstd"), py::arg("w"), py::arg("dres"),
        py::arg("need_dw"), py::arg("dw_acc") = py::none());
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd, py::arg("dq"), py::arg("dk"), py::arg("qkv"), py::arg("dqkv"),
        py::arg("Hq"), py::arg("Hkv"), py::arg("wq"), py::arg("wk"), py::arg("pos"), py::arg("axis_of"),
        py::arg("cos_tab"), py::arg("sin_tab"), py::arg("rstd"), py::arg("route") = py::none(),
        py::arg("dwq_acc") = py::none(), py::arg("dwk_acc") = py::none());
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("layernorm_fwd", &layernorm_fwd, "LayerNorm with bias (vision tower)");
  m.def("layernorm_bwd", &layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("mean"), py::arg("rstd"), py::arg("w"),
        py::arg("dw_acc") = py::none(), py::arg("db_acc") = py::none());
  m.def("bias_gelu_fwd", &bias_gelu_fwd, "y = gelu(x + b), tanh or erf form");
  m.def("bias_gelu_bwd", &bias_gelu_bwd, py::arg("dy"), py::arg("x"), py::arg("b"), py::arg("tanh_form"),
        py::arg("db_acc") = py::none());
  m.def("bias_residual_fwd", &bias_residual_fwd, "x + (y + b), each add rounded to bf16");
  m.def("bias_grad", &bias_grad, "fp32 column sums of a bf16 matrix", py::arg("g"), py::arg("acc") = py::none());
  m.def("vision_rope_fwd", &vision_rope_fwd, "rotate-half RoPE of q / k (+ optional qkv bias), padded to DP columns",
        py::arg("qkv"), py::arg("nh"), py::arg("cos"), py::arg("sin"), py::arg("DP"), py::arg("bias") = py::none());
  m.def("vision_rope_bwd", &vision_rope_bwd, "inverse rotation of dq / dk, written with dv into dqkv");
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd_", &ce_bwd_);
  m.def("adamw_step_", &adamw_step_);
  m.def("sumsq", &sumsq);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd_", &embedding_bwd_);
  m.def("flash_attn_fwd", &flash_attn_fwd, "varlen flash attention forward (tcgen05)", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("cu_seqlens"), py::arg("softmax_scale"), py::arg("causal"), py::arg("status_ptr"),
        py::arg("cu_seqlens_k") = py::none(), py::arg("pull") = py::none(), py::arg("route") = py::none());
  m.def("peer_reduce_scatter", &peer_reduce_scatter,
        "pull reduce-scatter of a symmetric fp32 buffer over NVLink peers (bounded waits)");
  m.def("peer_barrier", &peer_barrier, "device-side barrier over peer signal slots (bounded)");
  m.def("peer_push_rows", &peer_push_rows, "copy a row slice into every rank's gather buffer, then publish");
  m.def("peer_wait_all", &peer_wait_all, "wait (bounded) until every rank published a sequence number");
  m.def("peer_slot_reduce", &peer_slot_reduce, "sum routed partial slots after the publish / wait handshake");
  m.def("gemm_ulysses", &gemm_ulysses, "two-SM GEMM whose epilogue scatters heads to their context ranks");
  m.def("gemm_pair_tp", &gemm_pair_tp, "two-SM GEMM with per-slice A readiness and routed output rows");
  m.def("flash_attn_bwd", &flash_attn_bwd, "varlen flash attention backward (tcgen05)", py::arg("dout"),
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"), py::arg("lse"), py::arg("cu_seqlens"),
        py::arg("softmax_scale"), py::arg("causal"), py::arg("status_ptr"), py::arg("dk_out") = py::none(),
        py::arg("dv_out") = py::none(), py::arg("cu_seqlens_k") = py::none(), py::arg("pull") = py::none(),
        py::arg("dq_accum") = py::none(), py::arg("dkv_f32") = py::none(), py::arg("route") = py::none());
  m.def("peer_gather_shards", &peer_gather_shards, "FSDP parameter gather: pull every rank's bf16 shard (bounded epoch wait)");
  m.def("gemm_pair_gather", &gemm_pair_gather, "two-SM GEMM carrying an FSDP shard pull in extra CTAs");
  m.def("publish_epoch", &publish_epoch, "system-scope release of an epoch number into a flag");
  m.def("peer_publish", &peer_publish, "publish a sequence number into every rank's signal slot");
  m.def("peer_slot_sum_f32", &peer_slot_sum_f32,
        "publish, wait for every rank, then sum fp32 partial slots [W, n] into bf16 [n]");
}
