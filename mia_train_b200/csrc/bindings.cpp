// Python bindings of the mia_train_b200._C extension (all kernels are sm_100a).
#include <torch/extension.h>

#include "errors.h"

namespace mia {
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor d, c10::optional<torch::Tensor> bias,
          c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> gamma,
          c10::optional<torch::Tensor> aux_out, bool a_kmajor, bool b_kmajor, int64_t act, bool accumulate,
          c10::optional<torch::Tensor> colsum, double colsum_scale, c10::optional<torch::Tensor> a2,
          c10::optional<torch::Tensor> b2);
void column_sum(torch::Tensor x, torch::Tensor out, bool accumulate);
int64_t set_gemm_pair_mode(int64_t mode);
void zscore_u8(torch::Tensor x, torch::Tensor out);
void sinkhorn_colsum(torch::Tensor x, double temperature, c10::optional<torch::Tensor> s, torch::Tensor out);
void sinkhorn_rowsum(torch::Tensor x, double temperature, torch::Tensor r, torch::Tensor out);
void sinkhorn_scale(torch::Tensor x, double temperature, torch::Tensor r, torch::Tensor s, double factor,
                    torch::Tensor out);
void set_tc_attention_mode(int64_t mode);
int64_t tc_attention_mode();
int64_t tc_attention_launches();
void layernorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> w, c10::optional<torch::Tensor> b, torch::Tensor y,
                   torch::Tensor mean, torch::Tensor rstd, double eps, bool rms);
void layernorm_bwd(torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> w, torch::Tensor mean,
                   torch::Tensor rstd, torch::Tensor dx, c10::optional<torch::Tensor> dw,
                   c10::optional<torch::Tensor> db, bool rms, c10::optional<torch::Tensor> dres);
void attention_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse, double scale);
void attention_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                   torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, double scale);
void rope_qk_fwd(torch::Tensor qkv, torch::Tensor angles, torch::Tensor pairs, torch::Tensor qk);
void attention_fwd_strided(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse,
                           double scale);
void rope_attention_bwd_packed(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                               torch::Tensor lse, c10::optional<torch::Tensor> angles, torch::Tensor pairs,
                               torch::Tensor dqkv, c10::optional<torch::Tensor> dangles, double scale);
void multi_tensor_sumsq(std::vector<at::Tensor> tensors, at::Tensor out);
void multi_tensor_scale(std::vector<at::Tensor> tensors, at::Tensor coef);
void ema_update(std::vector<at::Tensor> teacher, std::vector<at::Tensor> student, double momentum);
void adamw_step(std::vector<at::Tensor> params, std::vector<at::Tensor> grads, std::vector<at::Tensor> exp_avgs,
                std::vector<at::Tensor> exp_avg_sqs, std::vector<at::Tensor> steps, at::Tensor group_index,
                at::Tensor hyper, double eps, c10::optional<at::Tensor> grad_scale, std::vector<at::Tensor> shadows);
void patch_gather(torch::Tensor vol, torch::Tensor index, torch::Tensor out, int64_t pd, int64_t ph, int64_t pw);
void mae_restore_fwd(torch::Tensor visible, torch::Tensor token, torch::Tensor restore, torch::Tensor out);
void mae_restore_bwd(torch::Tensor dout, torch::Tensor restore, torch::Tensor dvis, torch::Tensor dtok);
void norm_pix_mse(torch::Tensor pred, torch::Tensor vol, torch::Tensor mask, torch::Tensor loss, torch::Tensor grad,
                  int64_t pd, int64_t ph, int64_t pw, bool norm_pix);
at::Tensor affinity_bce_fwd(at::Tensor logits, at::Tensor labels, std::vector<int64_t> offsets, int64_t ignore_index);
at::Tensor affinity_bce_bwd(at::Tensor logits, at::Tensor labels, std::vector<int64_t> offsets, int64_t ignore_index,
                            at::Tensor sums, at::Tensor grad_out);
std::vector<at::Tensor> semantic_ce_fwd(at::Tensor logits, at::Tensor labels, c10::optional<at::Tensor> weights,
                                        int64_t ignore_index);
at::Tensor semantic_ce_bwd(at::Tensor logits, at::Tensor labels, c10::optional<at::Tensor> weights, int64_t ignore_index,
                           at::Tensor stats, at::Tensor grad_out);
at::Tensor connected_components_cpu(at::Tensor labels);
std::vector<at::Tensor> ipc_export(int64_t nbytes, int64_t device);
std::vector<int64_t> ipc_open(at::Tensor handles, int64_t rank, int64_t local_ptr, int64_t device);
void ipc_close(std::vector<int64_t> peers, int64_t rank, int64_t device);
void ipc_free(int64_t local_ptr, int64_t device);
int64_t comm_flag_bytes();
int64_t comm_max_blocks();
void zero_reduce_scatter(std::vector<int64_t> grad_peers, std::vector<int64_t> flag_peers, int64_t shard_off,
                         int64_t shard_len, at::Tensor partial, at::Tensor epoch, int64_t rank, double timeout_ms,
                         int64_t seq, int64_t threads);
void zero_norm_exchange(std::vector<int64_t> flag_peers, at::Tensor partial, at::Tensor epoch, int64_t rank,
                        double max_norm, at::Tensor grad_scale, at::Tensor grad_norm, double timeout_ms);
void zero_all_gather(std::vector<int64_t> data_peers, std::vector<int64_t> shadow_peers, std::vector<int64_t> flag_peers,
                     int64_t seg_lo, int64_t shard_len, int64_t bf16_begin, at::Tensor epoch, int64_t rank, int64_t blocks,
                     double timeout_ms, int64_t seq);
void zero_advance_epoch(at::Tensor epoch);
void zero_reduce_scatter_bf16(std::vector<int64_t> grad_peers, std::vector<int64_t> grad16_peers,
                              std::vector<int64_t> flag_peers, int64_t seg_lo, int64_t shard_len, at::Tensor partial,
                              at::Tensor epoch, int64_t rank, double timeout_ms, int64_t seq, int64_t threads);
void tp_ag_gemm(at::Tensor a_local, at::Tensor b, at::Tensor out, at::Tensor a_full, c10::optional<at::Tensor> bias,
                c10::optional<at::Tensor> aux, c10::optional<at::Tensor> aux_out, bool b_kmajor, int64_t act,
                std::vector<int64_t> flag_peers, std::vector<int64_t> send_peers, int64_t send_parity_bytes,
                int64_t rank, double timeout_ms);
void tp_gemm_rs(at::Tensor a, at::Tensor b, at::Tensor out, c10::optional<at::Tensor> bias,
                c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> residual,
                c10::optional<at::Tensor> pre_out, bool b_kmajor, std::vector<int64_t> flag_peers,
                std::vector<int64_t> recv_peers, int64_t recv_parity_bytes, int64_t rank, double timeout_ms,
                at::Tensor ident);
int64_t tp_flag_bytes();
at::Tensor tp_trace_read(int64_t device);
void soft_ce_fwd(at::Tensor S, at::Tensor T, at::Tensor tidx, at::Tensor w, double tau, at::Tensor lse, at::Tensor loss);
void soft_ce_bwd(at::Tensor S, at::Tensor T, at::Tensor tidx, at::Tensor w, double tau, at::Tensor lse,
                 at::Tensor grad_scale, at::Tensor dS);
int64_t set_attention_poly_exp(int64_t mode);
void masked_l1(torch::Tensor pred, torch::Tensor vol, torch::Tensor mask, torch::Tensor sums, torch::Tensor grad,
               int64_t pd, int64_t ph, int64_t pw, bool norm_pix);
void koleo_fwd(at::Tensor x, double eps, at::Tensor xn, at::Tensor nn, at::Tensor dist, at::Tensor loss);
void koleo_bwd(at::Tensor x, at::Tensor xn, at::Tensor nn, at::Tensor dist, double eps, at::Tensor grad,
               at::Tensor dxn, at::Tensor dx);
at::Tensor axial_angles_fwd(at::Tensor coords, std::vector<at::Tensor> freqs);
void axial_angles_bwd(at::Tensor dangles, at::Tensor coords, std::vector<at::Tensor> freqs,
                      std::vector<at::Tensor> dfreqs);
}  // namespace mia

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mia_train_b200 sm_100a kernels";
  m.def("gemm", &mia::gemm, "tcgen05 bf16 GEMM with fused epilogue", py::arg("a"), py::arg("b"), py::arg("d"),
        py::arg("bias"), py::arg("residual"), py::arg("aux"), py::arg("gamma"), py::arg("aux_out"), py::arg("a_kmajor"),
        py::arg("b_kmajor"), py::arg("act"), py::arg("accumulate"), py::arg("colsum") = py::none(),
        py::arg("colsum_scale") = 1.0, py::arg("a2") = py::none(), py::arg("b2") = py::none());
  m.def("column_sum", &mia::column_sum);
  m.def("layernorm_fwd", &mia::layernorm_fwd);
  m.def("layernorm_bwd", &mia::layernorm_bwd, "LayerNorm / RMSNorm backward; dres (optional) is added to dX",
        py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("mean"), py::arg("rstd"), py::arg("dx"), py::arg("dw"),
        py::arg("db"), py::arg("rms"), py::arg("dres") = py::none());
  m.def("attention_fwd", &mia::attention_fwd);
  m.def("attention_bwd", &mia::attention_bwd);
  m.def("rope_qk_fwd", &mia::rope_qk_fwd, "rotate q and k of a packed (B, N, 3, H, D) projection into (B, N, 2, H, D)");
  m.def("attention_fwd_strided", &mia::attention_fwd_strided, "attention on strided (B, N, H, D) views");
  m.def("rope_attention_bwd_packed", &mia::rope_attention_bwd_packed, "attention (+RoPE) backward into the packed gradient");
  m.def("multi_tensor_sumsq", &mia::multi_tensor_sumsq);
  m.def("multi_tensor_scale", &mia::multi_tensor_scale);
  m.def("ema_update", &mia::ema_update, "teacher = m * teacher + (1 - m) * student over tensor lists");
  m.def("adamw_step", &mia::adamw_step);
  m.def("patch_gather", &mia::patch_gather);
  m.def("mae_restore_fwd", &mia::mae_restore_fwd);
  m.def("mae_restore_bwd", &mia::mae_restore_bwd);
  m.def("norm_pix_mse", &mia::norm_pix_mse);
  m.def("affinity_bce_fwd", &mia::affinity_bce_fwd, "fused affinity targets + masked BCE statistics");
  m.def("affinity_bce_bwd", &mia::affinity_bce_bwd, "gradient of the fused affinity BCE");
  m.def("semantic_ce_fwd", &mia::semantic_ce_fwd, "fused softmax CE + confusion histogram");
  m.def("semantic_ce_bwd", &mia::semantic_ce_bwd, "gradient of the fused softmax CE");
  m.def("connected_components_cpu", &mia::connected_components_cpu, "connected components of equal positive labels (host)");
  m.def("ipc_export", &mia::ipc_export, "cudaMalloc + IPC handle: (local uint8 tensor, handle bytes, address)");
  m.def("ipc_open", &mia::ipc_open, "open every peer's IPC handle -> device pointers (own pointer at own rank)");
  m.def("ipc_close", &mia::ipc_close);
  m.def("ipc_free", &mia::ipc_free);
  m.def("comm_flag_bytes", &mia::comm_flag_bytes);
  m.def("comm_max_blocks", &mia::comm_max_blocks);
  m.def("zero_reduce_scatter", &mia::zero_reduce_scatter, "peer-memory gradient reduce-scatter + sum of squares");
  m.def("zero_norm_exchange", &mia::zero_norm_exchange, "cross-rank grad norm -> clip scale");
  m.def("zero_all_gather", &mia::zero_all_gather, "peer-memory parameter all-gather + local refresh");
  m.def("zero_advance_epoch", &mia::zero_advance_epoch);
  m.def("zero_reduce_scatter_bf16", &mia::zero_reduce_scatter_bf16,
        "peer-memory gradient reduce-scatter with bf16 on the wire (fp32 sum) + sum of squares");
  m.def("tp_ag_gemm", &mia::tp_ag_gemm, "fused all-gather (peer pushes) -> tcgen05 GEMM, sequence-parallel input");
  m.def("tp_gemm_rs", &mia::tp_gemm_rs, "fused tcgen05 GEMM -> reduce-scatter (peer stores) + bias/LayerScale/residual");
  m.def("tp_flag_bytes", &mia::tp_flag_bytes, "bytes of one rank's flag area for the fused TP kernels");
  m.def("tp_trace_read", &mia::tp_trace_read, "per-CTA timelines of the last fused TP launches (MIA_TP_TRACE=1)");
  m.def("soft_ce_fwd", &mia::soft_ce_fwd, "soft-target cross-entropy over prototypes (DINO / iBOT): lse + per-row loss");
  m.def("soft_ce_bwd", &mia::soft_ce_bwd, "gradient of soft_ce_fwd with respect to the student logits");
  m.def("set_attention_poly_exp", &mia::set_attention_poly_exp,
        "1: a quarter of the attention softmax exponentials on the FMA pipe; 0: all on MUFU; returns the previous");
  m.def("masked_l1", &mia::masked_l1, "SimMIM masked L1 (targets read from the volume) + gradient");
  m.def("koleo_fwd", &mia::koleo_fwd, "KoLeo: normalise, nearest neighbour, -mean log distance");
  m.def("koleo_bwd", &mia::koleo_bwd, "gradient of koleo_fwd");
  m.def("set_tc_attention_mode", &mia::set_tc_attention_mode, "1: tcgen05 attention where it applies (head dim 32 / 64); 0: warp-level kernels");
  m.def("tc_attention_mode", &mia::tc_attention_mode);
  m.def("tc_attention_launches", &mia::tc_attention_launches);
  m.def("sinkhorn_colsum", &mia::sinkhorn_colsum, "sum_b exp(x/T) s_b per prototype");
  m.def("sinkhorn_rowsum", &mia::sinkhorn_rowsum, "sum_k exp(x/T) r_k per sample");
  m.def("sinkhorn_scale", &mia::sinkhorn_scale, "exp(x/T) r_k s_b factor");
  m.def("zscore_u8", &mia::zscore_u8, "per-volume z-score of a uint8 batch into bf16 / fp32 (exact integer moments)");
  m.def("set_gemm_pair_mode", &mia::set_gemm_pair_mode, "0: single-CTA GEMM tiles; else CTA pairs when M >= 256; returns the previous mode");
  m.def("axial_angles_fwd", &mia::axial_angles_fwd, "angles[r, p] = coords[r, axis(p)] * freq(p)");
  m.def("axial_angles_bwd", &mia::axial_angles_bwd, "accumulate the frequency gradients of axial_angles_fwd");
  m.def("check_errors", &mia::read_and_clear_errors, "read and clear the device error word");
}
