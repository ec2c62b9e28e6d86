// Python bindings of the packbalance_b200 native extension (module
// ``packbalance_b200._C``).  Every op runs on the current CUDA stream of the input
// tensors' device.
#include <torch/extension.h>

#include "host_utils.h"

namespace pb {
int64_t gemm_pair_mode(int64_t mode);
int64_t gemm_pair_test_arm_limit(int64_t n);
void gemm_tc(at::Tensor a, at::Tensor b, at::Tensor out, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
             int64_t epi, int64_t bn, int64_t splits, int64_t max_ctas, double alpha,
             c10::optional<at::Tensor> aux, c10::optional<at::Tensor> pos, c10::optional<at::Tensor> cos_t,
             c10::optional<at::Tensor> sin_t, int64_t head_dim, int64_t n_rope_cols,
             c10::optional<at::Tensor> targets, c10::optional<at::Tensor> pmax, c10::optional<at::Tensor> psum,
             c10::optional<at::Tensor> tlogit, c10::optional<at::Tensor> lse, c10::optional<at::Tensor> row_scale,
             double z_coeff, std::vector<int64_t> ag);
std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, c10::optional<at::Tensor> delta, at::Tensor w, double eps,
                                        bool out_bf16);
void swiglu_bwd_packed(at::Tensor dh, at::Tensor gu, at::Tensor dgu);
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps, bool out_bf16);
at::Tensor rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, c10::optional<at::Tensor> dres,
                       c10::optional<at::Tensor> dx_bf16, at::Tensor dw_out, bool accumulate_dw);
at::Tensor swiglu_fwd(at::Tensor g, at::Tensor u);
std::vector<at::Tensor> swiglu_bwd(at::Tensor g, at::Tensor u, at::Tensor dh);
void rope_apply(at::Tensor x, at::Tensor pos, at::Tensor cos_t, at::Tensor sin_t, int64_t n_rope_cols,
                int64_t head_dim, bool inverse);
at::Tensor embedding_fwd(at::Tensor ids, at::Tensor w);
void embedding_bwd(at::Tensor ids, at::Tensor dx, at::Tensor grad, bool accumulate);
bool set_deterministic(bool on);
void ce_finalize(at::Tensor pmax, at::Tensor psum, at::Tensor tlogit, at::Tensor targets, int64_t ignore_index,
                 double z, at::Tensor lse, at::Tensor loss);
void ce_row_scale(at::Tensor targets, int64_t ignore_index, at::Tensor grad_out, at::Tensor scale);
void ce_dlogits(at::Tensor logits, at::Tensor lse, at::Tensor targets, at::Tensor scale, double z);
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, at::Tensor shadow, at::Tensor norm,
                at::Tensor skipped, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                double max_norm, bool write_shadow, c10::optional<at::Tensor> hparams);
at::Tensor l2_norm(at::Tensor x);
std::vector<at::Tensor> attn_fwd(at::Tensor qkv, at::Tensor doc_start, at::Tensor tiles, int64_t n_heads,
                                 int64_t n_kv_heads, int64_t head_dim, double scale, at::Tensor out);
void attn_trace(int64_t ptr);
void attn_bwd(at::Tensor qkv, at::Tensor out, at::Tensor dout, at::Tensor lse, at::Tensor doc_start,
              at::Tensor doc_end, at::Tensor items, int64_t H, int64_t Hkv, int64_t D, double scale, at::Tensor dqkv,
              at::Tensor dq_acc, at::Tensor dkv_acc, at::Tensor delta, c10::optional<at::Tensor> pos,
              c10::optional<at::Tensor> cos_t, c10::optional<at::Tensor> sin_t);
void comm_bindings(pybind11::module& m);
void fsdp_bindings(pybind11::module& m);

int64_t status_read(int64_t dev, bool clear) {
  int v = 0;
  int* p = status_ptr(static_cast<int>(dev));
  PB_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear && v != 0) PB_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return v;
}
}  // namespace pb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "packbalance_b200 native sm_100a kernels";
  m.def("gemm_tc", &pb::gemm_tc);
  m.def("gemm_pair_mode", &pb::gemm_pair_mode, "set (0/1) or read (-1) the CTA-pair GEMM mode; returns the previous");
  m.def("gemm_pair_test_arm_limit", &pb::gemm_pair_test_arm_limit,
        "tests only: the even CTA of pair GEMMs stalls after arming n k-blocks (0 = off); returns the previous");
  m.def("rmsnorm_fwd", &pb::rmsnorm_fwd);
  m.def("add_rmsnorm_fwd", &pb::add_rmsnorm_fwd);
  m.def("swiglu_bwd_packed", &pb::swiglu_bwd_packed);
  m.def("rmsnorm_bwd", &pb::rmsnorm_bwd);
  m.def("swiglu_fwd", &pb::swiglu_fwd);
  m.def("swiglu_bwd", &pb::swiglu_bwd);
  m.def("rope_apply", &pb::rope_apply);
  m.def("embedding_fwd", &pb::embedding_fwd);
  m.def("embedding_bwd", &pb::embedding_bwd);
  m.def("set_deterministic", &pb::set_deterministic,
        "fixed-order reductions for RMSNorm dw and the embedding gradient; returns the previous setting");
  m.def("ce_finalize", &pb::ce_finalize);
  m.def("ce_row_scale", &pb::ce_row_scale);
  m.def("ce_dlogits", &pb::ce_dlogits, "in-place dlogits over kept bf16 logits");
  m.def("adamw_step", &pb::adamw_step);
  m.def("l2_norm", &pb::l2_norm);
  m.def("status_read", &pb::status_read, pybind11::arg("dev"), pybind11::arg("clear") = true);
  m.def("attn_fwd", &pb::attn_fwd);
  m.def("attn_bwd", &pb::attn_bwd);
  m.def("attn_trace", &pb::attn_trace);
  pb::comm_bindings(m);
  pb::fsdp_bindings(m);
}
