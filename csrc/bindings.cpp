// Python bindings of the revpp CUDA extension (module revpp._C).
#include <torch/extension.h>

#include <vector>

#include "host.h"

namespace revpp {
// gemm.cu
void gemm_tc(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int64_t M, int64_t N, int64_t K,
             int64_t epi, torch::Tensor C, const c10::optional<torch::Tensor>& bias,
             const c10::optional<torch::Tensor>& aux, const c10::optional<torch::Tensor>& aux_out,
             const c10::optional<torch::Tensor>& resid, double sign, int64_t splits, int64_t variant,
             const c10::optional<torch::Tensor>& colsum);
int64_t gemm_suggest_splits(int64_t M, int64_t N, int64_t K, int64_t sms);
// norm.cu
void layernorm_fwd(const torch::Tensor& x, const torch::Tensor& gamma, const torch::Tensor& beta, double eps,
                   const c10::optional<torch::Tensor>& y_bf16, const c10::optional<torch::Tensor>& y_f32,
                   const c10::optional<torch::Tensor>& y2_f32, const c10::optional<torch::Tensor>& mean,
                   const c10::optional<torch::Tensor>& rstd);
void layernorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& gamma,
                   const torch::Tensor& mean, const torch::Tensor& rstd, const c10::optional<torch::Tensor>& dgamma,
                   const c10::optional<torch::Tensor>& dbeta, const c10::optional<torch::Tensor>& resid,
                   const c10::optional<torch::Tensor>& dx_f32, const c10::optional<torch::Tensor>& dx_bf16,
                   const c10::optional<torch::Tensor>& colsum);
void cast_colsum(const torch::Tensor& in, const c10::optional<torch::Tensor>& out,
                 const c10::optional<torch::Tensor>& colsum);
// attention.cu
void attn_fwd(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S, int64_t heads);
void attn_bwd(const torch::Tensor& qkv, const torch::Tensor& out, const torch::Tensor& dout, const torch::Tensor& lse,
              torch::Tensor dqkv, torch::Tensor dq_acc, torch::Tensor Dbuf, int64_t B, int64_t S, int64_t heads);
// optim.cu
void grad_sumsq(const torch::Tensor& g, torch::Tensor out);
void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v,
                const c10::optional<torch::Tensor>& shadow, double lr, double beta1, double beta2, double eps,
                double wd, int64_t step, double max_norm, const c10::optional<torch::Tensor>& sumsq,
                bool zero_grad);
void scale_(torch::Tensor x, double s);
// attention_tc.cu
void attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S,
                 int64_t heads, const c10::optional<torch::Tensor>& phase_ns);
void attn_fwd_persistent(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S,
                         int64_t heads);
// comm.cu
void dp_reduce_adamw(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs,
                     const std::vector<int64_t>& shadow_ptrs, const std::vector<int64_t>& flag_ptrs, torch::Tensor m,
                     torch::Tensor v, torch::Tensor scratch, int64_t n, int64_t rank, int64_t epoch, double lr,
                     double beta1, double beta2, double eps, double wd, int64_t step, double max_norm,
                     double timeout_s, bool zero_grad);
void flag_wait_probe(torch::Tensor flag, int64_t expect, double timeout_s, torch::Tensor result);
std::vector<int64_t> pointer_info(int64_t ptr);
int64_t ipc_open(const std::string& handle_bytes);
void ipc_close(int64_t base);
void copy_to_ptr(int64_t dst, const torch::Tensor& src);
std::vector<std::string> ipc_export(const torch::Tensor& t);
void attn_bwd_tc(const torch::Tensor& qkv, const torch::Tensor& out, const torch::Tensor& dout,
                 const torch::Tensor& lse, torch::Tensor dqkv, torch::Tensor dq_acc, torch::Tensor Dbuf, int64_t B,
                 int64_t S, int64_t heads, const c10::optional<torch::Tensor>& colsum,
                 const c10::optional<torch::Tensor>& phase_ns);
// embed_head.cu
void bert_embed_fwd(const torch::Tensor& ids, const torch::Tensor& tt, const torch::Tensor& word,
                    const torch::Tensor& pos, const torch::Tensor& type, const torch::Tensor& gamma,
                    const torch::Tensor& beta, double eps, torch::Tensor out);
void bert_embed_bwd(const torch::Tensor& ids, const torch::Tensor& tt, const torch::Tensor& word,
                    const torch::Tensor& pos, const torch::Tensor& type, const torch::Tensor& gamma, double eps,
                    const torch::Tensor& dx2, const c10::optional<torch::Tensor>& dx1, torch::Tensor dword,
                    torch::Tensor dpos, torch::Tensor dtype, torch::Tensor dgamma, torch::Tensor dbeta);
void im2col_patches(const torch::Tensor& img, int64_t patch, torch::Tensor out);
void vit_assemble_fwd(const torch::Tensor& conv, const torch::Tensor& cls, const torch::Tensor& pos,
                      const torch::Tensor& gamma, const torch::Tensor& beta, double eps, int64_t B, int64_t S,
                      torch::Tensor out);
void vit_assemble_bwd(const torch::Tensor& conv, const torch::Tensor& cls, const torch::Tensor& pos,
                      const torch::Tensor& gamma, double eps, int64_t B, int64_t S, const torch::Tensor& dx2,
                      const c10::optional<torch::Tensor>& dx1, torch::Tensor dconv, torch::Tensor dcls,
                      torch::Tensor dpos, torch::Tensor dgamma, torch::Tensor dbeta);
void head_fwd_bwd(const torch::Tensor& y2, const c10::optional<torch::Tensor>& y1, int64_t mode,
                  const torch::Tensor& gamma, const torch::Tensor& beta, double eps, const torch::Tensor& wb,
                  const torch::Tensor& bb, const c10::optional<torch::Tensor>& labels, double grad_scale,
                  torch::Tensor pooled, torch::Tensor logits, torch::Tensor loss, bool want_grad,
                  const c10::optional<torch::Tensor>& dlogits, const c10::optional<torch::Tensor>& hb,
                  const c10::optional<torch::Tensor>& dpooled, const c10::optional<torch::Tensor>& dW,
                  const c10::optional<torch::Tensor>& db, const c10::optional<torch::Tensor>& dgamma,
                  const c10::optional<torch::Tensor>& dbeta, const c10::optional<torch::Tensor>& dy2,
                  const c10::optional<torch::Tensor>& dy1);
// host.cpp
void set_sm_reserve(int n);
int sm_reserve();
}  // namespace revpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "revpp sm_100a kernels";
  m.def("status_peek", &revpp::status_peek, "Read the device error word of the current device");
  m.def("status_read_and_clear", &revpp::status_read_and_clear, "Read and clear the device error word");
  m.def("num_sms", &revpp::num_sms);
  m.def("launch_count", &revpp::launch_count, "kernels launched by this process through the extension");
  m.def("set_sm_reserve", &revpp::set_sm_reserve, "SMs left free of persistent GEMM CTAs");
  m.def("sm_reserve", &revpp::sm_reserve);
  m.def("grad_sumsq", &revpp::grad_sumsq, py::arg("g"), py::arg("out"));
  m.def("adamw_step", &revpp::adamw_step, py::arg("p"), py::arg("g"), py::arg("m"), py::arg("v"),
        py::arg("shadow") = py::none(), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"),
        py::arg("wd"), py::arg("step"), py::arg("max_norm"), py::arg("sumsq") = py::none(),
        py::arg("zero_grad") = true);
  m.def("scale_", &revpp::scale_, py::arg("x"), py::arg("s"));

  m.def("gemm_tc", &revpp::gemm_tc, "tcgen05 GEMM with fused epilogue", py::arg("A"), py::arg("a_mn"), py::arg("B"),
        py::arg("b_mn"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"), py::arg("C"),
        py::arg("bias") = py::none(), py::arg("aux") = py::none(), py::arg("aux_out") = py::none(),
        py::arg("resid") = py::none(), py::arg("sign") = 1.0, py::arg("splits") = 1, py::arg("variant") = 0,
        py::arg("colsum") = py::none());
  m.def("gemm_suggest_splits", &revpp::gemm_suggest_splits, py::arg("M"), py::arg("N"), py::arg("K"),
        py::arg("sms") = -1, "split-K count for the weight-gradient GEMM (sms <= 0: this device's SM count)");

  m.def("layernorm_fwd", &revpp::layernorm_fwd, py::arg("x"), py::arg("gamma"), py::arg("beta"), py::arg("eps"),
        py::arg("y_bf16") = py::none(), py::arg("y_f32") = py::none(), py::arg("y2_f32") = py::none(),
        py::arg("mean") = py::none(), py::arg("rstd") = py::none());
  m.def("layernorm_bwd", &revpp::layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("gamma"), py::arg("mean"),
        py::arg("rstd"), py::arg("dgamma") = py::none(), py::arg("dbeta") = py::none(), py::arg("resid") = py::none(),
        py::arg("dx_f32") = py::none(), py::arg("dx_bf16") = py::none(), py::arg("colsum") = py::none());
  m.def("attn_fwd", &revpp::attn_fwd, py::arg("qkv"), py::arg("out"), py::arg("lse"), py::arg("B"), py::arg("S"),
        py::arg("heads"));
  m.def("attn_fwd_persistent", &revpp::attn_fwd_persistent, "persistent tcgen05 flash attention forward",
        py::arg("qkv"), py::arg("out"), py::arg("lse"), py::arg("B"), py::arg("S"), py::arg("heads"));
  m.def("attn_fwd_tc", &revpp::attn_fwd_tc, py::arg("qkv"), py::arg("out"), py::arg("lse"), py::arg("B"),
        py::arg("S"), py::arg("heads"), py::arg("phase_ns") = py::none());
  m.def("attn_bwd_tc", &revpp::attn_bwd_tc, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"),
        py::arg("dqkv"), py::arg("dq_acc"), py::arg("D"), py::arg("B"), py::arg("S"), py::arg("heads"),
        py::arg("colsum") = py::none(), py::arg("phase_ns") = py::none());
  m.def("attn_bwd", &revpp::attn_bwd, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"), py::arg("dqkv"),
        py::arg("dq_acc"), py::arg("D"), py::arg("B"), py::arg("S"), py::arg("heads"));
  m.def("bert_embed_fwd", &revpp::bert_embed_fwd);
  m.def("bert_embed_bwd", &revpp::bert_embed_bwd, py::arg("ids"), py::arg("tt"), py::arg("word"), py::arg("pos"),
        py::arg("type"), py::arg("gamma"), py::arg("eps"), py::arg("dx2"), py::arg("dx1"), py::arg("dword"),
        py::arg("dpos"), py::arg("dtype"), py::arg("dgamma"), py::arg("dbeta"));
  m.def("im2col_patches", &revpp::im2col_patches);
  m.def("vit_assemble_fwd", &revpp::vit_assemble_fwd);
  m.def("vit_assemble_bwd", &revpp::vit_assemble_bwd, py::arg("conv"), py::arg("cls"), py::arg("pos"),
        py::arg("gamma"), py::arg("eps"), py::arg("B"), py::arg("S"), py::arg("dx2"), py::arg("dx1"),
        py::arg("dconv"), py::arg("dcls"), py::arg("dpos"), py::arg("dgamma"), py::arg("dbeta"));
  m.def("head_fwd_bwd", &revpp::head_fwd_bwd, py::arg("y2"), py::arg("y1"), py::arg("mode"), py::arg("gamma"),
        py::arg("beta"), py::arg("eps"), py::arg("wb"), py::arg("bb"), py::arg("labels"), py::arg("grad_scale"),
        py::arg("pooled"), py::arg("logits"), py::arg("loss"), py::arg("want_grad"), py::arg("dlogits") = py::none(),
        py::arg("hb") = py::none(), py::arg("dpooled") = py::none(), py::arg("dW") = py::none(),
        py::arg("db") = py::none(), py::arg("dgamma") = py::none(), py::arg("dbeta") = py::none(),
        py::arg("dy2") = py::none(), py::arg("dy1") = py::none());
  m.def("dp_reduce_adamw", &revpp::dp_reduce_adamw);
  m.def("pointer_info", &revpp::pointer_info);
  m.def("ipc_open", [](py::bytes h) { return revpp::ipc_open(std::string(h)); });
  m.def("ipc_close", &revpp::ipc_close);
  m.def("copy_to_ptr", &revpp::copy_to_ptr, "cudaMemcpyAsync of a contiguous tensor to a device address (a peer's IPC-mapped slot) on the current stream", py::arg("dst"), py::arg("src"));
  m.def("ipc_export", [](const torch::Tensor& t) {
    auto v = revpp::ipc_export(t);
    return py::make_tuple(py::bytes(v[0]), std::stoll(v[1]));
  });
  m.def("flag_wait_probe", &revpp::flag_wait_probe, py::arg("flag"), py::arg("expect"), py::arg("timeout_s"),
        py::arg("result"));
  m.def("cast_colsum", &revpp::cast_colsum, py::arg("inp"), py::arg("out") = py::none(),
        py::arg("colsum") = py::none());
}
