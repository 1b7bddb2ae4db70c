// Torch-facing bindings of the sm_100a kernels.  Only this file includes the
// torch headers; the kernels themselves are plain CUDA with raw-pointer
// launchers (launchers.h), which keeps them fast to compile and callable
// without the framework.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "launchers.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

int dt_code(const torch::Tensor& t) {
  if (t.scalar_type() == at::kBFloat16) return AHB_BF16;
  TORCH_CHECK(t.scalar_type() == at::kFloat, "expected bf16 or fp32 tensor, got ", t.scalar_type());
  return AHB_F32;
}

void check_cuda(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda(), n, " must be a CUDA tensor");
}

void check_acc(const torch::Tensor& t, int64_t n, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == n, name,
              " must be a contiguous fp32 CUDA tensor with ", n, " elements");
}

float* opt_ptr(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr<float>() : nullptr;
}

// ------------------------------------------------------------ elementwise
torch::Tensor sanitize(torch::Tensor x, double clip) {
  check_cuda(x, "x");
  auto xc = x.contiguous();
  auto out = torch::empty_like(xc);
  ahb_sanitize(out.data_ptr(), xc.data_ptr(), xc.numel(), dt_code(xc), (float)clip, cur_stream());
  return out;
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor scale, double eps) {
  check_cuda(x, "x");
  auto xc = x.contiguous();
  int D = (int)xc.size(-1);
  TORCH_CHECK(D <= 8192, "rmsnorm: D must be <= 8192");
  int64_t M = xc.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  auto y = torch::empty_like(xc);
  auto r = torch::empty({M}, xc.options().dtype(at::kFloat));
  ahb_rmsnorm_fwd(xc.data_ptr(), sc.data_ptr<float>(), y.data_ptr(), r.data_ptr<float>(), M, D, dt_code(xc),
                  (float)eps, cur_stream());
  return {y, r};
}

torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor scale, torch::Tensor rstd,
                          c10::optional<torch::Tensor> dscale_acc) {
  auto dyc = dy.contiguous();
  auto xc = x.contiguous();
  int D = (int)xc.size(-1);
  int64_t M = xc.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  if (dscale_acc.has_value()) check_acc(*dscale_acc, D, "dscale_acc");
  auto dx = torch::empty_like(xc);
  ahb_rmsnorm_bwd(dyc.data_ptr(), xc.data_ptr(), sc.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr(),
                  opt_ptr(dscale_acc), M, D, dt_code(xc), cur_stream());
  return dx;
}

void check_conv_x(const torch::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3 && x.stride(2) == 1 && x.stride(0) == x.size(1) * x.stride(1),
              "conv1d: x must be (B,L,C) with unit channel stride (a column slice is allowed)");
  TORCH_CHECK(x.size(2) % 8 == 0, "conv1d: C must be a multiple of 8");
}

torch::Tensor conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias, bool silu,
                         double clip) {
  check_conv_x(x);
  int B = (int)x.size(0), L = (int)x.size(1), C = (int)x.size(2);
  TORCH_CHECK(w.is_contiguous() && w.size(0) == C && w.size(1) == 4, "conv1d: w must be contiguous (C, 4)");
  auto y = torch::empty({B, L, C}, x.options());
  c10::optional<torch::Tensor> bf;
  if (bias.has_value()) bf = bias->to(at::kFloat).contiguous();
  ahb_conv1d_fwd(x.data_ptr(), x.stride(1), w.data_ptr(), dt_code(w), opt_ptr(bf), y.data_ptr(), B, L, C, dt_code(x),
                 silu ? 1 : 0, (float)clip, cur_stream());
  return y;
}

torch::Tensor conv1d_bwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias, torch::Tensor dy,
                         bool silu, double clip, torch::Tensor dw_acc, c10::optional<torch::Tensor> db_acc) {
  check_conv_x(x);
  int B = (int)x.size(0), L = (int)x.size(1), C = (int)x.size(2);
  check_acc(dw_acc, (int64_t)C * 4, "dw_acc");
  if (db_acc.has_value()) check_acc(*db_acc, C, "db_acc");
  c10::optional<torch::Tensor> bf;
  if (bias.has_value()) bf = bias->to(at::kFloat).contiguous();
  auto dyc = dy.contiguous();
  TORCH_CHECK(dyc.scalar_type() == x.scalar_type(), "conv1d_bwd: dy dtype");
  auto dx = torch::empty({B, L, C}, x.options());
  ahb_conv1d_bwd(x.data_ptr(), x.stride(1), w.data_ptr(), dt_code(w), opt_ptr(bf), dyc.data_ptr(), dx.data_ptr(),
                 dw_acc.data_ptr<float>(), opt_ptr(db_acc), B, L, C, dt_code(x), silu ? 1 : 0, (float)clip,
                 cur_stream());
  return dx;
}

void accumulate_(torch::Tensor acc, torch::Tensor g, double scale) {
  auto gc = g.contiguous();
  check_acc(acc, gc.numel(), "acc");
  ahb_accumulate(acc.data_ptr<float>(), gc.data_ptr(), gc.numel(), dt_code(gc), (float)scale, cur_stream());
}

torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor emb, at::ScalarType out_dtype) {
  auto idc = ids.to(at::kLong).contiguous();
  int64_t T = idc.numel();
  int D = (int)emb.size(1);
  TORCH_CHECK(emb.is_contiguous(), "embedding table must be contiguous");
  auto out = torch::empty({T, D}, emb.options().dtype(out_dtype));
  ahb_embedding_fwd(idc.data_ptr<int64_t>(), emb.data_ptr(), dt_code(emb), out.data_ptr(),
                    out_dtype == at::kBFloat16 ? AHB_BF16 : AHB_F32, T, D, emb.size(0), cur_stream());
  return out;
}

void embedding_bwd_(torch::Tensor ids, torch::Tensor dout, torch::Tensor acc) {
  auto idc = ids.to(at::kLong).contiguous();
  auto dc = dout.contiguous();
  check_acc(acc, acc.numel(), "acc");
  ahb_embedding_bwd(idc.data_ptr<int64_t>(), dc.data_ptr(), dt_code(dc), acc.data_ptr<float>(), idc.numel(),
                    (int)acc.size(1), acc.size(0), cur_stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "atomic_ai_hybrid_b200 sm_100a kernels";
  m.def("sanitize", &sanitize);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("conv1d_fwd", &conv1d_fwd);
  m.def("conv1d_bwd", &conv1d_bwd);
  m.def("accumulate_", &accumulate_);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd_", &embedding_bwd_);
}
