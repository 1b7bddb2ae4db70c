// Torch-facing bindings of the sm_100a kernels.  Only this file includes the
// torch headers; the kernels themselves are plain CUDA with raw-pointer
// launchers (launchers.h), which keeps them fast to compile and callable
// without the framework.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAGraphsC10Utils.h>
#include "launchers.h"
#include <cstdlib>
#include <map>
#include <mutex>

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

// expert weight-gradient accumulators: fp32, or bf16 for a store with 16-bit gradients
static bool check_acc_16(const torch::Tensor& t, int64_t n, const char* name) {
  TORCH_CHECK(t.is_cuda() && (t.scalar_type() == at::kFloat || t.scalar_type() == at::kBFloat16) &&
                  t.is_contiguous() && t.numel() == n,
              name, " must be a contiguous fp32 or bf16 CUDA tensor with ", n, " elements");
  return t.scalar_type() == at::kBFloat16;
}

// Fail loudly if a launch of this binding was rejected (bad configuration,
// missing shared-memory opt-in, no kernel image for the device ...).
void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, "atomic_ai_hybrid_b200: launch of ", what, " failed: ", cudaGetErrorString(e));
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
  check_launch("ahb_sanitize");
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
  check_launch("ahb_rmsnorm_fwd");
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
  torch::Tensor part;
  if (dscale_acc.has_value()) part = torch::zeros({(int64_t)ahb_rmsnorm_bwd_blocks(M, D), D}, xc.options().dtype(at::kFloat));
  ahb_rmsnorm_bwd(dyc.data_ptr(), xc.data_ptr(), sc.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr(),
                  opt_ptr(dscale_acc), part.defined() ? part.data_ptr<float>() : nullptr, M, D, dt_code(xc),
                  cur_stream());
  check_launch("ahb_rmsnorm_bwd");
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
  check_launch("ahb_conv1d_fwd");
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
  check_launch("ahb_conv1d_bwd");
  return dx;
}

void accumulate_(torch::Tensor acc, torch::Tensor g, double scale) {
  auto gc = g.contiguous();
  check_acc(acc, gc.numel(), "acc");
  ahb_accumulate(acc.data_ptr<float>(), gc.data_ptr(), gc.numel(), dt_code(gc), (float)scale, cur_stream());
  check_launch("ahb_accumulate");
}

torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor emb, at::ScalarType out_dtype) {
  auto idc = ids.to(at::kLong).contiguous();
  int64_t T = idc.numel();
  int D = (int)emb.size(1);
  TORCH_CHECK(emb.is_contiguous(), "embedding table must be contiguous");
  auto out = torch::empty({T, D}, emb.options().dtype(out_dtype));
  ahb_embedding_fwd(idc.data_ptr<int64_t>(), emb.data_ptr(), dt_code(emb), out.data_ptr(),
                    out_dtype == at::kBFloat16 ? AHB_BF16 : AHB_F32, T, D, emb.size(0), cur_stream());
  check_launch("ahb_embedding_fwd");
  return out;
}

void embedding_bwd_(torch::Tensor ids, torch::Tensor dout, torch::Tensor acc) {
  auto idc = ids.to(at::kLong).contiguous();
  auto dc = dout.contiguous();
  check_acc(acc, acc.numel(), "acc");
  ahb_embedding_bwd(idc.data_ptr<int64_t>(), dc.data_ptr(), dt_code(dc), acc.data_ptr<float>(), idc.numel(),
                    (int)acc.size(1), acc.size(0), cur_stream());
  check_launch("ahb_embedding_bwd");
}


// ------------------------------------------------------------ GDN-2
void check_gdn(const torch::Tensor& t, at::ScalarType dt, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == dt && t.dim() == 4, "gdn2: ", n,
              " must be a contiguous (B,L,H,128) CUDA tensor of type ", dt);
}

struct GdnShapes { int B, L, H, NC; };

GdnShapes gdn_shapes(const torch::Tensor& q) {
  int B = (int)q.size(0), L = (int)q.size(1), H = (int)q.size(2), D = (int)q.size(3);
  TORCH_CHECK(D == 128, "gdn2: head dim must be 128");
  TORCH_CHECK(L % 64 == 0, "gdn2: sequence length must be a multiple of 64");
  return {B, L, H, L / 64};
}

torch::Tensor& err_word();

void check_rc(int rc, const char* what);

// Points the scan kernels' per-phase cycle counters at `counters` (int64 (128,) on the device:
// SSD kernels slots 0-63, GDN kernels 64-127) or switches them off (None).
void phase_prof(c10::optional<torch::Tensor> counters) {
  char* p = nullptr;
  if (counters) {
    TORCH_CHECK(counters->is_cuda() && counters->scalar_type() == torch::kInt64 && counters->numel() >= 128 &&
                    counters->is_contiguous(),
                "phase_prof: int64 CUDA tensor of 128 counters");
    p = static_cast<char*>(counters->data_ptr());
  }
  check_rc(ahb_ssd_phase_prof(p), "ahb_ssd_phase_prof");
  check_rc(ahb_gdn_phase_prof(p ? p + 64 * 8 : nullptr), "ahb_gdn_phase_prof");
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "atomic_ai_hybrid_b200: ", what, " failed with code ", rc);
  check_launch(what);
}

// A (B,H,R,C) fp32 state argument: checked and made contiguous, or undefined when absent.
static torch::Tensor state_arg(const c10::optional<torch::Tensor>& t, const torch::Tensor& like, int64_t B, int64_t H,
                               int64_t R, int64_t Cc, const char* what) {
  if (!t.has_value() || !t->defined()) return torch::Tensor();
  TORCH_CHECK(t->is_cuda() && t->device() == like.device() && t->dim() == 4 && t->size(0) == B && t->size(1) == H &&
                  t->size(2) == R && t->size(3) == Cc,
              what, ": expected a (", B, ",", H, ",", R, ",", Cc, ") CUDA tensor");
  return t->to(at::kFloat).contiguous();
}

static float* fptr(const torch::Tensor& t) { return t.defined() ? t.data_ptr<float>() : nullptr; }

// Chunk intermediates of the forward: tile images wt, u, qg, kg (B,H,NC,64,128) and aqk
// (B,H,NC,64,64) bf16, gcl (B,H,NC,128) fp32, and the tile image of A (B,H,NC,64,64) bf16 when `want_a`.
struct GdnChunk { torch::Tensor wt, u, qg, kg, aqk, gcl, A; };

GdnChunk gdn_chunk(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& g,
                   const torch::Tensor& bg, const torch::Tensor& wg, float scale, bool want_a) {
  auto s = gdn_shapes(q);
  auto bf = q.options();
  auto f32 = q.options().dtype(at::kFloat);
  GdnChunk c;
  c.wt = torch::empty({s.B, s.H, s.NC, 64, 128}, bf);
  c.u = torch::empty_like(c.wt);
  c.qg = torch::empty_like(c.wt);
  c.kg = torch::empty_like(c.wt);
  c.aqk = torch::empty({s.B, s.H, s.NC, 64, 64}, bf);
  c.gcl = torch::empty({s.B, s.H, s.NC, 128}, f32);
  if (want_a) c.A = torch::empty({s.B, s.H, s.NC, 64, 64}, bf);
  check_rc(ahb_gdn_chunk_fwd_tc(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(), bg.data_ptr(),
                                wg.data_ptr(), scale, s.B, s.L, s.H, c.wt.data_ptr(), c.u.data_ptr(), c.qg.data_ptr(),
                                c.kg.data_ptr(), c.aqk.data_ptr(), c.gcl.data_ptr<float>(),
                                want_a ? c.A.data_ptr() : nullptr, err_word().data_ptr<int>(), cur_stream()),
           "ahb_gdn_chunk_fwd_tc");
  return c;
}

std::vector<torch::Tensor> gdn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                   torch::Tensor bg, torch::Tensor wg, double scale, bool want_state,
                                   c10::optional<torch::Tensor> h0) {
  for (auto* t : {&q, &k, &v, &bg, &wg}) check_gdn(*t, at::kBFloat16, "q/k/v/b/w");
  check_gdn(g, at::kFloat, "g");
  auto s = gdn_shapes(q);
  auto h0c = state_arg(h0, q, s.B, s.H, 128, 128, "gdn2 h0");
  auto c = gdn_chunk(q, k, v, g, bg, wg, (float)scale, false);
  auto o = torch::empty_like(q);
  torch::Tensor hf;
  if (want_state) hf = torch::empty({s.B, s.H, 128, 128}, q.options().dtype(at::kFloat));
  check_rc(ahb_gdn_state_fwd_tc(c.wt.data_ptr(), c.u.data_ptr(), c.qg.data_ptr(), c.kg.data_ptr(), c.aqk.data_ptr(),
                                c.gcl.data_ptr<float>(), (float)scale, s.B, s.L, s.H, fptr(h0c), o.data_ptr(),
                                want_state ? hf.data_ptr<float>() : nullptr, nullptr, nullptr,
                                err_word().data_ptr<int>(), cur_stream()),
           "ahb_gdn_state_fwd_tc");
  if (want_state) return {o, hf};
  return {o};
}

// Backward from the chunk intermediates of the forward (wt, qg, kg, aqk, gcl, A and the
// per-chunk states hs / vn): reverse state recurrence (from the gradient of the final state
// when given; it returns the gradient of the initial state when `want_dh0`), then the
// chunk-local backward.
static std::vector<torch::Tensor> gdn_bwd_core(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                                               const torch::Tensor& g, const torch::Tensor& bg,
                                               const torch::Tensor& wg, const torch::Tensor& doc, float sc,
                                               torch::Tensor wt, torch::Tensor qg, torch::Tensor kg,
                                               torch::Tensor aqk, const torch::Tensor& gcl,
                                               const torch::Tensor& A, torch::Tensor hs, torch::Tensor vn,
                                               const torch::Tensor& dhf, bool want_dh0) {
  auto s = gdn_shapes(q);
  auto st = cur_stream();
  auto dhs = torch::empty_like(hs);
  auto dvn = torch::empty({s.B, s.H, s.NC, 64, 128}, q.options());
  torch::Tensor dh0;
  if (want_dh0) dh0 = torch::empty({s.B, s.H, 128, 128}, q.options().dtype(at::kFloat));
  check_rc(ahb_gdn_state_bwd_tc(wt.data_ptr(), qg.data_ptr(), kg.data_ptr(), aqk.data_ptr(), gcl.data_ptr<float>(),
                                doc.data_ptr(), sc, s.B, s.L, s.H, fptr(dhf), dhs.data_ptr(), dvn.data_ptr(),
                                fptr(dh0), err_word().data_ptr<int>(), st),
           "ahb_gdn_state_bwd_tc");
  qg = torch::Tensor(); kg = torch::Tensor(); wt = torch::Tensor(); aqk = torch::Tensor();
  auto dq = torch::empty_like(q), dk = torch::empty_like(q), dv = torch::empty_like(q), db = torch::empty_like(q),
       dw = torch::empty_like(q);
  auto dg = torch::empty_like(g);
  check_rc(ahb_gdn_chunk_bwd_tc(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(), bg.data_ptr(),
                                wg.data_ptr(), doc.data_ptr(), hs.data_ptr(), dhs.data_ptr(), vn.data_ptr(),
                                dvn.data_ptr(), A.data_ptr(), sc, s.B, s.L, s.H, dq.data_ptr(), dk.data_ptr(),
                                dv.data_ptr(), db.data_ptr(), dw.data_ptr(), dg.data_ptr<float>(),
                                err_word().data_ptr<int>(), st),
           "ahb_gdn_chunk_bwd_tc");
  if (want_dh0) return {dq, dk, dv, dg, db, dw, dh0};
  return {dq, dk, dv, dg, db, dw};
}

static void gdn_states(const GdnChunk& c, const torch::Tensor& q, float sc, torch::Tensor* o, torch::Tensor& hs,
                       torch::Tensor& vn, const torch::Tensor& h0 = torch::Tensor(),
                       torch::Tensor* hf = nullptr) {
  auto s = gdn_shapes(q);
  hs = torch::empty({s.B, s.H, s.NC, 128, 128}, q.options());
  vn = torch::empty({s.B, s.H, s.NC, 64, 128}, q.options());
  if (hf) *hf = torch::empty({s.B, s.H, 128, 128}, q.options().dtype(at::kFloat));
  check_rc(ahb_gdn_state_fwd_tc(c.wt.data_ptr(), c.u.data_ptr(), c.qg.data_ptr(), c.kg.data_ptr(), c.aqk.data_ptr(),
                                c.gcl.data_ptr<float>(), sc, s.B, s.L, s.H, fptr(h0), o ? o->data_ptr() : nullptr,
                                hf ? hf->data_ptr<float>() : nullptr, hs.data_ptr(), vn.data_ptr(),
                                err_word().data_ptr<int>(), cur_stream()),
           "ahb_gdn_state_fwd_tc");
}

// Forward for training: also returns the chunk intermediates the backward needs
// {o, wt, qg, kg, aqk, gcl, A, hs, vn}, so nothing is recomputed there; the recurrence starts
// from `h0` (B,H,128,128) when given, and `want_final` appends the final state (fp32).
std::vector<torch::Tensor> gdn_fwd_train(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                         torch::Tensor bg, torch::Tensor wg, double scale,
                                         c10::optional<torch::Tensor> h0, bool want_final) {
  for (auto* t : {&q, &k, &v, &bg, &wg}) check_gdn(*t, at::kBFloat16, "q/k/v/b/w");
  check_gdn(g, at::kFloat, "g");
  auto s = gdn_shapes(q);
  auto h0c = state_arg(h0, q, s.B, s.H, 128, 128, "gdn2 h0");
  auto c = gdn_chunk(q, k, v, g, bg, wg, (float)scale, true);
  auto o = torch::empty_like(q);
  torch::Tensor hs, vn, hf;
  gdn_states(c, q, (float)scale, &o, hs, vn, h0c, want_final ? &hf : nullptr);
  if (want_final) return {o, c.wt, c.qg, c.kg, c.aqk, c.gcl, c.A, hs, vn, hf};
  return {o, c.wt, c.qg, c.kg, c.aqk, c.gcl, c.A, hs, vn};
}

// `dh_final`: gradient of the final state (or none); `want_dh0` appends the gradient of the
// initial state to {dq, dk, dv, dg, db, dw}.
std::vector<torch::Tensor> gdn_bwd_saved(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                         torch::Tensor bg, torch::Tensor wg, torch::Tensor dout, double scale,
                                         std::vector<torch::Tensor> saved, c10::optional<torch::Tensor> dh_final,
                                         bool want_dh0) {
  TORCH_CHECK(saved.size() == 8, "gdn_bwd_saved: expects {wt, qg, kg, aqk, gcl, A, hs, vn}");
  auto s = gdn_shapes(q);
  auto doc = dout.to(at::kBFloat16).contiguous();
  auto dhf = state_arg(dh_final, q, s.B, s.H, 128, 128, "gdn2 dh_final");
  return gdn_bwd_core(q, k, v, g, bg, wg, doc, (float)scale, saved[0], saved[1], saved[2], saved[3], saved[4],
                      saved[5], saved[6], saved[7], dhf, want_dh0);
}

// Backward that recomputes the forward's chunk intermediates (memory-lean path); `h0` is the
// forward's initial state.
std::vector<torch::Tensor> gdn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                   torch::Tensor bg, torch::Tensor wg, torch::Tensor dout, double scale,
                                   c10::optional<torch::Tensor> h0, c10::optional<torch::Tensor> dh_final,
                                   bool want_dh0) {
  auto s = gdn_shapes(q);
  auto doc = dout.to(at::kBFloat16).contiguous();
  const float sc = (float)scale;
  auto h0c = state_arg(h0, q, s.B, s.H, 128, 128, "gdn2 h0");
  auto dhf = state_arg(dh_final, q, s.B, s.H, 128, 128, "gdn2 dh_final");
  auto c = gdn_chunk(q, k, v, g, bg, wg, sc, true);
  torch::Tensor hs, vn;
  gdn_states(c, q, sc, nullptr, hs, vn, h0c);
  c.u = torch::Tensor();
  return gdn_bwd_core(q, k, v, g, bg, wg, doc, sc, c.wt, c.qg, c.kg, c.aqk, c.gcl, c.A, hs, vn, dhf, want_dh0);
}

// ------------------------------------------------------------ Mamba2 SSD
void check_ssd(const torch::Tensor& x, const torch::Tensor& dt, const torch::Tensor& A, const torch::Tensor& Bm,
               const torch::Tensor& Cm) {
  for (auto* t : {&x, &dt, &Bm, &Cm})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                "ssd: x, dt, B, C must be contiguous bf16 CUDA tensors");
  TORCH_CHECK(x.dim() == 4 && dt.sizes() == x.sizes(), "ssd: x, dt must be (B,L,H,64)");
  TORCH_CHECK(ahb_ssd_supported((int)x.size(3), (int)Bm.size(2)) == 64, "ssd: head dim 64 and d_state 128 only");
  TORCH_CHECK(x.size(1) % 64 == 0, "ssd: L must be a multiple of 64");
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kFloat && A.numel() == x.size(2), "ssd: A must be fp32 (H,)");
  TORCH_CHECK(Bm.dim() == 3 && Bm.sizes() == Cm.sizes() && Bm.size(0) == x.size(0) && Bm.size(1) == x.size(1),
              "ssd: B, C must be (B,L,128)");
}

struct SsdFwd { torch::Tensor y, sin_t, dec_t, cl, yd_t, s_final; };

// Forward (chunk kernel + state recurrence, from the initial state `s0` (B,H,64,128) when
// defined); with `keep_states` also the per-chunk incoming states (tile images) the backward
// needs, beside the decay images and last cumsums; `want_final` keeps the final state (fp32).
static SsdFwd ssd_forward(const torch::Tensor& x, const torch::Tensor& dt, const torch::Tensor& A,
                          const torch::Tensor& Bm, const torch::Tensor& Cm, bool keep_states, bool want_y,
                          const torch::Tensor& s0 = torch::Tensor(), bool want_final = false) {
  int B = (int)x.size(0), L = (int)x.size(1), H = (int)x.size(2), NC = L / 64;
  auto bf = x.options();
  SsdFwd f;
  if (want_final) f.s_final = torch::empty({B, H, 64, 128}, x.options().dtype(at::kFloat));
  auto send = torch::empty({B, H, NC, 128, 64}, bf);
  f.yd_t = torch::empty({B, H, NC, 64, 64}, x.options().dtype(at::kFloat));
  f.dec_t = torch::empty({B, H, NC, 64, 64}, bf);
  f.cl = torch::empty({B, H, NC, 64}, x.options().dtype(at::kFloat));
  if (keep_states) f.sin_t = torch::empty({B, H, NC, 128, 64}, bf);
  f.y = torch::empty_like(x);
  check_rc(ahb_ssd_fwd_tc(x.data_ptr(), dt.data_ptr(), A.data_ptr<float>(), Bm.data_ptr(), Cm.data_ptr(), B, L, H,
                          send.data_ptr(), f.yd_t.data_ptr(), f.dec_t.data_ptr(), f.cl.data_ptr<float>(), fptr(s0),
                          fptr(f.s_final),
                          f.y.data_ptr(), keep_states ? f.sin_t.data_ptr() : nullptr, err_word().data_ptr<int>(),
                          cur_stream()),
           "ahb_ssd_fwd_tc");
  (void)want_y;
  return f;
}

torch::Tensor ssd_fwd(torch::Tensor x, torch::Tensor dt, torch::Tensor A, torch::Tensor Bm, torch::Tensor Cm) {
  check_ssd(x, dt, A, Bm, Cm);
  return ssd_forward(x, dt, A, Bm, Cm, false, true).y;
}

// Forward for training: {y, incoming states (tile images), decay images, last cumsums, intra-chunk
// outputs}; ssd_bwd takes the last four back.  The recurrence starts from `s0` (B,H,64,128)
// when given; `want_final` appends the final state (fp32).
std::vector<torch::Tensor> ssd_fwd_train(torch::Tensor x, torch::Tensor dt, torch::Tensor A, torch::Tensor Bm,
                                         torch::Tensor Cm, c10::optional<torch::Tensor> s0, bool want_final) {
  check_ssd(x, dt, A, Bm, Cm);
  auto s0c = state_arg(s0, x, x.size(0), x.size(2), 64, 128, "ssd s0");
  auto f = ssd_forward(x, dt, A, Bm, Cm, true, true, s0c, want_final);
  if (want_final) return {f.y, f.sin_t, f.dec_t, f.cl, f.yd_t, f.s_final};
  return {f.y, f.sin_t, f.dec_t, f.cl, f.yd_t};
}

// {dx, ddt, dA, dB, dC} (+ the gradient of the initial state with `want_ds0`); `s0` is the
// forward's initial state (used when the saved states are absent and the forward reruns),
// `ds_final` the gradient of its final state.
std::vector<torch::Tensor> ssd_bwd(torch::Tensor x, torch::Tensor dt, torch::Tensor A, torch::Tensor Bm,
                                   torch::Tensor Cm, torch::Tensor dy, c10::optional<torch::Tensor> states,
                                   c10::optional<torch::Tensor> decays, c10::optional<torch::Tensor> cumsums,
                                   c10::optional<torch::Tensor> ydiag, c10::optional<torch::Tensor> s0,
                                   c10::optional<torch::Tensor> ds_final, bool want_ds0) {
  check_ssd(x, dt, A, Bm, Cm);
  int B = (int)x.size(0), L = (int)x.size(1), H = (int)x.size(2), NC = L / 64;
  auto s0c = state_arg(s0, x, B, H, 64, 128, "ssd s0");
  auto dsf = state_arg(ds_final, x, B, H, 64, 128, "ssd ds_final");
  auto dyc = dy.to(at::kBFloat16).contiguous();
  auto f32 = x.options().dtype(at::kFloat);
  const bool ready = states.has_value() && states->defined() && decays.has_value() && decays->defined() &&
                     cumsums.has_value() && cumsums->defined() && ydiag.has_value() && ydiag->defined();
  SsdFwd f;
  if (ready) {
    f.sin_t = *states;
    f.dec_t = *decays;
    f.cl = *cumsums;
    f.yd_t = *ydiag;
    TORCH_CHECK(f.yd_t.numel() == (int64_t)B * H * NC * 64 * 64, "ssd_bwd: saved intra-chunk outputs do not match");
    TORCH_CHECK(f.sin_t.numel() == (int64_t)B * H * NC * 128 * 64 && f.dec_t.numel() == (int64_t)B * H * NC * 64 * 64 &&
                    f.cl.numel() == (int64_t)B * H * NC * 64,
                "ssd_bwd: saved states do not match");
  } else {
    f = ssd_forward(x, dt, A, Bm, Cm, true, false, s0c);
  }
  auto st = cur_stream();
  auto dse = torch::empty({B, H, NC, 128, 64}, x.options());
  torch::Tensor ds0;
  if (want_ds0) ds0 = torch::empty({B, H, 64, 128}, f32);
  check_rc(ahb_ssd_state_bwd_tc(Cm.data_ptr(), dyc.data_ptr(), f.dec_t.data_ptr(), f.cl.data_ptr<float>(), B, L, H,
                                fptr(dsf), dse.data_ptr(), fptr(ds0), err_word().data_ptr<int>(), st),
           "ahb_ssd_state_bwd_tc");
  auto dx = torch::empty_like(x), ddt = torch::empty_like(x);
  auto dB = torch::empty(Bm.sizes(), f32), dC = torch::empty(Cm.sizes(), f32);
  auto dA = torch::zeros({H}, f32);
  const int G = ahb_ssd_head_groups(H);
  auto dBp = torch::empty({G, B, L, 128}, f32), dCp = torch::empty({G, B, L, 128}, f32);
  check_rc(ahb_ssd_bwd_chunk_tc(x.data_ptr(), dt.data_ptr(), A.data_ptr<float>(), Bm.data_ptr(), Cm.data_ptr(),
                                dyc.data_ptr(), B, L, H, f.sin_t.data_ptr(), dse.data_ptr(), f.yd_t.data_ptr(),
                                dx.data_ptr(), ddt.data_ptr(), dB.data_ptr<float>(), dC.data_ptr<float>(),
                                dA.data_ptr<float>(), dBp.data_ptr<float>(), dCp.data_ptr<float>(),
                                err_word().data_ptr<int>(), st),
           "ahb_ssd_bwd_chunk_tc");
  if (want_ds0) return {dx, ddt, dA, dB, dC, ds0};
  return {dx, ddt, dA, dB, dC};
}

static std::pair<void* const*, int> peer_table(const c10::optional<torch::Tensor>& t);

// ------------------------------------------------------------ MoE (grouped GEMM on tcgen05)
int num_sms() {
  static int n = 0;
  if (!n) { int d; cudaGetDevice(&d); cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d); }
  return n;
}

torch::Tensor& err_word() {
  static torch::Tensor e;
  if (!e.defined()) e = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA));
  return e;
}

int64_t gemm_error() { return err_word().item<int>(); }
void gemm_error_reset() { err_word().zero_(); }

void gemm_check(int rc, const char* what) { TORCH_CHECK(rc == 0, "moe_gemm (", what, ") setup failed: code ", rc); }

// Generic access for tests: C = A B^T (A: M x K, B: N x K, bf16, K-major), single group; `pair` runs
// the CTA-pair kernel (256 x 256 tiles; rows of the last tile beyond M are read as zeros and not
// stored).
torch::Tensor gemm_dense(torch::Tensor a, torch::Tensor b, bool pair) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.is_contiguous() && b.is_contiguous() &&
              b.scalar_type() == at::kBFloat16, "gemm_dense: bf16 contiguous");
  int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(K % 64 == 0 && N % 32 == 0 && (pair || M % 128 == 0), "gemm_dense: K%64, N%32, M%128 (single CTA)");
  const int64_t Mp = pair ? (M + 255) / 256 * 256 : M;
  auto off = torch::arange(0, Mp + 1, Mp, torch::dtype(torch::kInt32).device(a.device()));
  auto c = torch::empty({M, N}, a.options());
  int rc = ahb_moe_gemm(AHB_GEMM_DENSE | (pair ? AHB_GEMM_PAIR : 0), a.data_ptr(), nullptr, M, K, b.data_ptr(),
                        nullptr, N, K, 0, off.data_ptr<int>(), 1, (int)N, 0, (int)K, (int)(K / 64), c.data_ptr(),
                        nullptr, nullptr, nullptr, nullptr, 0.f, err_word().data_ptr<int>(), num_sms(), cur_stream(),
                        nullptr, pair ? (int)M : 0);
  gemm_check(rc, "dense");
  return c;
}

// CTA-pair grouped GEMMs (256 x 256 tiles over two SMs) for the local MoE layer, whose routing
// then pads each expert's segment to 256 rows; AHB_MOE_PAIR=0 keeps the single-CTA kernel and
// 128-row segments.  Fixed for the process, so a forward and its backward agree.
static bool moe_pair() {
  static const bool on = [] {
    const char* e = std::getenv("AHB_MOE_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Expert FFN on expert-grouped rows (segments of `off`, padded to 128 rows, or to 256 with
// `pair`, which runs the M-grouped GEMMs on CTA pairs): returns {a1, a3 (empty for GELU), h, ys}.
static std::vector<torch::Tensor> moe_expert_fwd_impl(const torch::Tensor& xs, const torch::Tensor& off, int64_t R,
                                                      const torch::Tensor& w1, const torch::Tensor& w2,
                                                      const c10::optional<torch::Tensor>& w3, bool swiglu,
                                                      bool pair = false) {
  const int PM = pair ? AHB_GEMM_PAIR : 0;
  const int d = (int)xs.size(1), E = (int)w1.size(0), F = (int)w1.size(2);
  TORCH_CHECK(d % 256 == 0 && F % 256 == 0, "moe: d_model and d_ff must be multiples of 256");
  TORCH_CHECK(E <= 192, "moe: at most 192 experts per call");
  auto st = cur_stream();
  auto h = torch::empty({R, F}, xs.options());
  auto a1 = torch::empty_like(h);
  torch::Tensor a3;
  int* err = err_word().data_ptr<int>();
  int rc;
  if (swiglu) {
    TORCH_CHECK(w3.has_value(), "moe: swiglu needs w3");
    a3 = torch::empty_like(h);
    rc = ahb_moe_gemm(AHB_GEMM_FWD_SWIGLU | PM, xs.data_ptr(), nullptr, R, d, w1.data_ptr(), w3->data_ptr(),
                      (int64_t)E * d, F, d, off.data_ptr<int>(), E, F, 0, d, d / 64, h.data_ptr(), a1.data_ptr(),
                      a3.data_ptr(), nullptr, nullptr, 1e3f, err, num_sms(), st);
  } else {
    rc = ahb_moe_gemm(AHB_GEMM_FWD_GELU | PM, xs.data_ptr(), nullptr, R, d, w1.data_ptr(), nullptr, (int64_t)E * d, F, d,
                      off.data_ptr<int>(), E, F, 0, d, d / 64, h.data_ptr(), a1.data_ptr(), nullptr, nullptr, nullptr,
                      1e3f, err, num_sms(), st);
    a3 = torch::empty({0}, xs.options());
  }
  gemm_check(rc, "fwd up");
  auto ys = torch::empty({R, d}, xs.options());
  rc = ahb_moe_gemm(AHB_GEMM_FWD_DOWN | PM, h.data_ptr(), nullptr, R, F, w2.data_ptr(), nullptr, (int64_t)E * F, d, F,
                    off.data_ptr<int>(), E, d, 0, F, F / 64, ys.data_ptr(), nullptr, nullptr, nullptr, nullptr, 1e3f,
                    err, num_sms(), st);
  gemm_check(rc, "fwd down");
  return {a1, a3, h, ys};
}

// Backward of the expert FFN from the row gradients dys (padding rows zero): weight
// gradients are ADDED into dw*_acc; returns the row gradients dxs.  The K-grouped weight
// gradients always run on CTA pairs (their rows are d_model / d_ff, multiples of 256); the
// M-grouped products do with `pair` (segments padded to 256 rows).
static torch::Tensor moe_expert_bwd_impl(const torch::Tensor& dys, const torch::Tensor& off, const torch::Tensor& xs,
                                         const torch::Tensor& a1, const torch::Tensor& a3, const torch::Tensor& h,
                                         const torch::Tensor& w1, const torch::Tensor& w2,
                                         const c10::optional<torch::Tensor>& w3, const torch::Tensor& dw1_acc,
                                         const torch::Tensor& dw2_acc, const c10::optional<torch::Tensor>& dw3_acc,
                                         bool swiglu, bool pair = false) {
  const int PM = pair ? AHB_GEMM_PAIR : 0;
  int PW = moe_pair() ? AHB_GEMM_PAIR : 0;
  const int64_t R = xs.size(0);
  const int d = (int)xs.size(1), E = (int)w1.size(0), F = (int)w1.size(2);
  auto st = cur_stream();
  const bool a16 = check_acc_16(dw1_acc, w1.numel(), "dw1_acc");
  TORCH_CHECK(check_acc_16(dw2_acc, w2.numel(), "dw2_acc") == a16, "moe_bwd: accumulators of one dtype");
  if (a16) PW |= AHB_GEMM_ACC_BF16;
  int* err = err_word().data_ptr<int>();
  auto dA1 = torch::empty({R, F}, xs.options());
  torch::Tensor dA3;
  int rc;
  if (swiglu) {
    dA3 = torch::empty_like(dA1);
    rc = ahb_moe_gemm(AHB_GEMM_DH_SWIGLU | PM, dys.data_ptr(), nullptr, R, d, w2.data_ptr(), nullptr, (int64_t)E * F, d,
                      F, off.data_ptr<int>(), E, F, 0, d, d / 64, dA1.data_ptr(), dA3.data_ptr(), nullptr,
                      a1.data_ptr(), a3.data_ptr(), 0.f, err, num_sms(), st);
  } else {
    rc = ahb_moe_gemm(AHB_GEMM_DH_GELU | PM, dys.data_ptr(), nullptr, R, d, w2.data_ptr(), nullptr, (int64_t)E * F, d, F,
                      off.data_ptr<int>(), E, F, 0, d, d / 64, dA1.data_ptr(), nullptr, nullptr, a1.data_ptr(),
                      nullptr, 0.f, err, num_sms(), st);
  }
  gemm_check(rc, "dh");
  rc = ahb_moe_gemm(AHB_GEMM_WGRAD | PW, h.data_ptr(), nullptr, R, F, dys.data_ptr(), nullptr, R, d, 0,
                    off.data_ptr<int>(), E, d, F, 0, 0, dw2_acc.data_ptr(), nullptr, nullptr, nullptr, nullptr,
                    0.f, err, num_sms(), st);
  gemm_check(rc, "wgrad w2");
  auto dxs = torch::empty({R, d}, xs.options());
  if (swiglu) {
    rc = ahb_moe_gemm(AHB_GEMM_DX | PM, dA1.data_ptr(), dA3.data_ptr(), R, F, w1.data_ptr(), w3->data_ptr(),
                      (int64_t)E * d, F, d, off.data_ptr<int>(), E, d, 0, 2 * F, F / 64, dxs.data_ptr(), nullptr,
                      nullptr, nullptr, nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "dx");
    TORCH_CHECK(dw3_acc.has_value(), "moe_bwd: dw3_acc");
    TORCH_CHECK(check_acc_16(*dw3_acc, w3->numel(), "dw3_acc") == a16, "moe_bwd: accumulators of one dtype");
    rc = ahb_moe_gemm(AHB_GEMM_WGRAD_DUAL | PW, xs.data_ptr(), nullptr, R, d, dA1.data_ptr(), dA3.data_ptr(), R, F, 0,
                      off.data_ptr<int>(), E, F, d, 0, 0, dw1_acc.data_ptr(), dw3_acc->data_ptr(),
                      nullptr, nullptr, nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "wgrad w1/w3");
  } else {
    rc = ahb_moe_gemm(AHB_GEMM_DX | PM, dA1.data_ptr(), nullptr, R, F, w1.data_ptr(), nullptr, (int64_t)E * d, F, d,
                      off.data_ptr<int>(), E, d, 0, F, F / 64, dxs.data_ptr(), nullptr, nullptr, nullptr, nullptr,
                      0.f, err, num_sms(), st);
    gemm_check(rc, "dx");
    rc = ahb_moe_gemm(AHB_GEMM_WGRAD | PW, xs.data_ptr(), nullptr, R, d, dA1.data_ptr(), nullptr, R, F, 0,
                      off.data_ptr<int>(), E, F, d, 0, 0, dw1_acc.data_ptr(), nullptr, nullptr, nullptr,
                      nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "wgrad w1");
  }
  return dxs;
}

// forward: returns {out, pos, off, row_src, xs, a1, a3, h, ys}
std::vector<torch::Tensor> moe_fwd(torch::Tensor x, torch::Tensor top_idx, torch::Tensor gate, torch::Tensor w1,
                                   torch::Tensor w2, c10::optional<torch::Tensor> w3,
                                   c10::optional<torch::Tensor> shared, bool swiglu) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "moe: x bf16 (T,d)");
  for (auto* w : {&w1, &w2})
    TORCH_CHECK(w->scalar_type() == at::kBFloat16 && w->is_contiguous(), "moe: expert weights must be contiguous bf16");
  const int T = (int)x.size(0), d = (int)x.size(1), k = (int)top_idx.size(1);
  const int E = (int)w1.size(0), F = (int)w1.size(2);
  TORCH_CHECK(d % 256 == 0 && F % 256 == 0, "moe: d_model and d_ff must be multiples of 256");
  TORCH_CHECK(E <= 192 && k <= 8, "moe: at most 192 routed experts and top-8 per kernel call");
  auto dev = x.device();
  auto i32 = torch::dtype(torch::kInt32).device(dev);
  auto eidx = top_idx.t().contiguous().to(torch::kInt32);
  auto gatec = gate.to(at::kFloat).contiguous();
  const bool pair = moe_pair();
  const int pad = pair ? 256 : 128;
  const int64_t Rcap = ((int64_t)T * k + (int64_t)E * pad + pad - 1) / pad * pad;
  auto counts = torch::empty({E}, i32), off = torch::empty({E + 1}, i32);
  auto pos = torch::empty({(int64_t)T * k}, i32), row_src = torch::empty({Rcap}, i32);
  auto st = cur_stream();
  ahb_moe_route(eidx.data_ptr<int>(), T, k, E, counts.data_ptr<int>(), off.data_ptr<int>(), pos.data_ptr<int>(),
                row_src.data_ptr<int>(), Rcap, st, pad);
  check_launch("ahb_moe_route");
  auto xs = torch::empty({Rcap, d}, x.options());
  ahb_moe_gather(x.data_ptr(), row_src.data_ptr<int>(), Rcap, d, xs.data_ptr(), st);
  check_launch("ahb_moe_gather");
  auto g = moe_expert_fwd_impl(xs, off, Rcap, w1, w2, w3, swiglu, pair);
  auto a1 = g[0], a3 = g[1], h = g[2], ys = g[3];
  auto out = torch::empty_like(x);
  const void* sh = nullptr;
  torch::Tensor shc;
  if (shared.has_value() && shared->defined()) {
    shc = shared->to(at::kBFloat16).contiguous();
    sh = shc.data_ptr();
  }
  ahb_moe_combine(ys.data_ptr(), pos.data_ptr<int>(), gatec.data_ptr<float>(), sh, T, k, d, out.data_ptr(), st);
  check_launch("ahb_moe_combine");
  return {out, pos, off, row_src, xs, a1, a3, h, ys};
}

// backward: weight gradients are ADDED into dw*_acc (fp32, shapes of w*); returns {dx, dgate}
std::vector<torch::Tensor> moe_bwd(torch::Tensor dout, torch::Tensor gate, torch::Tensor w1, torch::Tensor w2,
                                   c10::optional<torch::Tensor> w3, torch::Tensor pos, torch::Tensor off,
                                   torch::Tensor row_src, torch::Tensor xs, torch::Tensor a1, torch::Tensor a3,
                                   torch::Tensor h, torch::Tensor ys, torch::Tensor dw1_acc, torch::Tensor dw2_acc,
                                   c10::optional<torch::Tensor> dw3_acc, bool swiglu) {
  const int T = (int)dout.size(0), d = (int)dout.size(1), k = (int)gate.size(1);
  const int64_t Rcap = xs.size(0);
  auto st = cur_stream();
  auto doc = dout.to(at::kBFloat16).contiguous();
  auto gatec = gate.to(at::kFloat).contiguous();
  auto dys = torch::empty({Rcap, d}, xs.options());
  ahb_moe_zero_pad(dys.data_ptr(), row_src.data_ptr<int>(), Rcap, d, st);
  check_launch("ahb_moe_zero_pad");
  auto dgate = torch::empty({T, k}, gatec.options());
  ahb_moe_combine_bwd(doc.data_ptr(), ys.data_ptr(), pos.data_ptr<int>(), gatec.data_ptr<float>(), T, k, d,
                      dys.data_ptr(), dgate.data_ptr<float>(), st);
  check_launch("ahb_moe_combine_bwd");
  auto dxs = moe_expert_bwd_impl(dys, off, xs, a1, a3, h, w1, w2, w3, dw1_acc, dw2_acc, dw3_acc, swiglu, moe_pair());
  auto dx = torch::empty({T, d}, xs.options());
  ahb_moe_scatter_add(dxs.data_ptr(), pos.data_ptr<int>(), T, k, d, dx.data_ptr(), st);
  check_launch("ahb_moe_scatter_add");
  return {dx, dgate};
}

// ------------------------------------------------------------ expert parallelism (ep.cu + the expert FFN)
// Local routing of this rank's assignments: {eidx (k*T, order a = j*T + t), counts (E), off (E+1, segments
// padded to 128), pos (k*T: off[e] + stable rank of a among the assignments to e)}
std::vector<torch::Tensor> moe_route_local(torch::Tensor top_idx, int64_t E) {
  const int T = (int)top_idx.size(0), k = (int)top_idx.size(1);
  auto i32 = torch::dtype(torch::kInt32).device(top_idx.device());
  auto eidx = top_idx.t().contiguous().to(torch::kInt32);
  const int64_t Rcap = ((int64_t)T * k + E * 128 + 127) / 128 * 128;
  auto counts = torch::empty({E}, i32), off = torch::empty({E + 1}, i32);
  auto pos = torch::empty({(int64_t)T * k}, i32), row_src = torch::empty({Rcap}, i32);
  ahb_moe_route(eidx.data_ptr<int>(), T, k, (int)E, counts.data_ptr<int>(), off.data_ptr<int>(), pos.data_ptr<int>(),
                row_src.data_ptr<int>(), Rcap, cur_stream());
  check_launch("ahb_moe_route");
  return {eidx, counts, off, pos};
}

void ep_publish(torch::Tensor counts, torch::Tensor peers, int64_t rank) {
  auto pt = peer_table(peers);
  ahb_ep_publish(counts.data_ptr<int>(), (int)counts.numel(), reinterpret_cast<int* const*>(pt.first), pt.second,
                 (int)rank, cur_stream());
  check_launch("ahb_ep_publish");
}

// src: x (T, d) when src_by_token, else rows (k*T, d) in assignment order
void ep_dispatch(torch::Tensor src, bool src_by_token, int64_t T, int64_t k, torch::Tensor eidx, torch::Tensor pos,
                 torch::Tensor off, torch::Tensor dst_base, int64_t El, torch::Tensor recv_peers,
                 c10::optional<torch::Tensor> meta_peers, int64_t rank, c10::optional<torch::Tensor> dst_pos) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.size(1) % 8 == 0,
              "ep_dispatch: bf16 rows");
  auto rp = peer_table(recv_peers);
  auto mp = peer_table(meta_peers);
  ahb_ep_dispatch(src.data_ptr(), src_by_token ? 1 : 0, (int)T, (int)k, (int)src.size(1), eidx.data_ptr<int>(),
                  pos.data_ptr<int>(), off.data_ptr<int>(), dst_base.data_ptr<int>(), (int)El, rp.first, mp.first,
                  (int)rank, dst_pos.has_value() && dst_pos->defined() ? dst_pos->data_ptr<int>() : nullptr,
                  cur_stream());
  check_launch("ahb_ep_dispatch");
}

void ep_return(torch::Tensor rows, torch::Tensor meta, int64_t R, torch::Tensor ret_peers) {
  auto pt = peer_table(ret_peers);
  ahb_ep_return(rows.data_ptr(), meta.data_ptr(), R, (int)rows.size(1), pt.first, cur_stream());
  check_launch("ahb_ep_return");
}

void ep_zero_pad(torch::Tensor rows, c10::optional<torch::Tensor> meta, torch::Tensor off, torch::Tensor seg) {
  ahb_ep_zero_pad(rows.data_ptr(), meta.has_value() && meta->defined() ? meta->data_ptr() : nullptr,
                  off.data_ptr<int>(), seg.data_ptr<int>(), (int)seg.numel(), (int)rows.size(1), cur_stream());
  check_launch("ahb_ep_zero_pad");
}

std::vector<torch::Tensor> moe_expert_fwd(torch::Tensor xs, torch::Tensor off, torch::Tensor w1, torch::Tensor w2,
                                          c10::optional<torch::Tensor> w3, bool swiglu) {
  return moe_expert_fwd_impl(xs, off, xs.size(0), w1, w2, w3, swiglu);
}

torch::Tensor moe_expert_bwd(torch::Tensor dys, torch::Tensor off, torch::Tensor xs, torch::Tensor a1,
                             torch::Tensor a3, torch::Tensor h, torch::Tensor w1, torch::Tensor w2,
                             c10::optional<torch::Tensor> w3, torch::Tensor dw1_acc, torch::Tensor dw2_acc,
                             c10::optional<torch::Tensor> dw3_acc, bool swiglu) {
  return moe_expert_bwd_impl(dys, off, xs, a1, a3, h, w1, w2, w3, dw1_acc, dw2_acc, dw3_acc, swiglu);
}

// rows (k*T, d) in assignment order: out[t] = sanitize(shared[t] + sum_j gate[t,j] sanitize(rows[j*T+t]))
torch::Tensor moe_combine_rows(torch::Tensor rows, torch::Tensor gate, c10::optional<torch::Tensor> shared) {
  const int T = (int)gate.size(0), k = (int)gate.size(1), d = (int)rows.size(1);
  auto ident = torch::arange(0, (int64_t)T * k, rows.options().dtype(at::kInt));
  auto gatec = gate.to(at::kFloat).contiguous();
  auto out = torch::empty({T, d}, rows.options());
  torch::Tensor shc;
  if (shared.has_value() && shared->defined()) shc = shared->to(at::kBFloat16).contiguous();
  ahb_moe_combine(rows.data_ptr(), ident.data_ptr<int>(), gatec.data_ptr<float>(),
                  shc.defined() ? shc.data_ptr() : nullptr, T, k, d, out.data_ptr(), cur_stream());
  check_launch("ahb_moe_combine");
  return out;
}

// {drows (k*T, d), dgate (T, k)}
std::vector<torch::Tensor> moe_combine_rows_bwd(torch::Tensor dout, torch::Tensor rows, torch::Tensor gate) {
  const int T = (int)gate.size(0), k = (int)gate.size(1), d = (int)rows.size(1);
  auto ident = torch::arange(0, (int64_t)T * k, rows.options().dtype(at::kInt));
  auto doc = dout.to(at::kBFloat16).contiguous();
  auto gatec = gate.to(at::kFloat).contiguous();
  auto drows = torch::empty_like(rows);
  auto dgate = torch::empty({T, k}, gatec.options());
  ahb_moe_combine_bwd(doc.data_ptr(), rows.data_ptr(), ident.data_ptr<int>(), gatec.data_ptr<float>(), T, k, d,
                      drows.data_ptr(), dgate.data_ptr<float>(), cur_stream());
  check_launch("ahb_moe_combine_bwd");
  return {drows, dgate};
}

// dx[t] = sum_j rows[j*T+t]
torch::Tensor moe_sum_rows(torch::Tensor rows, int64_t T, int64_t k) {
  const int d = (int)rows.size(1);
  auto ident = torch::arange(0, T * k, rows.options().dtype(at::kInt));
  auto dx = torch::empty({T, d}, rows.options());
  ahb_moe_scatter_add(rows.data_ptr(), ident.data_ptr<int>(), (int)T, (int)k, d, dx.data_ptr(), cur_stream());
  check_launch("ahb_moe_scatter_add");
  return dx;
}

// ------------------------------------------------------------ fused optimizer
// table: int64 (S, 8) = [off, coff, len, label, group, flags, bias_row, 0]; gscale fp32 (S,)
// returns {segs (uint8 device), cstart (int32 device, S+1)} and the block count in cstart[S]
std::vector<torch::Tensor> optim_make_table(torch::Tensor table, torch::Tensor gscale, int64_t device_index) {
  TORCH_CHECK(table.device().is_cpu() && table.scalar_type() == at::kLong && table.dim() == 2 && table.size(1) == 8,
              "optim_make_table: int64 (S,8) CPU table");
  const int64_t S = table.size(0);
  auto t = table.contiguous();
  auto gs = gscale.to(at::kFloat).contiguous();
  auto host = torch::empty({S * (int64_t)sizeof(AhbSegInfo)}, torch::kUInt8);
  auto cs = torch::empty({S + 1}, torch::kInt32);
  AhbSegInfo* info = reinterpret_cast<AhbSegInfo*>(host.data_ptr<uint8_t>());
  const int64_t* tp = t.data_ptr<int64_t>();
  int* cp = cs.data_ptr<int>();
  const int chunk = ahb_optim_chunk();
  int64_t blocks = 0;
  for (int64_t i = 0; i < S; ++i) {
    info[i].off = tp[i * 8 + 0];
    info[i].coff = tp[i * 8 + 1];
    info[i].len = tp[i * 8 + 2];
    info[i].label = (int32_t)tp[i * 8 + 3];
    info[i].group = (int32_t)tp[i * 8 + 4];
    info[i].flags = (int32_t)tp[i * 8 + 5];
    info[i].bias_row = (int32_t)tp[i * 8 + 6];
    info[i].gscale = gs.data_ptr<float>()[i];
    info[i].pad = 0;
    cp[i] = (int)blocks;
    blocks += (info[i].len + chunk - 1) / chunk;
  }
  TORCH_CHECK(blocks < (1ll << 31), "optim table: too many blocks");
  cp[S] = (int)blocks;
  auto dev = torch::Device(torch::kCUDA, (int)device_index);
  return {host.to(dev), cs.to(dev)};
}

// peer tables: int64 CUDA tensors of device pointers, one per rank (own rank included)
static std::pair<void* const*, int> peer_table(const c10::optional<torch::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return {nullptr, 0};
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kLong && t->is_contiguous(), "peer table: int64 CUDA tensor");
  return {reinterpret_cast<void* const*>(t->data_ptr<int64_t>()), (int)t->numel()};
}

void optim_prepare(torch::Tensor segs, torch::Tensor cstart, int64_t nblocks, torch::Tensor grad_shard,
                   torch::Tensor master, double inv, torch::Tensor red, torch::Tensor flags,
                   c10::optional<torch::Tensor> grad_peers, int64_t lo) {
  TORCH_CHECK(red.scalar_type() == at::kDouble && flags.scalar_type() == at::kInt, "optim_prepare: red f64, flags i32");
  TORCH_CHECK(grad_shard.scalar_type() == at::kFloat || grad_shard.scalar_type() == at::kBFloat16,
              "optim_prepare: fp32 or bf16 gradients");
  auto pt = peer_table(grad_peers);
  TORCH_CHECK(pt.second == 0 || grad_shard.scalar_type() == at::kFloat, "optim_prepare: peer gradients are fp32");
  ahb_optim_prepare(reinterpret_cast<const AhbSegInfo*>(segs.data_ptr<uint8_t>()), cstart.data_ptr<int>(),
                    (int)(cstart.numel() - 1), (int)nblocks, grad_shard.data_ptr(),
                    grad_shard.scalar_type() == at::kBFloat16, master.data_ptr<float>(),
                    (float)inv, red.data_ptr<double>(), flags.data_ptr<int>(),
                    reinterpret_cast<const float* const*>(pt.first), pt.second, lo, cur_stream());
  check_launch("ahb_optim_prepare");
}

void optim_apply(torch::Tensor segs, torch::Tensor cstart, int64_t nblocks, torch::Tensor master, torch::Tensor m,
                 torch::Tensor v, torch::Tensor grad_shard, torch::Tensor coef, torch::Tensor compute,
                 c10::optional<torch::Tensor> frac, std::vector<double> lr, std::vector<double> wd, double bc1,
                 double bc2, c10::optional<torch::Tensor> compute_peers) {
  TORCH_CHECK(lr.size() == 5 && wd.size() == 5, "optim_apply: 5 labels");
  TORCH_CHECK(grad_shard.scalar_type() == at::kFloat || grad_shard.scalar_type() == at::kBFloat16,
              "optim_apply: fp32 or bf16 gradients");
  AhbOptimArgs a;
  for (int i = 0; i < 5; ++i) { a.lr[i] = (float)lr[i]; a.wd[i] = (float)wd[i]; }
  a.bc1 = (float)bc1;
  a.bc2 = (float)bc2;
  const float* fp = nullptr;
  int fe = 0;
  torch::Tensor fc;
  if (frac.has_value() && frac->defined()) {
    fc = frac->to(at::kFloat).contiguous();
    fp = fc.data_ptr<float>();
    fe = (int)fc.size(-1);
  }
  ahb_optim_apply(reinterpret_cast<const AhbSegInfo*>(segs.data_ptr<uint8_t>()), cstart.data_ptr<int>(),
                  (int)(cstart.numel() - 1), (int)nblocks, master.data_ptr<float>(), m.data_ptr<float>(),
                  v.data_ptr<float>(), grad_shard.data_ptr(), grad_shard.scalar_type() == at::kBFloat16,
                  coef.data_ptr<float>(), compute.data_ptr(), fp, fe,
                  a, peer_table(compute_peers).first, peer_table(compute_peers).second, cur_stream());
  check_launch("ahb_optim_apply");
}

// Muon's Newton-Schulz iteration (reference optimizer.py:53-77) in place on X (E, r, c), fp32, each
// matrix already divided by its norm, r <= c.  Per step: G_e = X_e X_e^T for all E matrices in one
// grouped tcgen05 GEMM (B read K-major), Y_e = G_e X_e in a second (B read row-major), then the fused
// update.  The GEMM operands are bf16 images of X with fp32 accumulation in TMEM; X stays fp32.
void muon_ns(torch::Tensor X, int64_t steps) {
  TORCH_CHECK(X.is_cuda() && X.scalar_type() == at::kFloat && X.is_contiguous() && X.dim() == 3,
              "muon_ns: X must be a contiguous (E, r, c) fp32 CUDA tensor");
  const int64_t E = X.size(0), r = X.size(1), c = X.size(2);
  TORCH_CHECK(E >= 1 && E <= 192 && r <= c && r % 128 == 0 && c % 64 == 0,
              "muon_ns: 1..192 matrices of r x c with r <= c, r % 128 == 0, c % 64 == 0");
  const bool pair = moe_pair() && r % 256 == 0;  // CTA-pair groups start on 256-row boundaries
  const int PM = pair ? AHB_GEMM_PAIR : 0;
  auto ob = X.options().dtype(at::kBFloat16);
  auto Xb = torch::empty({E * r, c}, ob);
  auto G = torch::empty({E * r, r}, ob);
  auto Y = torch::empty({E * r, c}, ob);
  auto off = torch::arange(0, E * r + 1, r, torch::dtype(torch::kInt32).device(X.device()));
  int* err = err_word().data_ptr<int>();
  auto st = cur_stream();
  ahb_ns_update(X.data_ptr<float>(), nullptr, Xb.data_ptr(), X.numel(), num_sms(), st);
  check_launch("ahb_ns_update");
  for (int64_t s = 0; s < steps; ++s) {
    int rc = ahb_moe_gemm(AHB_GEMM_DX | PM, Xb.data_ptr(), nullptr, E * r, c, Xb.data_ptr(), nullptr, E * r, c, (int)r,
                          off.data_ptr<int>(), (int)E, (int)r, 0, (int)c, (int)(c / 64), G.data_ptr(), nullptr,
                          nullptr, nullptr, nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "muon X X^T");
    rc = ahb_moe_gemm(AHB_GEMM_FWD_DOWN | PM, G.data_ptr(), nullptr, E * r, r, Xb.data_ptr(), nullptr, E * r, c,
                      (int)r, off.data_ptr<int>(), (int)E, (int)c, 0, (int)r, (int)(r / 64), Y.data_ptr(), nullptr,
                      nullptr, nullptr, nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "muon G X");
    ahb_ns_update(X.data_ptr<float>(), Y.data_ptr(), Xb.data_ptr(), X.numel(), num_sms(), st);
    check_launch("ahb_ns_update");
  }
}

// The same iteration on tall matrices (E >= 2 of a x b, a > b) without transposing them: the Gram
// matrix G_e = X_e^T X_e (b x b) comes from the K-grouped GEMM (groups of a rows, summed into zeroed
// bf16 accumulators) and Y_e = X_e G_e from the M-grouped GEMM that reads B row-major.
void muon_ns_tall(torch::Tensor X, int64_t steps) {
  TORCH_CHECK(X.is_cuda() && X.scalar_type() == at::kFloat && X.is_contiguous() && X.dim() == 3,
              "muon_ns_tall: X must be a contiguous (E, a, b) fp32 CUDA tensor");
  const int64_t E = X.size(0), a = X.size(1), b = X.size(2);
  TORCH_CHECK(E >= 2 && E <= 192 && a > b && a % 128 == 0 && b % 128 == 0,
              "muon_ns_tall: 2..192 matrices of a x b with a > b, a % 128 == 0, b % 128 == 0");
  const int PM = moe_pair() && a % 256 == 0 ? AHB_GEMM_PAIR : 0;  // row groups start on 256-row boundaries
  const int PW = moe_pair() && b % 256 == 0 ? AHB_GEMM_PAIR : 0;  // Gram rows a multiple of 256
  auto ob = X.options().dtype(at::kBFloat16);
  auto Xb = torch::empty({E * a, b}, ob);
  auto G = torch::empty({E * b, b}, ob);
  auto Y = torch::empty({E * a, b}, ob);
  auto off = torch::arange(0, E * a + 1, a, torch::dtype(torch::kInt32).device(X.device()));
  int* err = err_word().data_ptr<int>();
  auto st = cur_stream();
  ahb_ns_update(X.data_ptr<float>(), nullptr, Xb.data_ptr(), X.numel(), num_sms(), st);
  check_launch("ahb_ns_update");
  for (int64_t s = 0; s < steps; ++s) {
    G.zero_();
    int rc = ahb_moe_gemm(AHB_GEMM_WGRAD | AHB_GEMM_ACC_BF16 | PW, Xb.data_ptr(), nullptr, E * a, b, Xb.data_ptr(),
                          nullptr, E * a, b, 0, off.data_ptr<int>(), (int)E, (int)b, (int)b, 0, 0, G.data_ptr(),
                          nullptr, nullptr, nullptr, nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "muon X^T X");
    rc = ahb_moe_gemm(AHB_GEMM_FWD_DOWN | PM, Xb.data_ptr(), nullptr, E * a, b, G.data_ptr(), nullptr, E * b, b,
                      (int)b, off.data_ptr<int>(), (int)E, (int)b, 0, (int)b, (int)(b / 64), Y.data_ptr(), nullptr,
                      nullptr, nullptr, nullptr, 0.f, err, num_sms(), st);
    gemm_check(rc, "muon X G");
    ahb_ns_update(X.data_ptr<float>(), Y.data_ptr(), Xb.data_ptr(), X.numel(), num_sms(), st);
    check_launch("ahb_ns_update");
  }
}

// ------------------------------------------------------------ fused layer glue (fused_norm.cu)
static void check_rows(const torch::Tensor& t, int64_t D, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.size(-1) == D, n,
              ": contiguous bf16 CUDA tensor with last dim ", D);
}

static void add_scale_grad(const torch::Tensor& part, const c10::optional<torch::Tensor>& acc, int64_t D) {
  if (!acc.has_value() || !acc->defined()) return;
  check_acc(*acc, D, "dscale_acc");
  ahb_colsum_add(part.data_ptr<float>(), (int)part.size(0), (int)D, acc->data_ptr<float>(), cur_stream());
  check_launch("ahb_colsum_add");
}

std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor delta, torch::Tensor scale, double clip,
                                           double eps, c10::optional<torch::Tensor> stats) {
  const int64_t D = x.size(-1);
  TORCH_CHECK(ahb_row_supported((int)D), "add_rmsnorm: D % 256 != 0");
  check_rows(x, D, "x");
  check_rows(delta, D, "delta");
  TORCH_CHECK(delta.numel() == x.numel(), "add_rmsnorm: shape mismatch");
  const int64_t M = x.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  auto xo = torch::empty_like(x), y = torch::empty_like(x);
  auto r = torch::empty({M}, x.options().dtype(at::kFloat));
  float* sp = nullptr;
  if (stats.has_value() && stats->defined()) {
    TORCH_CHECK(stats->is_cuda() && stats->scalar_type() == at::kFloat && stats->is_contiguous() && stats->numel() >= 2,
                "add_rmsnorm: stats fp32 (2,)");
    sp = stats->data_ptr<float>();
  }
  ahb_add_rmsnorm_fwd(x.data_ptr(), delta.data_ptr(), sc.data_ptr<float>(), xo.data_ptr(), y.data_ptr(),
                      r.data_ptr<float>(), M, (int)D, (float)clip, (float)eps, cur_stream(), sp);
  check_launch("ahb_add_rmsnorm_fwd");
  return {xo, y, r};
}

std::vector<torch::Tensor> add_rmsnorm_bwd(torch::Tensor dy, c10::optional<torch::Tensor> gres, torch::Tensor xo,
                                           torch::Tensor scale, torch::Tensor rstd, double clip, bool want_ddelta,
                                           c10::optional<torch::Tensor> dscale_acc) {
  const int64_t D = xo.size(-1);
  check_rows(xo, D, "xo");
  auto dyc = dy.contiguous();
  check_rows(dyc, D, "dy");
  torch::Tensor gr;
  if (gres.has_value() && gres->defined()) {
    gr = gres->contiguous();
    check_rows(gr, D, "gres");
  }
  const int64_t M = xo.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  auto dx = torch::empty_like(xo);
  torch::Tensor dd = want_ddelta ? torch::empty_like(xo) : torch::Tensor();
  const bool wacc = dscale_acc.has_value() && dscale_acc->defined();
  torch::Tensor part;
  if (wacc) part = torch::empty({(int64_t)ahb_row_bwd_blocks(M), D}, xo.options().dtype(at::kFloat));
  ahb_add_rmsnorm_bwd(dyc.data_ptr(), gr.defined() ? gr.data_ptr() : nullptr, xo.data_ptr(), sc.data_ptr<float>(),
                      rstd.data_ptr<float>(), dx.data_ptr(), dd.defined() ? dd.data_ptr() : nullptr,
                      wacc ? part.data_ptr<float>() : nullptr, M, (int)D, (float)clip, cur_stream());
  check_launch("ahb_add_rmsnorm_bwd");
  if (wacc) add_scale_grad(part, dscale_acc, D);
  return {dx, dd.defined() ? dd : dx};
}

std::vector<torch::Tensor> norm_gate_fwd(torch::Tensor x, torch::Tensor z, torch::Tensor scale, double eps,
                                         double zclip, double oclip) {
  const int64_t D = x.size(-1);
  TORCH_CHECK(ahb_row_supported((int)D), "norm_gate: D % 256 != 0");
  check_rows(x, D, "x");
  TORCH_CHECK(z.is_cuda() && z.scalar_type() == at::kBFloat16 && z.stride(-1) == 1 && z.size(-1) == D &&
                  z.numel() == x.numel() && z.dim() >= 2, "norm_gate: z bf16 with unit channel stride");
  const int64_t zs = z.stride(-2);
  for (int i = 0; i < z.dim() - 2; ++i)
    TORCH_CHECK(z.stride(i) == z.size(i + 1) * z.stride(i + 1), "norm_gate: z rows must be evenly strided");
  TORCH_CHECK(zs % 8 == 0, "norm_gate: z row stride must be a multiple of 8");
  const int64_t M = x.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  auto y = torch::empty_like(x);
  auto r = torch::empty({M}, x.options().dtype(at::kFloat));
  ahb_norm_gate_fwd(x.data_ptr(), z.data_ptr(), zs, sc.data_ptr<float>(), y.data_ptr(), r.data_ptr<float>(), M,
                    (int)D, (float)eps, (float)zclip, (float)oclip, cur_stream());
  check_launch("ahb_norm_gate_fwd");
  return {y, r};
}

std::vector<torch::Tensor> norm_gate_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor z, torch::Tensor scale,
                                         torch::Tensor rstd, double zclip, double oclip,
                                         c10::optional<torch::Tensor> dscale_acc) {
  const int64_t D = x.size(-1);
  check_rows(x, D, "x");
  auto dyc = dy.contiguous();
  check_rows(dyc, D, "dy");
  const int64_t zs = z.stride(-2);
  const int64_t M = x.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  auto dx = torch::empty_like(x);
  auto dz = torch::empty_like(x);
  const bool wacc = dscale_acc.has_value() && dscale_acc->defined();
  torch::Tensor part;
  if (wacc) part = torch::empty({(int64_t)ahb_row_bwd_blocks(M), D}, x.options().dtype(at::kFloat));
  ahb_norm_gate_bwd(dyc.data_ptr(), x.data_ptr(), z.data_ptr(), zs, sc.data_ptr<float>(), rstd.data_ptr<float>(),
                    dx.data_ptr(), dz.data_ptr(), wacc ? part.data_ptr<float>() : nullptr, M, (int)D, (float)zclip,
                    (float)oclip, cur_stream());
  check_launch("ahb_norm_gate_bwd");
  if (wacc) add_scale_grad(part, dscale_acc, D);
  return {dx, dz};
}

// Shared-expert SwiGLU gate: h = silu(a) * b (bf16, contiguous, equal shapes) and its backward
static void check_swiglu(const torch::Tensor& t, const torch::Tensor& ref, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.sizes() == ref.sizes() &&
                  t.numel() % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "swiglu: ", n, " must be a contiguous 16-byte-aligned bf16 CUDA tensor shaped like a (numel % 8 == 0)");
}

torch::Tensor swiglu_fwd(torch::Tensor a, torch::Tensor b) {
  check_swiglu(a, a, "a");
  check_swiglu(b, a, "b");
  auto h = torch::empty_like(a);
  ahb_swiglu_fwd(a.data_ptr(), b.data_ptr(), h.data_ptr(), a.numel(), cur_stream());
  check_launch("ahb_swiglu_fwd");
  return h;
}

std::vector<torch::Tensor> swiglu_bwd(torch::Tensor dh, torch::Tensor a, torch::Tensor b) {
  auto dhc = dh.contiguous();
  check_swiglu(a, a, "a");
  check_swiglu(b, a, "b");
  check_swiglu(dhc, a, "dh");
  auto da = torch::empty_like(a), db = torch::empty_like(b);
  ahb_swiglu_bwd(dhc.data_ptr(), a.data_ptr(), b.data_ptr(), da.data_ptr(), db.data_ptr(), a.numel(), cur_stream());
  check_launch("ahb_swiglu_bwd");
  return {da, db};
}

// Tensor-parallel (head-split) RMSNorm, gated by z when given (ops.kernels.tp_norm): x (..., D) holds D
// of the row's Dfull channels; the caller all-reduces the row sums (ss, dot) over the group between
// the passes.
static int64_t tp_z_stride(const c10::optional<torch::Tensor>& z, const torch::Tensor& x, int64_t D) {
  if (!z.has_value() || !z->defined()) return 0;
  TORCH_CHECK(z->is_cuda() && z->scalar_type() == at::kBFloat16 && z->stride(-1) == 1 && z->size(-1) == D &&
                  z->numel() == x.numel() && z->dim() >= 2, "tp_norm: z bf16 with unit channel stride");
  for (int i = 0; i < z->dim() - 2; ++i)
    TORCH_CHECK(z->stride(i) == z->size(i + 1) * z->stride(i + 1), "tp_norm: z rows must be evenly strided");
  TORCH_CHECK(z->stride(-2) % 8 == 0, "tp_norm: z row stride must be a multiple of 8");
  return z->stride(-2);
}

static const void* opt_any(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr() : nullptr;
}

torch::Tensor tp_norm_sumsq(torch::Tensor x) {
  const int64_t D = x.size(-1);
  TORCH_CHECK(ahb_row_supported((int)D), "tp_norm: D % 256 != 0");
  check_rows(x, D, "x");
  const int64_t M = x.numel() / D;
  auto ss = torch::empty({M}, x.options().dtype(at::kFloat));
  ahb_tp_norm_sumsq(x.data_ptr(), ss.data_ptr<float>(), M, (int)D, cur_stream());
  check_launch("ahb_tp_norm_sumsq");
  return ss;
}

std::vector<torch::Tensor> tp_norm_fwd(torch::Tensor x, c10::optional<torch::Tensor> z, torch::Tensor scale,
                                       torch::Tensor ss, double eps, double inv_dfull, double zclip, double oclip) {
  const int64_t D = x.size(-1);
  TORCH_CHECK(ahb_row_supported((int)D), "tp_norm: D % 256 != 0");
  check_rows(x, D, "x");
  const int64_t zs = tp_z_stride(z, x, D);
  const int64_t M = x.numel() / D;
  TORCH_CHECK(ss.is_cuda() && ss.scalar_type() == at::kFloat && ss.is_contiguous() && ss.numel() == M,
              "tp_norm: ss (rows,) fp32");
  auto sc = scale.to(at::kFloat).contiguous();
  TORCH_CHECK(sc.numel() == D, "tp_norm: scale of D channels");
  auto y = torch::empty_like(x);
  auto r = torch::empty({M}, x.options().dtype(at::kFloat));
  ahb_tp_norm_fwd(x.data_ptr(), opt_any(z), zs, sc.data_ptr<float>(), ss.data_ptr<float>(), y.data_ptr(),
                  r.data_ptr<float>(), M, (int)D, (float)inv_dfull, (float)eps, (float)zclip, (float)oclip,
                  cur_stream());
  check_launch("ahb_tp_norm_fwd");
  return {y, r};
}

// returns {dz (empty without a gate), local dot}; the scale gradient is added into dscale_acc
std::vector<torch::Tensor> tp_norm_bwd_dot(torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> z,
                                           torch::Tensor scale, torch::Tensor rstd, double zclip, double oclip,
                                           c10::optional<torch::Tensor> dscale_acc) {
  const int64_t D = x.size(-1);
  check_rows(x, D, "x");
  check_rows(dy, D, "dy");
  const int64_t zs = tp_z_stride(z, x, D);
  const int64_t M = x.numel() / D;
  auto sc = scale.to(at::kFloat).contiguous();
  const bool gated = opt_any(z) != nullptr;
  auto dz = gated ? torch::empty_like(x) : torch::empty({0}, x.options());
  auto dot = torch::empty({M}, x.options().dtype(at::kFloat));
  const bool wacc = dscale_acc.has_value() && dscale_acc->defined();
  torch::Tensor part;
  if (wacc) part = torch::empty({(int64_t)ahb_row_bwd_blocks(M), D}, x.options().dtype(at::kFloat));
  ahb_tp_norm_bwd_dot(dy.data_ptr(), x.data_ptr(), opt_any(z), zs, sc.data_ptr<float>(), rstd.data_ptr<float>(),
                      gated ? dz.data_ptr() : nullptr, dot.data_ptr<float>(), wacc ? part.data_ptr<float>() : nullptr,
                      M, (int)D, (float)zclip, (float)oclip, cur_stream());
  check_launch("ahb_tp_norm_bwd_dot");
  if (wacc) add_scale_grad(part, dscale_acc, D);
  return {dz, dot};
}

torch::Tensor tp_norm_bwd_dx(torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> z, torch::Tensor scale,
                             torch::Tensor rstd, torch::Tensor dot, double inv_dfull, double zclip, double oclip) {
  const int64_t D = x.size(-1);
  check_rows(x, D, "x");
  check_rows(dy, D, "dy");
  const int64_t zs = tp_z_stride(z, x, D);
  const int64_t M = x.numel() / D;
  TORCH_CHECK(dot.is_cuda() && dot.scalar_type() == at::kFloat && dot.is_contiguous() && dot.numel() == M,
              "tp_norm: dot (rows,) fp32");
  auto sc = scale.to(at::kFloat).contiguous();
  auto dx = torch::empty_like(x);
  ahb_tp_norm_bwd_dx(dy.data_ptr(), x.data_ptr(), opt_any(z), zs, sc.data_ptr<float>(), rstd.data_ptr<float>(),
                     dot.data_ptr<float>(), dx.data_ptr(), M, (int)D, (float)inv_dfull, (float)zclip, (float)oclip,
                     cur_stream());
  check_launch("ahb_tp_norm_bwd_dx");
  return dx;
}

std::vector<torch::Tensor> gdn_gates_fwd(torch::Tensor bp, torch::Tensor wp, torch::Tensor fp, torch::Tensor decay_a,
                                         int64_t Dh) {
  const int64_t d = bp.size(-1);
  for (auto* t : {&bp, &wp, &fp}) check_rows(*t, d, "gate input");
  TORCH_CHECK(wp.numel() == bp.numel() && fp.numel() == bp.numel() && d % Dh == 0 && Dh % 8 == 0,
              "gdn_gates: shapes");
  auto a = decay_a.to(at::kFloat).contiguous();
  TORCH_CHECK(a.numel() == d / Dh, "gdn_gates: decay_a must have d/Dh entries");
  auto bg = torch::empty_like(bp), wg = torch::empty_like(bp);
  auto g = torch::empty(bp.sizes(), bp.options().dtype(at::kFloat));
  ahb_gdn_gates_fwd(bp.data_ptr(), wp.data_ptr(), fp.data_ptr(), a.data_ptr<float>(), bg.data_ptr(), wg.data_ptr(),
                    g.data_ptr<float>(), bp.numel(), (int)d, (int)Dh, cur_stream());
  check_launch("ahb_gdn_gates_fwd");
  return {bg, wg, g};
}

std::vector<torch::Tensor> gdn_gates_bwd(torch::Tensor dbg, torch::Tensor dwg, torch::Tensor dg, torch::Tensor bg,
                                         torch::Tensor wg, torch::Tensor fp, torch::Tensor decay_a, int64_t Dh,
                                         c10::optional<torch::Tensor> da_acc) {
  const int64_t d = bg.size(-1);
  auto dbc = dbg.to(at::kBFloat16).contiguous(), dwc = dwg.to(at::kBFloat16).contiguous();
  auto dgc = dg.to(at::kFloat).contiguous();
  for (auto* t : {&dbc, &dwc, &bg, &wg, &fp}) check_rows(*t, d, "gate tensor");
  auto a = decay_a.to(at::kFloat).contiguous();
  torch::Tensor acc;
  if (da_acc.has_value() && da_acc->defined()) {
    check_acc(*da_acc, d / Dh, "da_acc");
    acc = *da_acc;
  } else {
    acc = torch::zeros({d / Dh}, bg.options().dtype(at::kFloat));
  }
  auto dbp = torch::empty_like(bg), dwp = torch::empty_like(bg), dfp = torch::empty_like(bg);
  ahb_gdn_gates_bwd(dbc.data_ptr(), dwc.data_ptr(), dgc.data_ptr<float>(), bg.data_ptr(), wg.data_ptr(),
                    fp.data_ptr(), a.data_ptr<float>(), dbp.data_ptr(), dwp.data_ptr(), dfp.data_ptr(),
                    acc.data_ptr<float>(), bg.numel(), (int)d, (int)Dh, cur_stream());
  check_launch("ahb_gdn_gates_bwd");
  return {dbp, dwp, dfp, acc};
}

std::vector<torch::Tensor> l2norm_heads_fwd(torch::Tensor x) {
  TORCH_CHECK(x.size(-1) == 128, "l2norm_heads: head dim 128");
  check_rows(x, 128, "x");
  const int64_t nh = x.numel() / 128;
  auto y = torch::empty_like(x);
  auto rn = torch::empty({nh}, x.options().dtype(at::kFloat));
  ahb_l2norm_heads_fwd(x.data_ptr(), y.data_ptr(), rn.data_ptr<float>(), nh, cur_stream());
  check_launch("ahb_l2norm_heads_fwd");
  return {y, rn};
}

torch::Tensor l2norm_heads_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor rn) {
  auto dyc = dy.to(at::kBFloat16).contiguous();
  check_rows(dyc, 128, "dy");
  check_rows(x, 128, "x");
  auto dx = torch::empty_like(x);
  ahb_l2norm_heads_bwd(dyc.data_ptr(), x.data_ptr(), rn.data_ptr<float>(), dx.data_ptr(), x.numel() / 128,
                       cur_stream());
  check_launch("ahb_l2norm_heads_bwd");
  return dx;
}

torch::Tensor dt_act_fwd(torch::Tensor u) {
  TORCH_CHECK(u.is_cuda() && u.scalar_type() == at::kBFloat16 && u.is_contiguous() && u.numel() % 8 == 0,
              "dt_act: contiguous bf16, numel % 8 == 0");
  auto dt = torch::empty_like(u);
  ahb_dt_act_fwd(u.data_ptr(), dt.data_ptr(), u.numel(), cur_stream());
  check_launch("ahb_dt_act_fwd");
  return dt;
}

torch::Tensor dt_act_bwd(torch::Tensor ddt, torch::Tensor u) {
  auto dc = ddt.to(at::kBFloat16).contiguous();
  TORCH_CHECK(dc.numel() == u.numel() && u.is_contiguous(), "dt_act_bwd: shapes");
  auto du = torch::empty_like(u);
  ahb_dt_act_bwd(dc.data_ptr(), u.data_ptr(), du.data_ptr(), u.numel(), cur_stream());
  check_launch("ahb_dt_act_bwd");
  return du;
}

// ------------------------------------------------------------ fused MoE router (router.cu)
bool router_supported(int64_t d, int64_t E, int64_t k) { return ahb_router_supported((int)d, (int)E, (int)k) != 0; }

// kn (d, E) fp32 -> zero-padded bf16 terms hi (+ mid (+ lo)) whose sum is kn;
// transposed: (terms, EP, d), else (terms, d, EP)
static torch::Tensor router_split(const torch::Tensor& kn, int terms, bool transposed) {
  const int64_t d = kn.size(0), E = kn.size(1), EP = ahb_router_padded_experts((int)E);
  auto knp = torch::zeros({d, EP}, kn.options());
  knp.narrow(1, 0, E).copy_(kn);
  std::vector<torch::Tensor> parts;
  auto rem = knp;
  for (int i = 0; i < terms; ++i) {
    auto h = rem.to(at::kBFloat16);
    parts.push_back(transposed ? h.t() : h);
    rem = rem - h.to(at::kFloat);
  }
  return torch::stack(parts).contiguous();
}

std::vector<torch::Tensor> router_fwd(torch::Tensor x, torch::Tensor kn, torch::Tensor temp, torch::Tensor bias,
                                      c10::optional<torch::Tensor> noise, int64_t k) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2,
              "router: x (T, d) contiguous bf16");
  const int64_t T = x.size(0), d = x.size(1);
  auto knc = kn.to(at::kFloat).contiguous();
  TORCH_CHECK(knc.dim() == 2 && knc.size(0) == d, "router: kn (d, E)");
  const int64_t E = knc.size(1);
  TORCH_CHECK(ahb_router_supported((int)d, (int)E, (int)k), "router: unsupported d / E / k");
  auto knT3 = router_split(knc, 3, true);
  auto tc = temp.to(at::kFloat).contiguous();
  auto bc = bias.to(at::kFloat).contiguous();
  torch::Tensor nz;
  if (noise.has_value() && noise->defined()) {
    nz = noise->to(at::kFloat).contiguous();
    TORCH_CHECK(nz.numel() == T * E, "router: noise (T, E)");
  }
  auto f32 = x.options().dtype(at::kFloat);
  auto logits = torch::empty({T, E}, f32), cosv = torch::empty({T, E}, f32);
  auto rn = torch::empty({T}, f32);
  auto top = torch::empty({T, k}, x.options().dtype(at::kLong));
  auto gate = torch::empty({T, k}, f32);
  auto psum = torch::zeros({E}, f32), counts = torch::zeros({E}, f32);
  // [sum lse^2, max |pre|, sum |x|, max |x|, min |x| (starts at the largest finite float)]
  auto scal = torch::arange(0, 5, f32).mul_(0).add_(torch::arange(0, 5, f32).eq(4).to(at::kFloat).mul_(3.0e38));
  ahb_router_fwd(x.data_ptr(), knT3.data_ptr(), tc.data_ptr<float>(), bc.data_ptr<float>(),
                 nz.defined() ? nz.data_ptr<float>() : nullptr, T, (int)d, (int)E, (int)k, logits.data_ptr<float>(),
                 cosv.data_ptr<float>(), rn.data_ptr<float>(), top.data_ptr<int64_t>(), gate.data_ptr<float>(),
                 psum.data_ptr<float>(), scal.data_ptr<float>(), counts.data_ptr<float>(), cur_stream());
  check_launch("ahb_router_fwd");
  return {logits, cosv, rn, top, gate, psum, scal, counts};
}

std::vector<torch::Tensor> router_bwd(torch::Tensor x, torch::Tensor kn, torch::Tensor temp, torch::Tensor logits,
                                      torch::Tensor cosv, torch::Tensor rn, torch::Tensor top, torch::Tensor gate,
                                      torch::Tensor dgate, torch::Tensor dps, c10::optional<torch::Tensor> dlse_sq) {
  const int64_t T = x.size(0), d = x.size(1), E = logits.size(1), k = top.size(1);
  auto knc = kn.to(at::kFloat).contiguous();
  auto tc = temp.to(at::kFloat).contiguous();
  auto dg = dgate.to(at::kFloat).contiguous();
  auto dp = dps.to(at::kFloat).contiguous();
  torch::Tensor dl;
  if (dlse_sq.has_value() && dlse_sq->defined()) dl = dlse_sq->to(at::kFloat).contiguous();
  auto f32 = x.options().dtype(at::kFloat);
  auto kn2 = router_split(knc, 2, false);
  auto dcos = torch::empty({T, (int64_t)ahb_router_padded_experts((int)E)}, f32);
  auto dtemp = torch::zeros({1}, f32);
  auto dkn = torch::zeros({d, E}, f32);
  auto dx = torch::empty_like(x);
  ahb_router_bwd(x.data_ptr(), kn2.data_ptr(), tc.data_ptr<float>(), logits.data_ptr<float>(),
                 cosv.data_ptr<float>(), rn.data_ptr<float>(), top.data_ptr<int64_t>(), gate.data_ptr<float>(),
                 dg.data_ptr<float>(), dp.data_ptr<float>(), dl.defined() ? dl.data_ptr<float>() : nullptr, T, (int)d,
                 (int)E, (int)k, dcos.data_ptr<float>(), dtemp.data_ptr<float>(), dx.data_ptr(),
                 dkn.data_ptr<float>(), cur_stream());
  check_launch("ahb_router_bwd");
  return {dx, dkn, dtemp};
}

// ------------------------------------------------------------ causal flash attention (attention.cu)
static void check_attn(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.dim() == 4, n,
              ": contiguous bf16 (B, H, L, D)");
}

std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale) {
  for (auto* t : {&q, &k, &v}) check_attn(*t, "attention");
  const int64_t B = q.size(0), H = q.size(1), L = q.size(2), D = q.size(3);
  TORCH_CHECK(k.sizes() == q.sizes() && v.sizes() == q.sizes() && ahb_attn_supported((int)D), "attention: shapes / D");
  auto o = torch::empty_like(q);
  auto lse = torch::empty({B, H, L}, q.options().dtype(at::kFloat));
  TORCH_CHECK(ahb_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), (int)(B * H), (int)L, (int)D, (float)scale,
                           o.data_ptr(), lse.data_ptr<float>(), cur_stream()) == 0, "attention: setup failed");
  check_launch("ahb_attn_fwd");
  return {o, lse};
}

std::vector<torch::Tensor> attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                                    torch::Tensor dout, torch::Tensor lse, double scale) {
  auto doc = dout.to(at::kBFloat16).contiguous();
  for (auto* t : {&q, &k, &v, &o, &doc}) check_attn(*t, "attention bwd");
  const int64_t B = q.size(0), H = q.size(1), L = q.size(2), D = q.size(3);
  auto delta = (doc.to(at::kFloat) * o.to(at::kFloat)).sum(-1).contiguous();
  auto dq = torch::zeros(q.sizes(), q.options().dtype(at::kFloat));
  auto dk = torch::empty_like(k), dv = torch::empty_like(v);
  TORCH_CHECK(ahb_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), doc.data_ptr(), lse.data_ptr<float>(),
                           delta.data_ptr<float>(), (int)(B * H), (int)L, (int)D, (float)scale, dq.data_ptr<float>(),
                           dk.data_ptr(), dv.data_ptr(), cur_stream()) == 0, "attention bwd: setup failed");
  check_launch("ahb_attn_bwd");
  return {dq.to(at::kBFloat16), dk, dv};
}

// ------------------------------------------------------------ BlockDAR source softmax (source_mix.cu)
static torch::Tensor ptr_table(const std::vector<torch::Tensor>& ts, int64_t numel, const torch::Device& dev,
                               const char* what) {
  std::vector<int64_t> p;
  for (const auto& t : ts) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.numel() == numel, what,
                ": contiguous bf16 tensors of equal size");
    p.push_back(reinterpret_cast<int64_t>(t.data_ptr()));
  }
  return torch::tensor(p, torch::kInt64).to(dev);
}

std::vector<torch::Tensor> source_mix_fwd(torch::Tensor q, std::vector<torch::Tensor> ks, std::vector<torch::Tensor> ss,
                                          double scale) {
  const int n = (int)ks.size();
  TORCH_CHECK(n >= 1 && n <= ahb_source_mix_max() && (int)ss.size() == n, "source_mix: 1..32 sources");
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous(), "source_mix: q bf16");
  const int64_t dl = q.size(-1), T = q.numel() / dl, d = ss[0].size(-1);
  auto kt = ptr_table(ks, T * dl, q.device(), "keys");
  auto st_ = ptr_table(ss, T * d, q.device(), "sources");
  auto out = torch::empty_like(ss[0]);
  auto wts = torch::empty({n, T}, q.options().dtype(at::kFloat));
  ahb_source_mix_fwd(q.data_ptr(), reinterpret_cast<const void* const*>(kt.data_ptr<int64_t>()),
                     reinterpret_cast<const void* const*>(st_.data_ptr<int64_t>()), n, T, (int)dl, (int)d,
                     (float)scale, out.data_ptr(), wts.data_ptr<float>(), cur_stream());
  check_launch("ahb_source_mix_fwd");
  return {out, wts};
}

// returns [dq, dk_0..dk_{n-1}, ds_0..ds_{n-1}]
std::vector<torch::Tensor> source_mix_bwd(torch::Tensor g, torch::Tensor q, std::vector<torch::Tensor> ks,
                                          std::vector<torch::Tensor> ss, torch::Tensor wts, double scale) {
  const int n = (int)ks.size();
  const int64_t dl = q.size(-1), T = q.numel() / dl, d = ss[0].size(-1);
  auto gc = g.to(at::kBFloat16).contiguous();
  auto kt = ptr_table(ks, T * dl, q.device(), "keys");
  auto st_ = ptr_table(ss, T * d, q.device(), "sources");
  std::vector<torch::Tensor> out{torch::empty_like(q)};
  std::vector<torch::Tensor> dks, dss;
  for (int i = 0; i < n; ++i) dks.push_back(torch::empty_like(ks[i]));
  for (int i = 0; i < n; ++i) dss.push_back(torch::empty_like(ss[i]));
  auto dkt = ptr_table(dks, T * dl, q.device(), "dk");
  auto dst = ptr_table(dss, T * d, q.device(), "ds");
  ahb_source_mix_bwd(gc.data_ptr(), q.data_ptr(), reinterpret_cast<const void* const*>(kt.data_ptr<int64_t>()),
                     reinterpret_cast<const void* const*>(st_.data_ptr<int64_t>()), wts.data_ptr<float>(), n, T,
                     (int)dl, (int)d, (float)scale, out[0].data_ptr(),
                     reinterpret_cast<void* const*>(dkt.data_ptr<int64_t>()),
                     reinterpret_cast<void* const*>(dst.data_ptr<int64_t>()), cur_stream());
  check_launch("ahb_source_mix_bwd");
  out.insert(out.end(), dks.begin(), dks.end());
  out.insert(out.end(), dss.begin(), dss.end());
  return out;
}

// ------------------------------------------------------------ NVLink peer memory (CUDA IPC)
int64_t ipc_alloc(int64_t nbytes) {
  void* p = nullptr;
  TORCH_CHECK(ahb_ipc_alloc(nbytes, &p) == 0, "ipc_alloc failed (", nbytes, " bytes)");
  return reinterpret_cast<int64_t>(p);
}
void ipc_free(int64_t ptr) { TORCH_CHECK(ahb_ipc_free(reinterpret_cast<void*>(ptr)) == 0, "ipc_free failed"); }
torch::Tensor ipc_handle(int64_t ptr) {
  auto h = torch::empty({64}, torch::kUInt8);
  TORCH_CHECK(ahb_ipc_handle(reinterpret_cast<void*>(ptr), h.data_ptr<uint8_t>()) == 0, "cudaIpcGetMemHandle failed");
  return h;
}
int64_t ipc_open(torch::Tensor handle) {
  TORCH_CHECK(handle.device().is_cpu() && handle.numel() == 64 && handle.scalar_type() == at::kByte, "ipc_open: 64 bytes");
  void* p = nullptr;
  TORCH_CHECK(ahb_ipc_open(handle.contiguous().data_ptr<uint8_t>(), &p) == 0, "cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}
void ipc_close(int64_t ptr) { TORCH_CHECK(ahb_ipc_close(reinterpret_cast<void*>(ptr)) == 0, "ipc_close failed"); }
// a tensor view of raw device memory; the caller keeps the allocation alive
torch::Tensor ipc_tensor(int64_t ptr, int64_t numel, torch::Tensor like) {
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, like.options());
}
void symm_barrier(torch::Tensor pads, int64_t rank, int64_t epoch, torch::Tensor err, double timeout_s) {
  TORCH_CHECK(pads.is_cuda() && pads.scalar_type() == at::kLong && pads.numel() <= 32, "symm_barrier: <= 32 ranks");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "symm_barrier: err int32");
  ahb_symm_barrier(reinterpret_cast<uint32_t* const*>(pads.data_ptr<int64_t>()), (int)rank, (int)pads.numel(),
                   (uint32_t)epoch, err.data_ptr<int>(), timeout_s, cur_stream());
  check_launch("ahb_symm_barrier");
}
void reduce_scatter_f32(torch::Tensor peers, int64_t lo, torch::Tensor out) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() % 4 == 0 &&
                  lo % 4 == 0, "reduce_scatter_f32: fp32 out, 16-byte aligned slice");
  auto pt = peer_table(peers);
  ahb_reduce_scatter_f32(reinterpret_cast<const float* const*>(pt.first), pt.second, lo, out.numel(),
                         out.data_ptr<float>(), cur_stream());
  check_launch("ahb_reduce_scatter_f32");
}
void copy_out(torch::Tensor src, torch::Tensor peers, int64_t off_bytes) {
  const int64_t nb = src.numel() * src.element_size();
  TORCH_CHECK(src.is_cuda() && src.is_contiguous() && nb % 16 == 0 && off_bytes % 16 == 0,
              "copy_out: 16-byte aligned slice");
  auto pt = peer_table(peers);
  ahb_copy_out(src.data_ptr(), pt.first, pt.second, off_bytes, nb, cur_stream());
  check_launch("ahb_copy_out");
}

// acc (N,) fp32 += column sums of dy (M, N) bf16: the bias gradient added into the gradient store
void bias_grad_acc(torch::Tensor dy, torch::Tensor acc) {
  TORCH_CHECK(dy.is_cuda() && dy.scalar_type() == at::kBFloat16 && dy.dim() == 2 && dy.stride(1) == 1 &&
                  dy.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(dy.data_ptr()) % 16 == 0 &&
                  dy.size(1) % 8 == 0,
              "bias_grad_acc: dy bf16 (M, N), N % 8 == 0, unit column stride, 16-byte-aligned rows");
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.numel() == dy.size(1),
              "bias_grad_acc: acc fp32 (N,)");
  ahb_bias_grad_acc(dy.data_ptr(), dy.size(0), (int)dy.size(1), dy.stride(0), acc.data_ptr<float>(), cur_stream());
  check_launch("ahb_bias_grad_acc");
}

// ------------------------------------------------------------ tensor parallelism over peer memory
// Row-parallel projection with the reduce-scatter in the epilogue: rows of group g of `a` times `b`
// are stored at out_ptrs[g] (rank g's receive slot for this rank; raw device pointers, peers' included).
void tp_gemm_rs(torch::Tensor a, torch::Tensor b, torch::Tensor grp_off, std::vector<int64_t> out_ptrs, int64_t m_rot) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.dim() == 2 && a.is_contiguous(), "tp_gemm_rs: a bf16 (M,K)");
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == at::kBFloat16 && b.dim() == 2 && b.is_contiguous() &&
                  b.size(0) == a.size(1), "tp_gemm_rs: b bf16 (K,N)");
  TORCH_CHECK(grp_off.is_cuda() && grp_off.scalar_type() == at::kInt && grp_off.numel() == (int64_t)out_ptrs.size() + 1,
              "tp_gemm_rs: grp_off int32 (W+1)");
  std::vector<void*> tab(out_ptrs.size());
  for (size_t i = 0; i < out_ptrs.size(); ++i) tab[i] = reinterpret_cast<void*>(out_ptrs[i]);
  const int rc = ahb_gemm_rs_peer(a.data_ptr(), a.size(0), a.size(1), b.data_ptr(), b.size(1), grp_off.data_ptr<int>(),
                                  (int)out_ptrs.size(), tab.data(), (int)m_rot, err_word().data_ptr<int>(), num_sms(),
                                  cur_stream());
  TORCH_CHECK(rc == 0, "ahb_gemm_rs_peer failed: ", rc);
  check_launch("ahb_gemm_rs_peer");
}
// out = sum of `nslots` bf16 slots of out.numel() elements, `stride` elements apart, from raw memory
void sum_slots(int64_t slots, int64_t nslots, int64_t stride, torch::Tensor out) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() % 8 == 0 &&
                  stride % 8 == 0, "sum_slots: bf16 out, 16-byte multiples");
  ahb_sum_slots_bf16(reinterpret_cast<const void*>(slots), (int)nslots, stride, out.numel(), out.data_ptr(), cur_stream());
  check_launch("ahb_sum_slots_bf16");
}
// cudaMemcpyAsync between raw device addresses (peer IPC mappings included) on a given stream
void memcpy_async(int64_t dst, int64_t src, int64_t nbytes, int64_t stream) {
  TORCH_CHECK(ahb_memcpy_async(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), nbytes,
                               reinterpret_cast<cudaStream_t>(stream)) == 0, "memcpy_async failed");
}

// ------------------------------------------------------------ dense projections (tcgen05 GEMM)
// y = x W (+ b) for a kernel W (in, out), its input gradient dx (+)= dy W^T and its fp32 weight
// gradient acc += x^T dy, on the grouped GEMM with one group (CTA pairs from 256 rows on).
static bool dense_pair(int64_t M) { return moe_pair() && M >= 256; }

// {0, M padded to `tile`} on the device, made once per (device, padded M) and kept: the grouped
// GEMM reads its group offsets from device memory, and a fresh tensor per call would add a
// launch to every projection (and an allocation inside captured graphs)
static torch::Tensor dense_off(int64_t M, int64_t tile, const torch::Device& dev) {
  static std::mutex mu;
  static std::map<std::pair<int, int64_t>, torch::Tensor> cache;
  const int64_t Mp = (M + tile - 1) / tile * tile;
  if (c10::cuda::currentStreamCaptureStatusMayInitCtx() != c10::cuda::CaptureStatus::None)  // a device write,
    return torch::arange(0, Mp + 1, Mp, torch::dtype(torch::kInt32).device(dev));          // no host copy
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair((int)dev.index(), Mp);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto t = torch::tensor({0, (int)Mp}, torch::dtype(torch::kInt32)).to(dev);
  cache.emplace(key, t);
  return t;
}

// 2-D bf16 with unit column stride and 16-byte-aligned rows (a column slice of wider rows is fine)
static void check_dense(const torch::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                  t.stride(0) % 8 == 0 && t.stride(0) >= t.size(1) &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "dense: ", n, " must be a 2-D bf16 CUDA tensor with unit column stride and 16-byte-aligned rows");
}

torch::Tensor dense_fwd(torch::Tensor x, torch::Tensor W, c10::optional<torch::Tensor> bias) {
  check_dense(x, "x");
  check_dense(W, "W");
  const int64_t M = x.size(0), K = x.size(1), N = W.size(1);
  TORCH_CHECK(W.size(0) == K && K % 64 == 0 && N % 32 == 0, "dense_fwd: x (M,K), W (K,N), K % 64, N % 32");
  torch::Tensor bc;
  if (bias.has_value() && bias->defined()) {
    bc = bias->to(at::kBFloat16).contiguous();
    TORCH_CHECK(bc.numel() == N, "dense_fwd: bias of N elements");
  }
  const bool pair = dense_pair(M);
  auto off = dense_off(M, pair ? 256 : 128, x.device());
  auto y = torch::empty({M, N}, x.options());
  int rc = ahb_dense_gemm(0, x.data_ptr(), x.stride(0), W.data_ptr(), W.stride(0), M, (int)K, (int)N,
                          bc.defined() ? bc.data_ptr() : nullptr, nullptr, y.data_ptr(), off.data_ptr<int>(),
                          err_word().data_ptr<int>(), num_sms(), cur_stream(), pair);
  gemm_check(rc, "dense fwd");
  return y;
}

// dx (M, in) = dy (M, out) W^T, plus dx's previous value when `accumulate`
void dense_dgrad(torch::Tensor dy, torch::Tensor W, torch::Tensor dx, bool accumulate) {
  check_dense(dy, "dy");
  check_dense(W, "W");
  check_dense(dx, "dx");
  TORCH_CHECK(dx.is_contiguous(), "dense_dgrad: dx contiguous");
  const int64_t M = dy.size(0), Nout = dy.size(1), Kin = W.size(0);
  TORCH_CHECK(W.size(1) == Nout && dx.size(0) == M && dx.size(1) == Kin && Nout % 64 == 0 && Kin % 32 == 0,
              "dense_dgrad: dy (M,out), W (in,out), dx (M,in), out % 64, in % 32");
  const bool pair = dense_pair(M);
  auto off = dense_off(M, pair ? 256 : 128, dy.device());
  int rc = ahb_dense_gemm(1, dy.data_ptr(), dy.stride(0), W.data_ptr(), W.stride(0), M, (int)Nout, (int)Kin,
                          nullptr, accumulate ? dx.data_ptr() : nullptr, dx.data_ptr(), off.data_ptr<int>(),
                          err_word().data_ptr<int>(), num_sms(), cur_stream(), pair);
  gemm_check(rc, "dense dgrad");
}

// acc (in, out) fp32 += x (M, in)^T dy (M, out)
void dense_wgrad(torch::Tensor x, torch::Tensor dy, torch::Tensor acc) {
  check_dense(x, "x");
  check_dense(dy, "dy");
  const int64_t M = x.size(0), K = x.size(1), N = dy.size(1);
  TORCH_CHECK(dy.size(0) == M && acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() &&
                  acc.numel() == K * N && K % 128 == 0 && N % 32 == 0,
              "dense_wgrad: x (M,in), dy (M,out), fp32 acc (in,out), in % 128, out % 32");
  const bool pair = moe_pair() && K % 256 == 0;
  auto off = dense_off(M, 64, x.device());
  int rc = ahb_dense_gemm(2, x.data_ptr(), x.stride(0), dy.data_ptr(), dy.stride(0), M, (int)K, (int)N, nullptr,
                          nullptr, acc.data_ptr(), off.data_ptr<int>(), err_word().data_ptr<int>(), num_sms(),
                          cur_stream(), pair);
  gemm_check(rc, "dense wgrad");
}

// ------------------------------------------------------------ fused LM head + cross entropy
// The logits h W^T exist only tile by tile inside the head GEMM.  Forward: per-(row, vocabulary
// tile) partials from the GEMM epilogue, combined per row into lse and the summed loss; returns
// {sum_loss, count, lse}.  Backward: for each chunk of at most `chunk_rows` rows the GEMM recomputes
// the logits into bf16 dlogits (chunk x V), then dh = g dlogits W and dW_acc += g dlogits^T h.
static bool ce_pair(int64_t rows) { return moe_pair() && rows >= 256; }

std::vector<torch::Tensor> ce_online_fwd(torch::Tensor h, torch::Tensor W, torch::Tensor labels, double ls) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == at::kBFloat16 && h.dim() == 2 && h.is_contiguous(),
              "ce: h contiguous bf16 (T,d)");
  TORCH_CHECK(W.scalar_type() == at::kBFloat16 && W.is_contiguous() && W.dim() == 2, "ce: W bf16 (V,d)");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == h.size(0),
              "ce: labels contiguous int64 (T,)");
  const int64_t T = h.size(0), d = h.size(1), V = W.size(0);
  TORCH_CHECK(W.size(1) == d && d % 64 == 0 && V % 64 == 0, "ce: d % 64 == 0 and V % 64 == 0");
  const bool pair = ce_pair(T);
  const int64_t tile = pair ? 256 : 128, Tp = (T + tile - 1) / tile * tile;
  const int ntiles = (int)((V + 255) / 256);
  auto f32 = h.options().dtype(at::kFloat);
  auto part = torch::empty({T, ntiles, 4}, f32);
  auto off = dense_off(Tp, tile, h.device());
  int rc = ahb_ce_gemm(false, h.data_ptr(), T, (int)d, W.data_ptr(), (int)V, off.data_ptr<int>(),
                       labels.data_ptr<int64_t>(), nullptr, (float)ls, part.data_ptr(), err_word().data_ptr<int>(),
                       num_sms(), cur_stream(), pair);
  gemm_check(rc, "ce logits partials");
  auto lse = torch::empty({T}, f32);
  auto acc = torch::zeros({2}, f32);
  ahb_ce_combine(part.data_ptr(), ntiles, labels.data_ptr<int64_t>(), T, (int)V, (float)ls, lse.data_ptr<float>(),
                 acc.data_ptr<float>(), acc.data_ptr<float>() + 1, cur_stream());
  check_launch("ahb_ce_combine");
  return {acc.narrow(0, 0, 1), acc.narrow(0, 1, 1), lse};
}

torch::Tensor ce_online_bwd(torch::Tensor h, torch::Tensor W, torch::Tensor labels, torch::Tensor lse, double ls,
                            torch::Tensor g, torch::Tensor dW_acc, int64_t chunk_rows) {
  const int64_t T = h.size(0), d = h.size(1), V = W.size(0);
  check_acc(dW_acc, V * d, "dW_acc");
  TORCH_CHECK(V % 128 == 0, "ce: V must be a multiple of 128 for the weight gradient");
  TORCH_CHECK(chunk_rows >= 256 && chunk_rows % 256 == 0, "ce: chunk_rows a positive multiple of 256");
  auto gc = g.to(at::kFloat).reshape({1}).contiguous();
  auto dh = torch::empty({T, d}, h.options());
  const int64_t cap = std::min<int64_t>(chunk_rows, (T + 255) / 256 * 256);
  auto dl = torch::empty({cap, V}, h.options());
  int* err = err_word().data_ptr<int>();
  auto st = cur_stream();
  const char* hb = static_cast<const char*>(h.data_ptr());
  for (int64_t r0 = 0; r0 < T; r0 += chunk_rows) {
    const int64_t rows = std::min<int64_t>(chunk_rows, T - r0);
    const bool pair = ce_pair(rows);
    const int64_t tile = pair ? 256 : 128, rp = (rows + tile - 1) / tile * tile;
    auto off = dense_off(rp, tile, h.device());
    const void* hc = hb + r0 * d * 2;
    int rc = ahb_ce_gemm(true, hc, rows, (int)d, W.data_ptr(), (int)V, off.data_ptr<int>(),
                         labels.data_ptr<int64_t>() + r0, lse.data_ptr<float>() + r0, (float)ls, dl.data_ptr(), err,
                         num_sms(), st, pair);
    gemm_check(rc, "ce dlogits");
    // dh rows of the chunk (rows beyond it are not stored)
    rc = ahb_moe_gemm(AHB_GEMM_FWD_DOWN | (pair ? AHB_GEMM_PAIR : 0), dl.data_ptr(), nullptr, rp, V, W.data_ptr(),
                      nullptr, V, d, 0, off.data_ptr<int>(), 1, (int)d, 0, (int)V, (int)(V / 64),
                      static_cast<char*>(dh.data_ptr()) + r0 * d * 2, nullptr, nullptr, nullptr, nullptr, 0.f, err,
                      num_sms(), st, gc.data_ptr<float>(), (int)rows);
    gemm_check(rc, "ce dh");
    // dW += dlogits^T h over the chunk's rows (the padding rows of dlogits are zero)
    rc = ahb_moe_gemm(AHB_GEMM_WGRAD, dl.data_ptr(), nullptr, rp, V, hc, nullptr, rows, d, 0, off.data_ptr<int>(), 1,
                      (int)d, (int)V, 0, 0, dW_acc.data_ptr<float>(), nullptr, nullptr, nullptr, nullptr, 0.f, err,
                      num_sms(), st, gc.data_ptr<float>());
    gemm_check(rc, "ce dW");
  }
  return dh;
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
  m.def("gdn_fwd", &gdn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("bg"), py::arg("wg"),
        py::arg("scale"), py::arg("want_state"), py::arg("h0") = py::none());
  m.def("gdn_bwd", &gdn_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("bg"), py::arg("wg"),
        py::arg("dout"), py::arg("scale"), py::arg("h0") = py::none(), py::arg("dh_final") = py::none(),
        py::arg("want_dh0") = false);
  m.def("gdn_fwd_train", &gdn_fwd_train, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("bg"),
        py::arg("wg"), py::arg("scale"), py::arg("h0") = py::none(), py::arg("want_final") = false);
  m.def("gdn_bwd_saved", &gdn_bwd_saved, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("bg"),
        py::arg("wg"), py::arg("dout"), py::arg("scale"), py::arg("saved"), py::arg("dh_final") = py::none(),
        py::arg("want_dh0") = false);
  m.def("ssd_fwd_train", &ssd_fwd_train, py::arg("x"), py::arg("dt"), py::arg("A"), py::arg("Bm"), py::arg("Cm"),
        py::arg("s0") = py::none(), py::arg("want_final") = false);
  m.def("ssd_fwd", &ssd_fwd);
  m.def("phase_prof", &phase_prof, py::arg("counters"));
  m.def("ssd_bwd", &ssd_bwd, py::arg("x"), py::arg("dt"), py::arg("A"), py::arg("Bm"), py::arg("Cm"), py::arg("dy"),
        py::arg("states") = py::none(), py::arg("decays") = py::none(), py::arg("cumsums") = py::none(),
        py::arg("ydiag") = py::none(), py::arg("s0") = py::none(), py::arg("ds_final") = py::none(),
        py::arg("want_ds0") = false);
  m.def("gemm_dense", &gemm_dense, py::arg("a"), py::arg("b"), py::arg("pair") = false);
  m.def("gemm_error", &gemm_error);
  m.def("gemm_error_reset", &gemm_error_reset);
  m.def("moe_fwd", &moe_fwd);
  m.def("moe_bwd", &moe_bwd);
  m.def("optim_make_table", &optim_make_table);
  m.def("dense_fwd", &dense_fwd, py::arg("x"), py::arg("W"), py::arg("bias") = py::none());
  m.def("dense_dgrad", &dense_dgrad);
  m.def("dense_wgrad", &dense_wgrad);
  m.def("ce_online_fwd", &ce_online_fwd);
  m.def("ce_online_bwd", &ce_online_bwd);
  m.def("optim_prepare", &optim_prepare);
  m.def("optim_apply", &optim_apply);
  m.def("muon_ns", &muon_ns);
  m.def("muon_ns_tall", &muon_ns_tall);
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd, py::arg("x"), py::arg("delta"), py::arg("scale"), py::arg("clip"),
        py::arg("eps"), py::arg("stats") = py::none());
  m.def("add_rmsnorm_bwd", &add_rmsnorm_bwd);
  m.def("norm_gate_fwd", &norm_gate_fwd);
  m.def("norm_gate_bwd", &norm_gate_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("tp_norm_sumsq", &tp_norm_sumsq);
  m.def("tp_norm_fwd", &tp_norm_fwd);
  m.def("tp_norm_bwd_dot", &tp_norm_bwd_dot);
  m.def("tp_norm_bwd_dx", &tp_norm_bwd_dx);
  m.def("gdn_gates_fwd", &gdn_gates_fwd);
  m.def("gdn_gates_bwd", &gdn_gates_bwd);
  m.def("l2norm_heads_fwd", &l2norm_heads_fwd);
  m.def("l2norm_heads_bwd", &l2norm_heads_bwd);
  m.def("dt_act_fwd", &dt_act_fwd);
  m.def("dt_act_bwd", &dt_act_bwd);
  m.def("router_supported", &router_supported);
  m.def("router_fwd", &router_fwd);
  m.def("router_bwd", &router_bwd);
  m.def("moe_route_local", &moe_route_local);
  m.def("ep_publish", &ep_publish);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_return", &ep_return);
  m.def("ep_zero_pad", &ep_zero_pad);
  m.def("moe_expert_fwd", &moe_expert_fwd);
  m.def("moe_expert_bwd", &moe_expert_bwd);
  m.def("moe_combine_rows", &moe_combine_rows);
  m.def("moe_combine_rows_bwd", &moe_combine_rows_bwd);
  m.def("moe_sum_rows", &moe_sum_rows);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd);
  m.def("source_mix_fwd", &source_mix_fwd);
  m.def("source_mix_bwd", &source_mix_bwd);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_free", &ipc_free);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_tensor", &ipc_tensor);
  m.def("symm_barrier", &symm_barrier);
  m.def("reduce_scatter_f32", &reduce_scatter_f32);
  m.def("copy_out", &copy_out);
  m.def("tp_gemm_rs", &tp_gemm_rs);
  m.def("bias_grad_acc", &bias_grad_acc);
  m.def("sum_slots", &sum_slots);
  m.def("memcpy_async", &memcpy_async);
}
