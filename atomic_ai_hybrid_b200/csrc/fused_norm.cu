// Fused memory-bound layer glue (forward + backward), one pass over HBM each:
//
// * add_rmsnorm:  xo = sanitize(x + delta, clip);  y = rmsnorm(xo) * scale
//   (the residual update of a layer fused with the next normalisation; reference
//   `model.py:850-891` residual clips, `nn.RMSNorm` eps 1e-6).  Backward takes the
//   gradients of both outputs, masks by |xo| < clip and optionally returns the
//   delta gradient sanitized to +-1e3 (the reference's grad sanitizer on the
//   sublayer output, `model.py:192-217`).
// * norm_gate:    y = clamp(rmsnorm(x) * scale * silu(clamp(z, +-zclip)), +-oclip)
//   (GDN-2 `out_norm` x SiLU(out_gate), `model.py:650-653`; Mamba2 `ssm_out_norm`
//   x SiLU(res) with the +-300 output clip, `model.py:520-524`).
// * gdn_gates:    b = sigmoid(bp), w = sigmoid(wp),
//                 g = clamp(nan_to_num(-exp(clamp(a_h, +-20)) * softplus(f)), +-1e3)
//   (per-channel gates, `model.py:595-619`); backward adds d a_h into the fp32
//   gradient store.
// * l2norm_heads: y = x * rsqrt(sum_head x^2 + 1e-12) per 128-channel head, with
//   the gradient sanitizer on dy in the backward (`model.py:427-434`).
// * dt_act:       dt = clamp(softplus(u), 0.01, 1)  (Mamba2, `model.py:508-512`).
//
// Rows of D channels are processed by D/8 threads with 16-byte vector accesses
// (D a multiple of 256); row kernels loop over rows so that the per-column
// weight-gradient partials of one CTA stay in registers.
#include "common.cuh"
#include "launchers.h"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

struct F8 {
  float v[8];
};

AHB_DEVICE F8 ld8(const bf16* p) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  F8 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    r.v[2 * i] = f.x;
    r.v[2 * i + 1] = f.y;
  }
  return r;
}

AHB_DEVICE void st8(bf16* p, const F8& r) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(r.v[2 * i], r.v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

AHB_DEVICE float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// sum over the CTA (one row per CTA); sh needs 32 floats
AHB_DEVICE float row_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += sh[i];
  __syncthreads();
  return t;
}

AHB_DEVICE float clampf(float x, float c) { return fminf(fmaxf(x, -c), c); }

// ------------------------------------------------------------------ add_rmsnorm
// stats (optional): stats[0] = max |x + delta| over finite sums (before the clip),
// stats[1] = 1 when delta holds a NaN / infinity.  Non-negative floats order like their
// bit patterns, so both are folded in with integer atomicMax.
__global__ void add_rmsnorm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ delta,
                                       const float* __restrict__ scale, bf16* __restrict__ xo, bf16* __restrict__ y,
                                       float* __restrict__ rstd, int64_t M, int D, float clip, float eps,
                                       float* __restrict__ stats) {
  __shared__ float sh[32];
  const int c0 = threadIdx.x * 8;
  float sc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sc[i] = scale[c0 + i];
  float mx = 0.f, nf = 0.f;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 a = ld8(x + o), b = ld8(delta + o);
    F8 s;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // bf16 residual add, then nan_to_num(clip): the value the unfused path stores
      const float raw = rnd(a.v[i] + b.v[i]);
      if (isfinite(raw)) mx = fmaxf(mx, fabsf(raw));
      if (!isfinite(b.v[i])) nf = 1.f;
      s.v[i] = sanitize(raw, clip);
      ss += s.v[i] * s.v[i];
    }
    st8(xo + o, s);
    const float r = rsqrtf(row_sum(ss, sh) / D + eps);
    if (threadIdx.x == 0) rstd[row] = r;
    F8 out;
#pragma unroll
    for (int i = 0; i < 8; ++i) out.v[i] = s.v[i] * r * sc[i];
    st8(y + o, out);
  }
  if (stats) {
    mx = warp_max(mx);
    nf = warp_max(nf);
    if ((threadIdx.x & 31) == 0) {
      atomicMax(reinterpret_cast<int*>(stats), __float_as_int(mx));
      if (nf > 0.f) atomicMax(reinterpret_cast<int*>(stats + 1), __float_as_int(1.f));
    }
  }
}

// The clip mask is taken from the stored value: |xo| < clip.  It equals the mask of
// the pre-clip sum except for a NaN sum (stored as 0), whose gradient passes here.
__global__ void add_rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ gres,
                                       const bf16* __restrict__ xo, const float* __restrict__ scale,
                                       const float* __restrict__ rstd, bf16* __restrict__ dx,
                                       bf16* __restrict__ ddelta, float* __restrict__ dscale_part, int64_t M, int D,
                                       float clip) {
  __shared__ float sh[32];
  const int c0 = threadIdx.x * 8;
  float sc[8], acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sc[i] = scale[c0 + i];
    acc[i] = 0.f;
  }
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 d = ld8(dy + o), xv = ld8(xo + o);
    const float r = rstd[row];
    float xh[8], g[8], dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xh[i] = xv.v[i] * r;
      g[i] = d.v[i] * sc[i];
      dot += g[i] * xh[i];
      acc[i] += d.v[i] * xh[i];
    }
    dot = row_sum(dot, sh) / D;
    F8 gr;
    if (gres) gr = ld8(gres + o);
    F8 ox, od;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v = r * (g[i] - xh[i] * dot) + (gres ? gr.v[i] : 0.f);
      v = fabsf(xv.v[i]) < clip ? v : 0.f;
      ox.v[i] = v;
      od.v[i] = sanitize(v, 1e3f);
    }
    st8(dx + o, ox);
    if (ddelta) st8(ddelta + o, od);
  }
  if (dscale_part) {
#pragma unroll
    for (int i = 0; i < 8; ++i) dscale_part[(int64_t)blockIdx.x * D + c0 + i] = acc[i];
  }
}

// ------------------------------------------------------------------ norm_gate
__global__ void norm_gate_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z, int64_t zs,
                                     const float* __restrict__ scale, bf16* __restrict__ y, float* __restrict__ rstd,
                                     int64_t M, int D, float eps, float zclip, float oclip) {
  __shared__ float sh[32];
  const int c0 = threadIdx.x * 8;
  float sc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sc[i] = scale[c0 + i];
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 xv = ld8(x + o), zv = ld8(z + row * zs + c0);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += xv.v[i] * xv.v[i];
    const float r = rsqrtf(row_sum(ss, sh) / D + eps);
    if (threadIdx.x == 0) rstd[row] = r;
    F8 out;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float zc = clampf(zv.v[i], zclip);
      out.v[i] = clampf(xv.v[i] * r * sc[i] * siluf_(zc), oclip);
    }
    st8(y + o, out);
  }
}

__global__ void norm_gate_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                     const bf16* __restrict__ z, int64_t zs, const float* __restrict__ scale,
                                     const float* __restrict__ rstd, bf16* __restrict__ dx, bf16* __restrict__ dz,
                                     float* __restrict__ dscale_part, int64_t M, int D, float zclip, float oclip) {
  __shared__ float sh[32];
  const int c0 = threadIdx.x * 8;
  float sc[8], acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sc[i] = scale[c0 + i];
    acc[i] = 0.f;
  }
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 d = ld8(dy + o), xv = ld8(x + o), zv = ld8(z + row * zs + c0);
    const float r = rstd[row];
    float xh[8], g[8], dot = 0.f;
    F8 dzo;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float zc = clampf(zv.v[i], zclip);
      const float sg = sigmoidf_(zc);
      const float sz = zc * sg;
      xh[i] = xv.v[i] * r;
      const float n = xh[i] * sc[i];
      // clamp passes the gradient on [-c, c] (inclusive), as torch.clamp does
      const float dout = fabsf(n * sz) <= oclip ? d.v[i] : 0.f;
      const float dn = dout * sz;
      dzo.v[i] = fabsf(zv.v[i]) <= zclip ? dout * n * sg * (1.f + zc * (1.f - sg)) : 0.f;
      acc[i] += dn * xh[i];
      g[i] = dn * sc[i];
      dot += g[i] * xh[i];
    }
    dot = row_sum(dot, sh) / D;
    F8 ox;
#pragma unroll
    for (int i = 0; i < 8; ++i) ox.v[i] = r * (g[i] - xh[i] * dot);
    st8(dx + o, ox);
    st8(dz + o, dzo);
  }
  if (dscale_part) {
#pragma unroll
    for (int i = 0; i < 8; ++i) dscale_part[(int64_t)blockIdx.x * D + c0 + i] = acc[i];
  }
}

// ------------------------------------------------------------------ tensor-parallel norm
// RMSNorm over the full width of a head-split activation, optionally gated as norm_gate: each rank
// holds D of the row's Dfull channels, so each row statistic is a sum over the tensor-parallel group
// that the host all-reduces between two passes.  Forward: pass 1 the local sum of squares, pass 2
// the output from the group's sum.  Backward: pass 1 dz, the scale-gradient partials and the local
// dot sum(g * x_hat) (g = dL/d(x_hat)), pass 2 dx = r (g - x_hat dot / Dfull) from the group's dot.
// z == nullptr: no gate (y = clamp(rmsnorm(x) * scale, +-oclip)).
AHB_DEVICE void tp_gate_terms(const F8& xv, const F8* zv, const F8& d, const float* sc, float r, float zclip,
                              float oclip, float* xh, float* g, float* dn_out, F8* dzo) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    xh[i] = xv.v[i] * r;
    const float n = xh[i] * sc[i];
    float sz = 1.f, sg = 0.f, zc = 0.f;
    if (zv) {
      zc = clampf(zv->v[i], zclip);
      sg = sigmoidf_(zc);
      sz = zc * sg;
    }
    const float dout = fabsf(n * sz) <= oclip ? d.v[i] : 0.f;
    const float dn = dout * sz;
    if (zv) dzo->v[i] = fabsf(zv->v[i]) <= zclip ? dout * n * sg * (1.f + zc * (1.f - sg)) : 0.f;
    dn_out[i] = dn;
    g[i] = dn * sc[i];
  }
}

__global__ void tp_norm_sumsq_kernel(const bf16* __restrict__ x, float* __restrict__ ss, int64_t M, int D) {
  __shared__ float sh[32];
  const int c0 = threadIdx.x * 8;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const F8 xv = ld8(x + row * D + c0);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += xv.v[i] * xv.v[i];
    s = row_sum(s, sh);
    if (threadIdx.x == 0) ss[row] = s;
  }
}

__global__ void tp_norm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z, int64_t zs,
                                   const float* __restrict__ scale, const float* __restrict__ ss,
                                   bf16* __restrict__ y, float* __restrict__ rstd, int64_t M, int D, float inv_dfull,
                                   float eps, float zclip, float oclip) {
  const int c0 = threadIdx.x * 8;
  float sc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sc[i] = scale[c0 + i];
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 xv = ld8(x + o);
    const float r = rsqrtf(ss[row] * inv_dfull + eps);
    if (threadIdx.x == 0) rstd[row] = r;
    F8 out;
    if (z) {
      const F8 zv = ld8(z + row * zs + c0);
#pragma unroll
      for (int i = 0; i < 8; ++i) out.v[i] = clampf(xv.v[i] * r * sc[i] * siluf_(clampf(zv.v[i], zclip)), oclip);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) out.v[i] = clampf(xv.v[i] * r * sc[i], oclip);
    }
    st8(y + o, out);
  }
}

__global__ void tp_norm_bwd_dot_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                       const bf16* __restrict__ z, int64_t zs, const float* __restrict__ scale,
                                       const float* __restrict__ rstd, bf16* __restrict__ dz, float* __restrict__ dot,
                                       float* __restrict__ dscale_part, int64_t M, int D, float zclip, float oclip) {
  __shared__ float sh[32];
  const int c0 = threadIdx.x * 8;
  float sc[8], acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sc[i] = scale[c0 + i];
    acc[i] = 0.f;
  }
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 d = ld8(dy + o), xv = ld8(x + o);
    F8 zv, dzo;
    if (z) zv = ld8(z + row * zs + c0);
    float xh[8], g[8], dn[8];
    tp_gate_terms(xv, z ? &zv : nullptr, d, sc, rstd[row], zclip, oclip, xh, g, dn, &dzo);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[i] += dn[i] * xh[i];
      s += g[i] * xh[i];
    }
    s = row_sum(s, sh);
    if (threadIdx.x == 0) dot[row] = s;
    if (z) st8(dz + o, dzo);
  }
  if (dscale_part) {
#pragma unroll
    for (int i = 0; i < 8; ++i) dscale_part[(int64_t)blockIdx.x * D + c0 + i] = acc[i];
  }
}

__global__ void tp_norm_bwd_dx_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                      const bf16* __restrict__ z, int64_t zs, const float* __restrict__ scale,
                                      const float* __restrict__ rstd, const float* __restrict__ dot,
                                      bf16* __restrict__ dx, int64_t M, int D, float inv_dfull, float zclip,
                                      float oclip) {
  const int c0 = threadIdx.x * 8;
  float sc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sc[i] = scale[c0 + i];
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x) {
    const int64_t o = row * D + c0;
    const F8 d = ld8(dy + o), xv = ld8(x + o);
    F8 zv, dzo;
    if (z) zv = ld8(z + row * zs + c0);
    const float r = rstd[row];
    float xh[8], g[8], dn[8];
    tp_gate_terms(xv, z ? &zv : nullptr, d, sc, r, zclip, oclip, xh, g, dn, &dzo);
    const float dm = dot[row] * inv_dfull;
    F8 ox;
#pragma unroll
    for (int i = 0; i < 8; ++i) ox.v[i] = r * (g[i] - xh[i] * dm);
    st8(dx + o, ox);
  }
}

// ------------------------------------------------------------------ gdn_gates
// Elementwise over (M, d) with head h = (c / Dh); 8 channels per thread.
__global__ void gdn_gates_fwd_kernel(const bf16* __restrict__ bp, const bf16* __restrict__ wp,
                                     const bf16* __restrict__ fp, const float* __restrict__ decay_a,
                                     bf16* __restrict__ bg, bf16* __restrict__ wg, float* __restrict__ g, int64_t n8,
                                     int d, int Dh) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i * 8;
    const int h = (int)(o % d) / Dh;
    const float ea = __expf(clampf(decay_a[h], 20.f));
    const F8 b = ld8(bp + o), w = ld8(wp + o), f = ld8(fp + o);
    F8 ob, ow;
    float gv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      ob.v[k] = sigmoidf_(b.v[k]);
      ow.v[k] = sigmoidf_(w.v[k]);
      float gr = -ea * softplusf_(f.v[k]);
      gr = gr != gr ? 0.f : (isinf(gr) ? (gr > 0.f ? 0.f : -20.f) : gr);
      gv[k] = clampf(gr, 1e3f);
    }
    st8(bg + o, ob);
    st8(wg + o, ow);
    float4* go = reinterpret_cast<float4*>(g + o);
    go[0] = make_float4(gv[0], gv[1], gv[2], gv[3]);
    go[1] = make_float4(gv[4], gv[5], gv[6], gv[7]);
  }
}

// dg arrives in fp32; the sigmoid derivatives use the stored gate values, as
// autograd does for torch.sigmoid.  d a_h is reduced per CTA, then added atomically.
__global__ void gdn_gates_bwd_kernel(const bf16* __restrict__ dbg, const bf16* __restrict__ dwg,
                                     const float* __restrict__ dg, const bf16* __restrict__ bg,
                                     const bf16* __restrict__ wg, const bf16* __restrict__ fp,
                                     const float* __restrict__ decay_a, bf16* __restrict__ dbp, bf16* __restrict__ dwp,
                                     bf16* __restrict__ dfp, float* __restrict__ da_acc, int64_t n8, int d, int Dh,
                                     int H) {
  extern __shared__ float sda[];  // H floats
  for (int h = threadIdx.x; h < H; h += blockDim.x) sda[h] = 0.f;
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i * 8;
    const int h = (int)(o % d) / Dh;
    const float a = decay_a[h];
    const float ea = __expf(clampf(a, 20.f));
    const F8 db = ld8(dbg + o), dw = ld8(dwg + o), b = ld8(bg + o), w = ld8(wg + o), f = ld8(fp + o);
    const float4 g0 = reinterpret_cast<const float4*>(dg + o)[0], g1 = reinterpret_cast<const float4*>(dg + o)[1];
    const float dgv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    F8 ob, ow, of;
    float da = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      ob.v[k] = db.v[k] * b.v[k] * (1.f - b.v[k]);
      ow.v[k] = dw.v[k] * w.v[k] * (1.f - w.v[k]);
      const float sp = softplusf_(f.v[k]);
      const float gr = -ea * sp;
      const bool pass = isfinite(gr) && fabsf(gr) <= 1e3f;
      const float dgr = pass ? dgv[k] : 0.f;
      of.v[k] = -dgr * ea * sigmoidf_(f.v[k]);
      if (pass) da += dgr * gr;  // a non-finite decay contributes nothing (not 0 * inf)
    }
    st8(dbp + o, ob);
    st8(dwp + o, ow);
    st8(dfp + o, of);
    if (fabsf(a) <= 20.f) atomicAdd(&sda[h], da);
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x)
    if (sda[h] != 0.f) atomicAdd(da_acc + h, sda[h]);
}

// ------------------------------------------------------------------ l2norm_heads
// One 128-channel head per 16 threads (8 channels each).
__global__ void l2norm_heads_fwd_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, float* __restrict__ rn,
                                        int64_t nheads) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t hid = t >> 4;
  const bool live = hid < nheads;
  const int64_t o = (live ? hid : 0) * 128 + (t & 15) * 8;
  const F8 v = ld8(x + o);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss += v.v[k] * v.v[k];
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if (!live) return;
  const float r = rsqrtf(ss + 1e-12f);
  if ((t & 15) == 0) rn[hid] = r;
  F8 out;
#pragma unroll
  for (int k = 0; k < 8; ++k) out.v[k] = v.v[k] * r;
  st8(y + o, out);
}

__global__ void l2norm_heads_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                        const float* __restrict__ rn, bf16* __restrict__ dx, int64_t nheads) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t hid = t >> 4;
  const bool live = hid < nheads;
  const int64_t o = (live ? hid : 0) * 128 + (t & 15) * 8;
  const F8 v = ld8(x + o), d = ld8(dy + o);
  float ds[8], dot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    ds[k] = sanitize(d.v[k], 1e3f);  // the sanitizer sits on the normalised output
    dot += ds[k] * v.v[k];
  }
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, m);
  if (!live) return;
  const float r = rn[hid];
  const float r3 = r * r * r;
  F8 out;
#pragma unroll
  for (int k = 0; k < 8; ++k) out.v[k] = r * ds[k] - v.v[k] * r3 * dot;
  st8(dx + o, out);
}

// ------------------------------------------------------------------ dt_act
__global__ void dt_act_fwd_kernel(const bf16* __restrict__ u, bf16* __restrict__ dt, int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const F8 v = ld8(u + i * 8);
    F8 out;
#pragma unroll
    for (int k = 0; k < 8; ++k) out.v[k] = fminf(fmaxf(rnd(softplusf_(v.v[k])), 1e-2f), 1.f);
    st8(dt + i * 8, out);
  }
}

__global__ void dt_act_bwd_kernel(const bf16* __restrict__ ddt, const bf16* __restrict__ u, bf16* __restrict__ du,
                                  int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const F8 v = ld8(u + i * 8), d = ld8(ddt + i * 8);
    F8 out;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sp = rnd(softplusf_(v.v[k]));
      out.v[k] = (sp >= 1e-2f && sp <= 1.f) ? d.v[k] * sigmoidf_(v.v[k]) : 0.f;
    }
    st8(du + i * 8, out);
  }
}

int sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

int ew_grid(int64_t n8) {
  const int64_t b = (n8 + 255) / 256;
  const int64_t cap = (int64_t)sms() * 16;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace

int ahb_row_supported(int D) { return D % 256 == 0 && D <= 8192; }

int ahb_row_bwd_blocks(int64_t M) {
  const int64_t cap = (int64_t)sms() * 4;
  return (int)(M < cap ? (M < 1 ? 1 : M) : cap);
}

void ahb_add_rmsnorm_fwd(const void* x, const void* delta, const float* scale, void* xo, void* y, float* rstd,
                         int64_t M, int D, float clip, float eps, cudaStream_t st, float* stats) {
  if (M <= 0) return;
  const int grid = (int)(M < (int64_t)sms() * 16 ? M : (int64_t)sms() * 16);
  add_rmsnorm_fwd_kernel<<<grid, D / 8, 0, st>>>((const bf16*)x, (const bf16*)delta, scale, (bf16*)xo, (bf16*)y,
                                                 rstd, M, D, clip, eps, stats);
}

void ahb_add_rmsnorm_bwd(const void* dy, const void* gres, const void* xo, const float* scale, const float* rstd,
                         void* dx, void* ddelta, float* dscale_part, int64_t M, int D, float clip, cudaStream_t st) {
  if (M <= 0) return;
  add_rmsnorm_bwd_kernel<<<ahb_row_bwd_blocks(M), D / 8, 0, st>>>(
      (const bf16*)dy, (const bf16*)gres, (const bf16*)xo, scale, rstd, (bf16*)dx, (bf16*)ddelta, dscale_part, M, D,
      clip);
}

void ahb_norm_gate_fwd(const void* x, const void* z, int64_t zs, const float* scale, void* y, float* rstd, int64_t M,
                       int D, float eps, float zclip, float oclip, cudaStream_t st) {
  if (M <= 0) return;
  const int grid = (int)(M < (int64_t)sms() * 16 ? M : (int64_t)sms() * 16);
  norm_gate_fwd_kernel<<<grid, D / 8, 0, st>>>((const bf16*)x, (const bf16*)z, zs, scale, (bf16*)y, rstd, M, D, eps,
                                               zclip, oclip);
}

void ahb_norm_gate_bwd(const void* dy, const void* x, const void* z, int64_t zs, const float* scale, const float* rstd,
                       void* dx, void* dz, float* dscale_part, int64_t M, int D, float zclip, float oclip,
                       cudaStream_t st) {
  if (M <= 0) return;
  norm_gate_bwd_kernel<<<ahb_row_bwd_blocks(M), D / 8, 0, st>>>((const bf16*)dy, (const bf16*)x, (const bf16*)z, zs,
                                                                scale, rstd, (bf16*)dx, (bf16*)dz, dscale_part, M, D,
                                                                zclip, oclip);
}

void ahb_gdn_gates_fwd(const void* bp, const void* wp, const void* fp, const float* decay_a, void* bg, void* wg,
                       float* g, int64_t n, int d, int Dh, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 <= 0) return;
  gdn_gates_fwd_kernel<<<ew_grid(n8), 256, 0, st>>>((const bf16*)bp, (const bf16*)wp, (const bf16*)fp, decay_a,
                                                    (bf16*)bg, (bf16*)wg, g, n8, d, Dh);
}

void ahb_gdn_gates_bwd(const void* dbg, const void* dwg, const float* dg, const void* bg, const void* wg,
                       const void* fp, const float* decay_a, void* dbp, void* dwp, void* dfp, float* da_acc,
                       int64_t n, int d, int Dh, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 <= 0) return;
  const int H = d / Dh;
  gdn_gates_bwd_kernel<<<ew_grid(n8), 256, H * sizeof(float), st>>>(
      (const bf16*)dbg, (const bf16*)dwg, dg, (const bf16*)bg, (const bf16*)wg, (const bf16*)fp, decay_a, (bf16*)dbp,
      (bf16*)dwp, (bf16*)dfp, da_acc, n8, d, Dh, H);
}

void ahb_l2norm_heads_fwd(const void* x, void* y, float* rn, int64_t nheads, cudaStream_t st) {
  if (nheads <= 0) return;
  const int64_t threads = nheads * 16;
  l2norm_heads_fwd_kernel<<<(int)((threads + 255) / 256), 256, 0, st>>>((const bf16*)x, (bf16*)y, rn, nheads);
}

void ahb_l2norm_heads_bwd(const void* dy, const void* x, const float* rn, void* dx, int64_t nheads, cudaStream_t st) {
  if (nheads <= 0) return;
  const int64_t threads = nheads * 16;
  l2norm_heads_bwd_kernel<<<(int)((threads + 255) / 256), 256, 0, st>>>((const bf16*)dy, (const bf16*)x, rn,
                                                                         (bf16*)dx, nheads);
}

void ahb_dt_act_fwd(const void* u, void* dt, int64_t n, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 <= 0) return;
  dt_act_fwd_kernel<<<ew_grid(n8), 256, 0, st>>>((const bf16*)u, (bf16*)dt, n8);
}

void ahb_dt_act_bwd(const void* ddt, const void* u, void* du, int64_t n, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 <= 0) return;
  dt_act_bwd_kernel<<<ew_grid(n8), 256, 0, st>>>((const bf16*)ddt, (const bf16*)u, (bf16*)du, n8);
}

static int tp_norm_grid(int64_t M) { return (int)(M < (int64_t)sms() * 16 ? M : (int64_t)sms() * 16); }

void ahb_tp_norm_sumsq(const void* x, float* ss, int64_t M, int D, cudaStream_t st) {
  if (M <= 0) return;
  tp_norm_sumsq_kernel<<<tp_norm_grid(M), D / 8, 0, st>>>((const bf16*)x, ss, M, D);
}

void ahb_tp_norm_fwd(const void* x, const void* z, int64_t zs, const float* scale, const float* ss, void* y,
                     float* rstd, int64_t M, int D, float inv_dfull, float eps, float zclip, float oclip,
                     cudaStream_t st) {
  if (M <= 0) return;
  tp_norm_fwd_kernel<<<tp_norm_grid(M), D / 8, 0, st>>>((const bf16*)x, (const bf16*)z, zs, scale, ss, (bf16*)y, rstd,
                                                        M, D, inv_dfull, eps, zclip, oclip);
}

void ahb_tp_norm_bwd_dot(const void* dy, const void* x, const void* z, int64_t zs, const float* scale,
                         const float* rstd, void* dz, float* dot, float* dscale_part, int64_t M, int D, float zclip,
                         float oclip, cudaStream_t st) {
  if (M <= 0) return;
  tp_norm_bwd_dot_kernel<<<ahb_row_bwd_blocks(M), D / 8, 0, st>>>((const bf16*)dy, (const bf16*)x, (const bf16*)z,
                                                                  zs, scale, rstd, (bf16*)dz, dot, dscale_part, M, D,
                                                                  zclip, oclip);
}

void ahb_tp_norm_bwd_dx(const void* dy, const void* x, const void* z, int64_t zs, const float* scale,
                        const float* rstd, const float* dot, void* dx, int64_t M, int D, float inv_dfull, float zclip,
                        float oclip, cudaStream_t st) {
  if (M <= 0) return;
  tp_norm_bwd_dx_kernel<<<tp_norm_grid(M), D / 8, 0, st>>>((const bf16*)dy, (const bf16*)x, (const bf16*)z, zs, scale,
                                                           rstd, dot, (bf16*)dx, M, D, inv_dfull, zclip, oclip);
}
