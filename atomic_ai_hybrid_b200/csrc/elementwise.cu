// Memory-bound kernels: sanitize, RMSNorm fwd/bwd, depthwise causal conv1d
// (+bias, +SiLU, +clamp) fwd/bwd, gradient accumulation and embedding gather/scatter.
//
// Weight gradients (RMSNorm scale, conv taps/bias, embedding rows) are added
// straight into the caller's fp32 accumulator (the flat gradient store), so no
// per-micro-step weight-gradient tensor is materialised.
//
// Plain CUDA (no framework headers): the launchers below take raw pointers and
// a stream; `bindings.cpp` adapts them to torch tensors.
#include "common.cuh"
#include "launchers.h"
#include <algorithm>

using namespace ahb;
using bf16 = __nv_bfloat16;
// ----------------------------------------------------------------- sanitize
template <typename T>
__global__ void sanitize_kernel(T* __restrict__ out, const T* __restrict__ in, int64_t n, float c) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f<T>(sanitize(to_f(in[i]), c));
}


// ----------------------------------------------------------------- RMSNorm
// A group of G warps handles one row; each thread holds VPL values (D <= 32*G*VPL).
// Blocks are 256 threads = 8/G rows.
template <int G>
AHB_DEVICE float group_sum(float v, float* sh) {
  v = warp_sum(v);
  if constexpr (G == 1) return v;
  // only the G warps of this row's group synchronise (named barrier 1 + group)
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = w / G;
  if (lane == 0) sh[w] = v;
  asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * G) : "memory");
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < G; ++i) t += sh[grp * G + i];
  asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * G) : "memory");
  return t;
}

template <typename T, int VPL, int G>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const T* __restrict__ x, const float* __restrict__ scale,
    T* __restrict__ y, float* __restrict__ rstd_out, int64_t M, int D, float eps) {
  __shared__ float sh[8];
  const int gl = threadIdx.x % (32 * G);
  const int64_t row = blockIdx.x * (int64_t)(8 / G) + threadIdx.x / (32 * G);
  const bool live = row < M;
  const T* xr = x + (live ? row : 0) * D;
  float v[VPL];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    int c = i * 32 * G + gl;
    v[i] = (live && c < D) ? to_f(xr[c]) : 0.f;
    ss += v[i] * v[i];
  }
  ss = group_sum<G>(ss, sh);
  if (!live) return;
  float r = rsqrtf(ss / D + eps);
  if (gl == 0) rstd_out[row] = r;
  T* yr = y + row * D;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    int c = i * 32 * G + gl;
    if (c < D) yr[c] = from_f<T>(v[i] * r * scale[c]);
  }
}

template <typename T, int VPL, int G>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x,
    const float* __restrict__ scale, const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ dscale,
    int64_t M, int D) {
  __shared__ float sh[8];
  const int gl = threadIdx.x % (32 * G);
  const int rpb = 8 / G;
  float acc[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
  const int64_t nrow_iters = (M + (int64_t)gridDim.x * rpb - 1) / ((int64_t)gridDim.x * rpb);
  for (int64_t it = 0; it < nrow_iters; ++it) {
    const int64_t row = (it * gridDim.x + blockIdx.x) * rpb + threadIdx.x / (32 * G);
    const bool live = row < M;
    const T* xr = x + (live ? row : 0) * D;
    const T* dyr = dy + (live ? row : 0) * D;
    float r = live ? rstd[row] : 0.f;
    float xh[VPL], g[VPL];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      int c = i * 32 * G + gl;
      bool ok = live && c < D;
      xh[i] = ok ? to_f(xr[c]) * r : 0.f;
      float d = ok ? to_f(dyr[c]) : 0.f;
      acc[i] += d * xh[i];
      g[i] = ok ? d * scale[c] : 0.f;
      dot += g[i] * xh[i];
    }
    dot = group_sum<G>(dot, sh) / D;
    if (live) {
      T* dxr = dx + row * D;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        int c = i * 32 * G + gl;
        if (c < D) dxr[c] = from_f<T>(r * (g[i] - xh[i] * dot));
      }
    }
  }
  if (dscale) {
    // partial column sums of this block -> dscale_part[blockIdx.x * D + c] (reduced by colsum_add_kernel)
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      int c = i * 32 * G + gl;
      if (c < D) atomicAdd(dscale + (int64_t)blockIdx.x * D + c, acc[i]);
    }
  }
}

// out[c] += sum_b part[b * D + c]: a block of 256 threads covers 32 columns, its 8 warps sum every
// 8th row (lane = column, coalesced), and the warps' sums are added in a fixed order
__global__ void __launch_bounds__(256) colsum_add_kernel(const float* __restrict__ part, int nb, int D,
                                                         float* __restrict__ out) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < D)
    for (int b = w; b < nb; b += 8) s += part[(int64_t)b * D + c];
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && c < D) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][lane];
    out[c] += t;
  }
}

// ----------------------------------------------------------------- bias gradient
// acc[c] += sum_r dy[r, c]  (dy bf16 (M, N) row-major, N % 8 == 0).  A block covers 256 columns
// (32 threads x 8 columns, 16-byte loads) and a slice of the rows (8 row lanes); the row lanes
// are reduced in shared memory and each column gets one fp32 atomic per block.
__global__ void bias_grad_kernel(const __nv_bfloat16* __restrict__ dy, int64_t M, int N, int64_t ld,
                                 int64_t rows_per, float* __restrict__ acc) {
  __shared__ float red[8][257];
  const int cg = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + cg * 8;
  const int64_t r_lo = blockIdx.y * rows_per, r_hi = r_lo + rows_per < M ? r_lo + rows_per : M;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < N) {
    for (int64_t r = r_lo + rl; r < r_hi; r += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(dy + r * ld + c0);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        a[2 * i] += f.x;
        a[2 * i + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[rl][cg * 8 + i] = a[i];
  __syncthreads();
  const int c = threadIdx.x;  // one column of the block per thread
  if (blockIdx.x * 256 + c < N) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += red[j][c];
    atomicAdd(acc + blockIdx.x * 256 + c, s);
  }
}

void ahb_bias_grad_acc(const void* dy, int64_t M, int N, int64_t ld, float* acc, cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int gx = (N + 255) / 256;
  int64_t gy = ((int64_t)sms * 8 + gx - 1) / gx;
  int64_t rows_per = (M + gy - 1) / gy;
  rows_per = (rows_per + 7) / 8 * 8;
  gy = (M + rows_per - 1) / rows_per;
  bias_grad_kernel<<<dim3(gx, (unsigned)gy), 256, 0, st>>>((const __nv_bfloat16*)dy, M, N, ld, rows_per, acc);
}

// ----------------------------------------------------------------- causal conv1d
// x: (B, L, C) with row stride `xs` (elements); w: (C, W) fp32 or bf16; b: (C,) fp32.
// y[b,t,c] = act(sum_k w[c,k] * x[b, t-(W-1)+k, c] + bias[c]), then clamp(+-clip) if clip>0.
// Each thread: 8 consecutive channels x TT consecutive timesteps.
constexpr int CONV_TT = 16;

template <typename T, typename WT, int W>
__global__ void conv1d_fwd_kernel(const T* __restrict__ x, int64_t xs, const WT* __restrict__ w,
                                  const float* __restrict__ bias, T* __restrict__ y, int B, int L, int C,
                                  bool silu, float clip) {
  const int cg = C / 8;
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int nt = (L + CONV_TT - 1) / CONV_TT;
  if (idx >= (int64_t)B * nt * cg) return;
  const int c0 = (int)(idx % cg) * 8;
  const int tb = (int)((idx / cg) % nt) * CONV_TT;
  const int b = (int)(idx / ((int64_t)cg * nt));
  float wk[8][W], bs[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int k = 0; k < W; ++k) wk[j][k] = to_f(w[(c0 + j) * W + k]);
    bs[j] = bias ? bias[c0 + j] : 0.f;
  }
  float hist[W][8];
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
    int t = tb - (W - 1) + k;
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[k][j] = t >= 0 ? to_f(x[((int64_t)b * L + t) * xs + c0 + j]) : 0.f;
  }
  for (int tt = 0; tt < CONV_TT; ++tt) {
    int t = tb + tt;
    if (t >= L) break;
    const T* xr = x + ((int64_t)b * L + t) * xs + c0;
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[W - 1][j] = to_f(xr[j]);
    T* yr = y + ((int64_t)b * L + t) * C + c0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = bs[j];
#pragma unroll
      for (int k = 0; k < W; ++k) a += wk[j][k] * hist[k][j];
      if (silu) a = siluf_(a);
      if (clip > 0.f) a = fminf(fmaxf(a, -clip), clip);
      yr[j] = from_f<T>(a);
    }
#pragma unroll
    for (int k = 0; k < W - 1; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) hist[k][j] = hist[k + 1][j];
  }
}

// Backward.  dpre[t] = dy[t] * act'(pre[t]) (masked by the clamp);
// dx[s] = sum_k w[k] dpre[s + W-1-k]; dw[k] += sum_t dpre[t] x[t-(W-1)+k]; db += sum_t dpre[t].
constexpr int CONV_SUB = 8;  // 16-step tiles per thread in the backward (fewer weight-grad atomics)

template <typename T, typename WT, int W>
__global__ void conv1d_bwd_kernel(const T* __restrict__ x, int64_t xs, const WT* __restrict__ w,
                                  const float* __restrict__ bias, const T* __restrict__ dy, T* __restrict__ dx,
                                  int64_t dxs, float* __restrict__ dw, float* __restrict__ db, int B, int L, int C,
                                  bool silu, float clip) {
  const int cg = C / 8;
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int span = CONV_TT * CONV_SUB;
  const int nt = (L + span - 1) / span;
  if (idx >= (int64_t)B * nt * cg) return;
  const int c0 = (int)(idx % cg) * 8;
  const int tspan = (int)((idx / cg) % nt) * span;
  const int b = (int)(idx / ((int64_t)cg * nt));
  float wk[8][W], bs[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int k = 0; k < W; ++k) wk[j][k] = to_f(w[(c0 + j) * W + k]);
    bs[j] = bias ? bias[c0 + j] : 0.f;
  }
  float dwl[8][W], dbl[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    dbl[j] = 0.f;
#pragma unroll
    for (int k = 0; k < W; ++k) dwl[j][k] = 0.f;
  }
  for (int sub = 0; sub < CONV_SUB; ++sub) {
    const int tb = tspan + sub * CONV_TT;
    if (tb >= L) break;
    // dpre for t in [tb, tb+TT+W-2] (needed by dx of s in [tb, tb+TT-1])
    float dp[CONV_TT + W - 1][8];
#pragma unroll
    for (int i = 0; i < CONV_TT + W - 1; ++i) {
      int t = tb + i;
      if (t >= L) {
#pragma unroll
        for (int j = 0; j < 8; ++j) dp[i][j] = 0.f;
        continue;
      }
      float xv[W][8];
#pragma unroll
      for (int k = 0; k < W; ++k) {
        int tx = t - (W - 1) + k;
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[k][j] = tx >= 0 ? to_f(x[((int64_t)b * L + tx) * xs + c0 + j]) : 0.f;
      }
      const T* dyr = dy + ((int64_t)b * L + t) * C + c0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float a = bs[j];
#pragma unroll
        for (int k = 0; k < W; ++k) a += wk[j][k] * xv[k][j];
        float g = to_f(dyr[j]);
        float post = a;
        if (silu) {
          float sg = sigmoidf_(a);
          post = a * sg;
          g *= sg * (1.f + a * (1.f - sg));
        }
        if (clip > 0.f && fabsf(post) > clip) g = 0.f;
        dp[i][j] = g;
        if (i < CONV_TT) {  // weight/bias grads counted once per t (owned t range)
          dbl[j] += g;
#pragma unroll
          for (int k = 0; k < W; ++k) dwl[j][k] += g * xv[k][j];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < CONV_TT; ++i) {
      int sidx = tb + i;
      if (sidx >= L) break;
      T* dxr = dx + ((int64_t)b * L + sidx) * dxs + c0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < W; ++k) a += wk[j][k] * dp[i + (W - 1) - k][j];
        dxr[j] = from_f<T>(a);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (db) atomicAdd(db + c0 + j, dbl[j]);
#pragma unroll
    for (int k = 0; k < W; ++k) atomicAdd(dw + (c0 + j) * W + k, dwl[j][k]);
  }
}

// Streaming variants for bf16 activations (C % 128 == 0): a warp owns 128 channels
// (4 per lane, 8-byte accesses) over a span of CSPAN steps and slides a 4-tap window
// along time, so every x / dy element is read once and dx is written once.  The 8
// warps of a CTA take consecutive spans of the same channels and pre-reduce the
// weight gradients in shared memory before one atomic per (channel, tap).
constexpr int CSPAN = 64;

AHB_DEVICE void ld4(const bf16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
AHB_DEVICE void st4(bf16* p, const float (&v)[4]) {
  uint2 u;
  *reinterpret_cast<__nv_bfloat162*>(&u.x) = __floats2bfloat162_rn(v[0], v[1]);
  *reinterpret_cast<__nv_bfloat162*>(&u.y) = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename WT>
__global__ void __launch_bounds__(256) conv1d_fwd_stream_kernel(const bf16* __restrict__ x, int64_t xs,
                                                                const WT* __restrict__ w,
                                                                const float* __restrict__ bias, bf16* __restrict__ y,
                                                                int B, int L, int C, bool silu, float clip) {
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 128 + lane * 4;
  const int nspan = (L + CSPAN - 1) / CSPAN;
  const int64_t gs = (int64_t)blockIdx.y * 8 + wp;
  if (gs >= (int64_t)B * nspan) return;
  const int b = (int)(gs / nspan), t0 = (int)(gs % nspan) * CSPAN;
  float wk[4][4], bs[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int k = 0; k < 4; ++k) wk[j][k] = to_f(w[(c0 + j) * 4 + k]);
    bs[j] = bias ? bias[c0 + j] : 0.f;
  }
  const bf16* xb = x + (int64_t)b * L * xs + c0;
  bf16* yb = y + (int64_t)b * L * C + c0;
  float xw[3][4];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int t = t0 - 3 + k;
    if (t >= 0) ld4(xb + (int64_t)t * xs, xw[k]);
    else { xw[k][0] = xw[k][1] = xw[k][2] = xw[k][3] = 0.f; }
  }
  const int tend = t0 + CSPAN < L ? t0 + CSPAN : L;
#pragma unroll 4
  for (int t = t0; t < tend; ++t) {
    float xc[4], o[4];
    ld4(xb + (int64_t)t * xs, xc);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = bs[j] + wk[j][0] * xw[0][j] + wk[j][1] * xw[1][j] + wk[j][2] * xw[2][j] + wk[j][3] * xc[j];
      if (silu) a = siluf_(a);
      if (clip > 0.f) a = fminf(fmaxf(a, -clip), clip);
      o[j] = a;
      xw[0][j] = xw[1][j];
      xw[1][j] = xw[2][j];
      xw[2][j] = xc[j];
    }
    st4(yb + (int64_t)t * C, o);
  }
}

template <typename WT>
__global__ void __launch_bounds__(256) conv1d_bwd_stream_kernel(const bf16* __restrict__ x, int64_t xs,
                                                                const WT* __restrict__ w,
                                                                const float* __restrict__ bias,
                                                                const bf16* __restrict__ dy, bf16* __restrict__ dx,
                                                                int64_t dxs, float* __restrict__ dw,
                                                                float* __restrict__ db, int B, int L, int C,
                                                                bool silu, float clip) {
  __shared__ float red[128][5];  // per channel: 4 taps + bias
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 128 * 5; i += blockDim.x) (&red[0][0])[i] = 0.f;
  __syncthreads();
  const int c0 = blockIdx.x * 128 + lane * 4;
  const int nspan = (L + CSPAN - 1) / CSPAN;
  const int64_t gs = (int64_t)blockIdx.y * 8 + wp;
  if (gs < (int64_t)B * nspan) {
    const int b = (int)(gs / nspan), t0 = (int)(gs % nspan) * CSPAN;
    float wk[4][4], bs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int k = 0; k < 4; ++k) wk[j][k] = to_f(w[(c0 + j) * 4 + k]);
      bs[j] = bias ? bias[c0 + j] : 0.f;
    }
    const bf16* xb = x + (int64_t)b * L * xs + c0;
    const bf16* dyb = dy + (int64_t)b * L * C + c0;
    bf16* dxb = dx + (int64_t)b * L * dxs + c0;
    float xw[3][4], dpw[3][4], dwl[4][4], dbl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dbl[j] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) dwl[j][k] = 0.f;
#pragma unroll
      for (int k = 0; k < 3; ++k) dpw[k][j] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int t = t0 - 3 + k;
      if (t >= 0) ld4(xb + (int64_t)t * xs, xw[k]);
      else { xw[k][0] = xw[k][1] = xw[k][2] = xw[k][3] = 0.f; }
    }
    const int own_end = t0 + CSPAN < L ? t0 + CSPAN : L;
    // dp(t) for t in [t0, own_end + 3): the last three steps only feed dx of the span's tail
#pragma unroll 2
    for (int t = t0; t < own_end + 3; ++t) {
      float xc[4] = {0.f, 0.f, 0.f, 0.f}, g[4] = {0.f, 0.f, 0.f, 0.f};
      if (t < L) {
        float dv[4];
        ld4(xb + (int64_t)t * xs, xc);
        ld4(dyb + (int64_t)t * C, dv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = bs[j] + wk[j][0] * xw[0][j] + wk[j][1] * xw[1][j] + wk[j][2] * xw[2][j] + wk[j][3] * xc[j];
          float gj = dv[j], post = a;
          if (silu) {
            const float sg = sigmoidf_(a);
            post = a * sg;
            gj *= sg * (1.f + a * (1.f - sg));
          }
          if (clip > 0.f && fabsf(post) > clip) gj = 0.f;
          g[j] = gj;
        }
        if (t < own_end) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            dbl[j] += g[j];
            dwl[j][0] += g[j] * xw[0][j];
            dwl[j][1] += g[j] * xw[1][j];
            dwl[j][2] += g[j] * xw[2][j];
            dwl[j][3] += g[j] * xc[j];
          }
        }
      }
      const int sx = t - 3;  // dx[s] = sum_k w_k dp[s + 3 - k]
      if (sx >= t0) {
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = wk[j][0] * g[j] + wk[j][1] * dpw[2][j] + wk[j][2] * dpw[1][j] + wk[j][3] * dpw[0][j];
        st4(dxb + (int64_t)sx * dxs, o);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xw[0][j] = xw[1][j];
        xw[1][j] = xw[2][j];
        xw[2][j] = xc[j];
        dpw[0][j] = dpw[1][j];
        dpw[1][j] = dpw[2][j];
        dpw[2][j] = g[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int k = 0; k < 4; ++k) atomicAdd(&red[lane * 4 + j][k], dwl[j][k]);
      atomicAdd(&red[lane * 4 + j][4], dbl[j]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 128 * 5; i += blockDim.x) {
    const int ch = blockIdx.x * 128 + i / 5, k = i % 5;
    const float v = (&red[0][0])[i];
    if (k < 4) atomicAdd(dw + ch * 4 + k, v);
    else if (db) atomicAdd(db + ch, v);
  }
}

// Same computation with the x / dy rows staged in shared memory by cp.async, two chunks of
// CPF steps per warp in flight: a warp's next chunk loads while it computes the current one
// (the kernel above keeps one load of each per warp in flight and waits on it every step).
// Needs 16-byte aligned rows (xs % 8 == 0).  Lanes 0-15 copy the x row of a step and lanes
// 16-31 its dy row, 16 bytes each; lane l computes channels 4l..4l+3 as above.
constexpr int CPF = 8;

AHB_DEVICE void ew_cp16(void* dst, const void* src) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(src) : "memory");
}
AHB_DEVICE void ew_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
AHB_DEVICE void ew_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename WT>
__global__ void __launch_bounds__(256, 2) conv1d_bwd_pf_kernel(const bf16* __restrict__ x, int64_t xs,
                                                               const WT* __restrict__ w,
                                                               const float* __restrict__ bias,
                                                               const bf16* __restrict__ dy, bf16* __restrict__ dx,
                                                               int64_t dxs, float* __restrict__ dw,
                                                               float* __restrict__ db, int B, int L, int C,
                                                               bool silu, float clip) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // per warp: [2 buffers][CPF steps][x row 128 | dy row 128] bf16
  bf16* ring = reinterpret_cast<bf16*>(smem_raw) + (threadIdx.x >> 5) * (2 * CPF * 256);
  __shared__ float red[128][5];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 128 * 5; i += blockDim.x) (&red[0][0])[i] = 0.f;
  __syncthreads();
  const int cb = blockIdx.x * 128;
  const int c0 = cb + lane * 4;
  const int nspan = (L + CSPAN - 1) / CSPAN;
  const int64_t gs = (int64_t)blockIdx.y * 8 + wp;
  if (gs < (int64_t)B * nspan) {
    const int b = (int)(gs / nspan), t0 = (int)(gs % nspan) * CSPAN;
    float wk[4][4], bs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int k = 0; k < 4; ++k) wk[j][k] = to_f(w[(c0 + j) * 4 + k]);
      bs[j] = bias ? bias[c0 + j] : 0.f;
    }
    const bf16* xblk = x + (int64_t)b * L * xs + cb;
    const bf16* dyblk = dy + (int64_t)b * L * C + cb;
    bf16* dxb = dx + (int64_t)b * L * dxs + c0;
    float xw[3][4], dpw[3][4], dwl[4][4], dbl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dbl[j] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) dwl[j][k] = 0.f;
#pragma unroll
      for (int k = 0; k < 3; ++k) dpw[k][j] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int t = t0 - 3 + k;
      if (t >= 0) ld4(x + (int64_t)b * L * xs + c0 + (int64_t)t * xs, xw[k]);
      else { xw[k][0] = xw[k][1] = xw[k][2] = xw[k][3] = 0.f; }
    }
    const int own_end = t0 + CSPAN < L ? t0 + CSPAN : L;
    const int t_last = own_end + 3 < L ? own_end + 3 : L;  // steps with x / dy to read
    const int t_stop = own_end + 3;                        // steps that produce dx rows
    const int nch = (t_stop - t0 + CPF - 1) / CPF;
    auto issue = [&](int ch) {
      bf16* dst = ring + (ch & 1) * (CPF * 256);
      const int half = lane >> 4, piece = lane & 15;
#pragma unroll
      for (int s = 0; s < CPF; ++s) {
        const int t = t0 + ch * CPF + s;
        if (t < t_last) {
          const bf16* src = half ? dyblk + (int64_t)t * C : xblk + (int64_t)t * xs;
          ew_cp16(dst + s * 256 + half * 128 + piece * 8, src + piece * 8);
        }
      }
      ew_cp_commit();
    };
    issue(0);
    for (int ch = 0; ch < nch; ++ch) {
      if (ch + 1 < nch) {
        issue(ch + 1);
        ew_cp_wait<1>();
      } else {
        ew_cp_wait<0>();
      }
      __syncwarp();
      const bf16* buf = ring + (ch & 1) * (CPF * 256);
#pragma unroll 2
      for (int s = 0; s < CPF; ++s) {
        const int t = t0 + ch * CPF + s;
        if (t >= t_stop) break;
        float xc[4] = {0.f, 0.f, 0.f, 0.f}, g[4] = {0.f, 0.f, 0.f, 0.f};
        if (t < L) {
          float dv[4];
          ld4(buf + s * 256 + lane * 4, xc);
          ld4(buf + s * 256 + 128 + lane * 4, dv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a = bs[j] + wk[j][0] * xw[0][j] + wk[j][1] * xw[1][j] + wk[j][2] * xw[2][j] + wk[j][3] * xc[j];
            float gj = dv[j], post = a;
            if (silu) {
              const float sg = sigmoidf_(a);
              post = a * sg;
              gj *= sg * (1.f + a * (1.f - sg));
            }
            if (clip > 0.f && fabsf(post) > clip) gj = 0.f;
            g[j] = gj;
          }
          if (t < own_end) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              dbl[j] += g[j];
              dwl[j][0] += g[j] * xw[0][j];
              dwl[j][1] += g[j] * xw[1][j];
              dwl[j][2] += g[j] * xw[2][j];
              dwl[j][3] += g[j] * xc[j];
            }
          }
        }
        const int sx = t - 3;  // dx[s] = sum_k w_k dp[s + 3 - k]
        if (sx >= t0) {
          float o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = wk[j][0] * g[j] + wk[j][1] * dpw[2][j] + wk[j][2] * dpw[1][j] + wk[j][3] * dpw[0][j];
          st4(dxb + (int64_t)sx * dxs, o);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          xw[0][j] = xw[1][j];
          xw[1][j] = xw[2][j];
          xw[2][j] = xc[j];
          dpw[0][j] = dpw[1][j];
          dpw[1][j] = dpw[2][j];
          dpw[2][j] = g[j];
        }
      }
      __syncwarp();  // every lane is done with this buffer before the next issue overwrites it
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int k = 0; k < 4; ++k) atomicAdd(&red[lane * 4 + j][k], dwl[j][k]);
      atomicAdd(&red[lane * 4 + j][4], dbl[j]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 128 * 5; i += blockDim.x) {
    const int ch = blockIdx.x * 128 + i / 5, k = i % 5;
    const float v = (&red[0][0])[i];
    if (k < 4) atomicAdd(dw + ch * 4 + k, v);
    else if (db) atomicAdd(db + ch, v);
  }
}

// ----------------------------------------------------------------- grad accumulate / embedding
template <typename T>
__global__ void accum_kernel(float* __restrict__ acc, const T* __restrict__ g, int64_t n, float scale) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    acc[i] += scale * to_f(g[i]);
}


// out[t, :] = emb[ids[t], :] (bf16 or fp32 table -> out dtype)
template <typename TI, typename TO>
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const TI* __restrict__ emb, TO* __restrict__ out,
                                 int64_t T, int D, int64_t V) {
  int64_t t = blockIdx.x;
  int64_t id = ids[t];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  for (int c = threadIdx.x; c < D; c += blockDim.x) out[t * D + c] = from_f<TO>(to_f(emb[id * D + c]));
}


template <typename T>
__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ dout, float* __restrict__ acc,
                                 int64_t T_, int D, int64_t V) {
  int64_t t = blockIdx.x;
  int64_t id = ids[t];
  if (id < 0 || id >= V) return;
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(acc + id * D + c, to_f(dout[t * D + c]));
}



// ===================================================================== launchers
static int sm_count() {
  static int n = 0;
  if (!n) { int d; cudaGetDevice(&d); cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d); }
  return n;
}
static int ew_blocks(int64_t n, int threads) {
  return (int)std::min<int64_t>((n + threads - 1) / threads, (int64_t)sm_count() * 16);
}

void ahb_sanitize(void* out, const void* in, int64_t n, int dtype, float clip, cudaStream_t st) {
  if (n == 0) return;
  if (dtype == AHB_BF16) sanitize_kernel<bf16><<<ew_blocks(n, 256), 256, 0, st>>>((bf16*)out, (const bf16*)in, n, clip);
  else sanitize_kernel<float><<<ew_blocks(n, 256), 256, 0, st>>>((float*)out, (const float*)in, n, clip);
}

static int rms_bwd_blocks(int64_t M, int D) {
  const int G = D <= 1024 ? 1 : (D <= 2048 ? 2 : (D <= 4096 ? 4 : 8));
  return (int)std::min<int64_t>((M + 8 / G - 1) / (8 / G), (int64_t)sm_count() * 2);
}

#define RMS_DISPATCH(KER, ...)                                                     \
  if (D <= 256) KER(T, 8, 1, __VA_ARGS__);                                         \
  else if (D <= 512) KER(T, 16, 1, __VA_ARGS__);                                   \
  else if (D <= 1024) KER(T, 32, 1, __VA_ARGS__);                                  \
  else if (D <= 2048) KER(T, 32, 2, __VA_ARGS__);                                  \
  else if (D <= 4096) KER(T, 32, 4, __VA_ARGS__);                                  \
  else KER(T, 32, 8, __VA_ARGS__);

#define RMS_F(T, V, G, _) rmsnorm_fwd_kernel<T, V, G><<<(unsigned)((M + 8 / G - 1) / (8 / G)), 256, 0, st>>>( \
    (const T*)x, s, (T*)y, r, M, D, eps)
template <typename T>
static void rms_fwd_t(const void* x, const float* s, void* y, float* r, int64_t M, int D, float eps, cudaStream_t st) {
  RMS_DISPATCH(RMS_F, 0)
}
#undef RMS_F
void ahb_rmsnorm_fwd(const void* x, const float* scale, void* y, float* rstd, int64_t M, int D, int dtype, float eps,
                     cudaStream_t st) {
  if (M == 0) return;
  if (D > 8192) return;
  if (dtype == AHB_BF16) rms_fwd_t<bf16>(x, scale, y, rstd, M, D, eps, st);
  else rms_fwd_t<float>(x, scale, y, rstd, M, D, eps, st);
}

#define RMS_B(T, V, G, _) rmsnorm_bwd_kernel<T, V, G><<<(unsigned)rms_bwd_blocks(M, D), 256, 0, st>>>( \
    (const T*)dy, (const T*)x, s, r, (T*)dx, ds, M, D)
template <typename T>
static void rms_bwd_t(const void* dy, const void* x, const float* s, const float* r, void* dx, float* ds, int64_t M,
                      int D, cudaStream_t st) {
  RMS_DISPATCH(RMS_B, 0)
}
#undef RMS_B
int ahb_rmsnorm_bwd_blocks(int64_t M, int D) { return rms_bwd_blocks(M, D); }

// dscale_part: zeroed fp32 scratch of ahb_rmsnorm_bwd_blocks(M, D) * D floats (or null);
// the column sums are added into dscale_acc.
void ahb_rmsnorm_bwd(const void* dy, const void* x, const float* scale, const float* rstd, void* dx, float* dscale_acc,
                     float* dscale_part, int64_t M, int D, int dtype, cudaStream_t st) {
  if (M == 0) return;
  float* ds = dscale_acc ? dscale_part : nullptr;
  if (dtype == AHB_BF16) rms_bwd_t<bf16>(dy, x, scale, rstd, dx, ds, M, D, st);
  else rms_bwd_t<float>(dy, x, scale, rstd, dx, ds, M, D, st);
  if (dscale_acc) colsum_add_kernel<<<(D + 31) / 32, 256, 0, st>>>(dscale_part, rms_bwd_blocks(M, D), D, dscale_acc);
}

void ahb_colsum_add(const float* part, int nb, int D, float* out, cudaStream_t st) {
  if (D <= 0 || nb <= 0) return;
  colsum_add_kernel<<<(D + 31) / 32, 256, 0, st>>>(part, nb, D, out);
}

void ahb_conv1d_fwd(const void* x, int64_t xs, const void* w, int wdtype, const float* bias, void* y, int B, int L,
                    int C, int dtype, int silu, float clip, cudaStream_t st) {
  if (dtype == AHB_BF16 && C % 128 == 0 && xs % 4 == 0 && B > 0 && L > 0) {
    const int64_t spans = (int64_t)B * ((L + CSPAN - 1) / CSPAN);
    const dim3 grid(C / 128, (unsigned)((spans + 7) / 8));
    if (wdtype == AHB_BF16)
      conv1d_fwd_stream_kernel<bf16><<<grid, 256, 0, st>>>((const bf16*)x, xs, (const bf16*)w, bias, (bf16*)y, B, L,
                                                           C, silu != 0, clip);
    else
      conv1d_fwd_stream_kernel<float><<<grid, 256, 0, st>>>((const bf16*)x, xs, (const float*)w, bias, (bf16*)y, B,
                                                            L, C, silu != 0, clip);
    return;
  }
  int64_t n = (int64_t)B * ((L + CONV_TT - 1) / CONV_TT) * (C / 8);
  if (n == 0) return;
  unsigned blocks = (unsigned)((n + 127) / 128);
#define CF(T, WT) conv1d_fwd_kernel<T, WT, 4><<<blocks, 128, 0, st>>>((const T*)x, xs, (const WT*)w, bias, (T*)y, B, L, C, silu != 0, clip)
  if (dtype == AHB_BF16) { if (wdtype == AHB_BF16) CF(bf16, bf16); else CF(bf16, float); }
  else { if (wdtype == AHB_BF16) CF(float, bf16); else CF(float, float); }
#undef CF
}

void ahb_conv1d_bwd(const void* x, int64_t xs, const void* w, int wdtype, const float* bias, const void* dy, void* dx,
                    float* dw_acc, float* db_acc, int B, int L, int C, int dtype, int silu, float clip,
                    cudaStream_t st) {
  if (dtype == AHB_BF16 && C % 128 == 0 && xs % 8 == 0 && B > 0 && L > 0) {
    const int64_t spans = (int64_t)B * ((L + CSPAN - 1) / CSPAN);
    const dim3 grid(C / 128, (unsigned)((spans + 7) / 8));
    constexpr int smem = 8 * 2 * CPF * 256 * 2;  // 8 warps x 2 buffers x CPF steps x (x + dy rows)
    static bool attr = false;
    if (!attr) {  // above the 48 KB default: opt in once per kernel
      cudaFuncSetAttribute(conv1d_bwd_pf_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      cudaFuncSetAttribute(conv1d_bwd_pf_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      attr = true;
    }
    if (wdtype == AHB_BF16)
      conv1d_bwd_pf_kernel<bf16><<<grid, 256, smem, st>>>((const bf16*)x, xs, (const bf16*)w, bias, (const bf16*)dy,
                                                          (bf16*)dx, (int64_t)C, dw_acc, db_acc, B, L, C, silu != 0,
                                                          clip);
    else
      conv1d_bwd_pf_kernel<float><<<grid, 256, smem, st>>>((const bf16*)x, xs, (const float*)w, bias,
                                                           (const bf16*)dy, (bf16*)dx, (int64_t)C, dw_acc, db_acc, B,
                                                           L, C, silu != 0, clip);
    return;
  }
  if (dtype == AHB_BF16 && C % 128 == 0 && xs % 4 == 0 && B > 0 && L > 0) {
    const int64_t spans = (int64_t)B * ((L + CSPAN - 1) / CSPAN);
    const dim3 grid(C / 128, (unsigned)((spans + 7) / 8));
    if (wdtype == AHB_BF16)
      conv1d_bwd_stream_kernel<bf16><<<grid, 256, 0, st>>>((const bf16*)x, xs, (const bf16*)w, bias, (const bf16*)dy,
                                                           (bf16*)dx, (int64_t)C, dw_acc, db_acc, B, L, C, silu != 0,
                                                           clip);
    else
      conv1d_bwd_stream_kernel<float><<<grid, 256, 0, st>>>((const bf16*)x, xs, (const float*)w, bias,
                                                            (const bf16*)dy, (bf16*)dx, (int64_t)C, dw_acc, db_acc, B,
                                                            L, C, silu != 0, clip);
    return;
  }
  int64_t n = (int64_t)B * ((L + CONV_TT * CONV_SUB - 1) / (CONV_TT * CONV_SUB)) * (C / 8);
  if (n == 0) return;
  unsigned blocks = (unsigned)((n + 127) / 128);
#define CB(T, WT) conv1d_bwd_kernel<T, WT, 4><<<blocks, 128, 0, st>>>((const T*)x, xs, (const WT*)w, bias, (const T*)dy, \
      (T*)dx, (int64_t)C, dw_acc, db_acc, B, L, C, silu != 0, clip)
  if (dtype == AHB_BF16) { if (wdtype == AHB_BF16) CB(bf16, bf16); else CB(bf16, float); }
  else { if (wdtype == AHB_BF16) CB(float, bf16); else CB(float, float); }
#undef CB
}

void ahb_accumulate(float* acc, const void* g, int64_t n, int dtype, float scale, cudaStream_t st) {
  if (n == 0) return;
  if (dtype == AHB_BF16) accum_kernel<bf16><<<ew_blocks(n, 256), 256, 0, st>>>(acc, (const bf16*)g, n, scale);
  else accum_kernel<float><<<ew_blocks(n, 256), 256, 0, st>>>(acc, (const float*)g, n, scale);
}

void ahb_embedding_fwd(const int64_t* ids, const void* emb, int edtype, void* out, int odtype, int64_t T, int D,
                       int64_t V, cudaStream_t st) {
  if (T == 0) return;
#define EF(TI, TO) embed_fwd_kernel<TI, TO><<<(unsigned)T, 256, 0, st>>>(ids, (const TI*)emb, (TO*)out, T, D, V)
  bool ib = edtype == AHB_BF16, ob = odtype == AHB_BF16;
  if (ib && ob) EF(bf16, bf16); else if (ib) EF(bf16, float); else if (ob) EF(float, bf16); else EF(float, float);
#undef EF
}

void ahb_embedding_bwd(const int64_t* ids, const void* dout, int dtype, float* acc, int64_t T, int D, int64_t V,
                       cudaStream_t st) {
  if (T == 0) return;
  if (dtype == AHB_BF16) embed_bwd_kernel<bf16><<<(unsigned)T, 256, 0, st>>>(ids, (const bf16*)dout, acc, T, D, V);
  else embed_bwd_kernel<float><<<(unsigned)T, 256, 0, st>>>(ids, (const float*)dout, acc, T, D, V);
}

// Shared-expert SwiGLU gate on the two up-projections (the SwiGLU configurations; the reference's
// shared expert, atomic_ops/moe_gmm.py:396-399, is the GELU variant):
// h = silu(a) * b in fp32 with one rounding, and its backward da = dh * b * silu'(a),
// db = dh * silu(a).  Eight bf16 elements per thread and step (n % 8 == 0).
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                                                         uint4* __restrict__ h, int64_t n8) {
  for (int64_t i = blockIdx.x * 256LL + threadIdx.x; i < n8; i += (int64_t)gridDim.x * 256) {
    const uint4 av = a[i], bv = b[i];
    const bf16* ap = reinterpret_cast<const bf16*>(&av);
    const bf16* bp = reinterpret_cast<const bf16*>(&bv);
    uint4 ov;
    bf16* op = reinterpret_cast<bf16*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) op[k] = __float2bfloat16_rn(siluf_(__bfloat162float(ap[k])) * __bfloat162float(bp[k]));
    h[i] = ov;
  }
}

__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const uint4* __restrict__ dh, const uint4* __restrict__ a,
                                                         const uint4* __restrict__ b, uint4* __restrict__ da,
                                                         uint4* __restrict__ db, int64_t n8) {
  for (int64_t i = blockIdx.x * 256LL + threadIdx.x; i < n8; i += (int64_t)gridDim.x * 256) {
    const uint4 dv = dh[i], av = a[i], bv = b[i];
    const bf16* dp = reinterpret_cast<const bf16*>(&dv);
    const bf16* ap = reinterpret_cast<const bf16*>(&av);
    const bf16* bp = reinterpret_cast<const bf16*>(&bv);
    uint4 dav, dbv;
    bf16* dap = reinterpret_cast<bf16*>(&dav);
    bf16* dbp = reinterpret_cast<bf16*>(&dbv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float x = __bfloat162float(ap[k]), g = __bfloat162float(dp[k]);
      const float sg = sigmoidf_(x);
      dap[k] = __float2bfloat16_rn(g * __bfloat162float(bp[k]) * sg * (1.f + x * (1.f - sg)));
      dbp[k] = __float2bfloat16_rn(g * x * sg);
    }
    da[i] = dav;
    db[i] = dbv;
  }
}

void ahb_swiglu_fwd(const void* a, const void* b, void* h, int64_t n, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 == 0) return;
  swiglu_fwd_kernel<<<ew_blocks(n8, 256), 256, 0, st>>>((const uint4*)a, (const uint4*)b, (uint4*)h, n8);
}

void ahb_swiglu_bwd(const void* dh, const void* a, const void* b, void* da, void* db, int64_t n, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 == 0) return;
  swiglu_bwd_kernel<<<ew_blocks(n8, 256), 256, 0, st>>>((const uint4*)dh, (const uint4*)a, (const uint4*)b, (uint4*)da,
                                                        (uint4*)db, n8);
}
