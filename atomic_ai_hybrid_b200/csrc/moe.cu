// MoE dispatch / combine kernels (dropless, reference `atomic_ops/moe_gmm.py:515-583`).
//
// Assignments are ordered like the reference's replicated token matrix:
// a = j*T + t for top-k choice j of token t.  Rows of the expert-sorted matrix
// keep that order inside each expert (a stable sort by expert id), and every
// expert's segment is padded to a multiple of 128 rows (256 for the CTA-pair
// GEMMs) so the grouped GEMM's tiles never straddle two experts; padding rows are zero.
#include "common.cuh"
#include "launchers.h"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

// counts[e] = #assignments to expert e  (grid E, block 1024)
__global__ void __launch_bounds__(1024) moe_count_kernel(const int* __restrict__ eidx, int64_t n, int* __restrict__ counts) {
  __shared__ float sh[32];
  const int e = blockIdx.x;
  float c = 0.f;
  for (int64_t a = threadIdx.x; a < n; a += blockDim.x) c += (eidx[a] == e) ? 1.f : 0.f;
  c = block_sum(c, sh);
  if (threadIdx.x == 0) counts[e] = (int)c;
}

// offsets (E+1) of the padded segments (single block)
__global__ void moe_offsets_kernel(const int* __restrict__ counts, int E, int pad, int* __restrict__ off) {
  if (threadIdx.x == 0) {
    int s = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = s;
      s += (counts[e] + pad - 1) / pad * pad;
    }
    off[E] = s;
  }
}

// pos[a] = off[e] + stable rank of a among assignments to e; row_src[pos] = token (grid E, block 1024).
// Each pass covers 4096 assignments, four consecutive ones per thread (one 16-byte load): the rank is
// the thread's own prefix, plus a warp shuffle scan of the per-thread counts, plus an exclusive scan
// of the 32 warp totals.
__global__ void __launch_bounds__(1024) moe_positions_kernel(const int* __restrict__ eidx, int64_t n, int T,
                                                             const int* __restrict__ off, int* __restrict__ pos,
                                                             int* __restrict__ row_src) {
  __shared__ int warp_ex[32];
  __shared__ int pass_tot;
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int base = off[e];
  int carry = 0;  // rows of expert e in the passes before (the same in every thread)
  for (int64_t a0 = 0; a0 < n; a0 += 4 * 1024) {
    const int64_t a = a0 + 4 * (int64_t)threadIdx.x;
    int f[4];
    if (a + 3 < n) {
      const int4 v = *reinterpret_cast<const int4*>(eidx + a);
      f[0] = v.x == e; f[1] = v.y == e; f[2] = v.z == e; f[3] = v.w == e;
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) f[q] = (a + q < n && eidx[a + q] == e) ? 1 : 0;
    }
    const int cnt = f[0] + f[1] + f[2] + f[3];
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_ex[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      const int v = warp_ex[lane];
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      warp_ex[lane] = inc - v;
      if (lane == 31) pass_tot = inc;
    }
    __syncthreads();
    int r = base + carry + warp_ex[wid] + incl - cnt;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (f[q]) {
        pos[a + q] = r;
        row_src[r] = (int)((a + q) % T);
        ++r;
      }
    carry += pass_tot;
    __syncthreads();  // warp_ex and pass_tot are rewritten by the next pass
  }
}

// xs[r] = row_src[r] >= 0 ? x[row_src[r]] : 0   (one warp per row, 16-byte vectors)
__global__ void moe_gather_kernel(const bf16* __restrict__ x, const int* __restrict__ row_src, int64_t R, int d,
                                  bf16* __restrict__ xs) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= R) return;
  const int lane = threadIdx.x & 31;
  const int src = row_src[r];
  uint4* dst = reinterpret_cast<uint4*>(xs + r * d);
  const uint4* s = reinterpret_cast<const uint4*>(x + (int64_t)(src < 0 ? 0 : src) * d);
  for (int c = lane; c < d / 8; c += 32) dst[c] = src >= 0 ? s[c] : make_uint4(0, 0, 0, 0);
}

// One token per CTA, d/8 threads, 16-byte vectors (8 bf16 channels per thread).
AHB_DEVICE void ld8f(const bf16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
AHB_DEVICE void st8f(bf16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// out[t] = sanitize(shared[t] + sum_j gate[t,j] * sanitize(ys[pos[j*T+t]], 1e3), 1e3):
// routed rows are clipped +-1e3 (reference sanitize after the second gmm), the sum again.
__global__ void moe_combine_kernel(const bf16* __restrict__ ys, const int* __restrict__ pos, const float* __restrict__ gate,
                                   const bf16* __restrict__ shared, int T, int k, int d, bf16* __restrict__ out) {
  const int t = blockIdx.x;
  const int c = threadIdx.x * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const int p = pos[(int64_t)j * T + t];
    const float g = gate[(int64_t)t * k + j];
    float v[8];
    ld8f(ys + (int64_t)p * d + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += g * sanitize(v[i], 1e3f);
  }
  if (shared) {
    float v[8];
    ld8f(shared + (int64_t)t * d + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = sanitize(acc[i], 1e3f);
  st8f(out + (int64_t)t * d + c, acc);
}

// dys[pos[a]] = gate[a] * dout[t];  dgate[t,j] = <dout[t], sanitize(ys[pos[a]])>
__global__ void moe_combine_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ ys,
                                       const int* __restrict__ pos, const float* __restrict__ gate, int T, int k,
                                       int d, bf16* __restrict__ dys, float* __restrict__ dgate) {
  __shared__ float sh[32][8];
  const int t = blockIdx.x;
  const int c = threadIdx.x * 8;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float dv[8];
  ld8f(dout + (int64_t)t * d + c, dv);
  float dots[8];
  for (int j = 0; j < k; ++j) {
    const int p = pos[(int64_t)j * T + t];
    const float g = gate[(int64_t)t * k + j];
    float yv[8], o[8];
    ld8f(ys + (int64_t)p * d + c, yv);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i] = g * dv[i];
      dot += dv[i] * sanitize(yv[i], 1e3f);
    }
    st8f(dys + (int64_t)p * d + c, o);
    dots[j] = warp_sum(dot);
  }
  if (lane == 0)
    for (int j = 0; j < k; ++j) sh[w][j] = dots[j];
  __syncthreads();
  if (threadIdx.x < k) {
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += sh[i][threadIdx.x];
    dgate[(int64_t)t * k + threadIdx.x] = s;
  }
}

// dx[t] = sum_j dxs[pos[j*T+t]]
__global__ void moe_scatter_add_kernel(const bf16* __restrict__ dxs, const int* __restrict__ pos, int T, int k, int d,
                                       bf16* __restrict__ dx) {
  const int t = blockIdx.x;
  const int c = threadIdx.x * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    float v[8];
    ld8f(dxs + (int64_t)pos[(int64_t)j * T + t] * d + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  st8f(dx + (int64_t)t * d + c, acc);
}

// zero the padding rows of a (R, d) bf16 matrix (rows with row_src < 0)
__global__ void moe_zero_pad_kernel(bf16* __restrict__ m, const int* __restrict__ row_src, int64_t R, int d) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= R || row_src[r] >= 0) return;
  uint4* dst = reinterpret_cast<uint4*>(m + r * d);
  for (int c = threadIdx.x & 31; c < d / 8; c += 32) dst[c] = make_uint4(0, 0, 0, 0);
}

}  // namespace

void ahb_moe_route(const int* eidx, int T, int k, int E, int* counts, int* off, int* pos, int* row_src, int64_t R_cap,
                   cudaStream_t st, int pad) {
  const int64_t n = (int64_t)T * k;
  cudaMemsetAsync(row_src, 0xff, R_cap * sizeof(int), st);
  moe_count_kernel<<<E, 1024, 0, st>>>(eidx, n, counts);
  moe_offsets_kernel<<<1, 32, 0, st>>>(counts, E, pad, off);
  moe_positions_kernel<<<E, 1024, 0, st>>>(eidx, n, T, off, pos, row_src);
}

void ahb_moe_gather(const void* x, const int* row_src, int64_t R, int d, void* xs, cudaStream_t st) {
  if (!R) return;
  moe_gather_kernel<<<(unsigned)((R + 7) / 8), 256, 0, st>>>((const bf16*)x, row_src, R, d, (bf16*)xs);
}

void ahb_moe_zero_pad(void* m, const int* row_src, int64_t R, int d, cudaStream_t st) {
  if (!R) return;
  moe_zero_pad_kernel<<<(unsigned)((R + 7) / 8), 256, 0, st>>>((bf16*)m, row_src, R, d);
}

void ahb_moe_combine(const void* ys, const int* pos, const float* gate, const void* shared, int T, int k, int d,
                     void* out, cudaStream_t st) {
  if (!T) return;
  moe_combine_kernel<<<T, d / 8, 0, st>>>((const bf16*)ys, pos, gate, (const bf16*)shared, T, k, d, (bf16*)out);
}

void ahb_moe_combine_bwd(const void* dout, const void* ys, const int* pos, const float* gate, int T, int k, int d,
                         void* dys, float* dgate, cudaStream_t st) {
  if (!T) return;
  moe_combine_bwd_kernel<<<T, d / 8, 0, st>>>((const bf16*)dout, (const bf16*)ys, pos, gate, T, k, d, (bf16*)dys,
                                            dgate);
}

void ahb_moe_scatter_add(const void* dxs, const int* pos, int T, int k, int d, void* dx, cudaStream_t st) {
  if (!T) return;
  moe_scatter_add_kernel<<<T, d / 8, 0, st>>>((const bf16*)dxs, pos, T, k, d, (bf16*)dx);
}
