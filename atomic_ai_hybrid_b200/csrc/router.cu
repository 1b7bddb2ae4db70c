// Fused MoE router (reference `atomic_ops/moe_gmm.py:409-507`), forward and backward.
//
// Forward, per token t (x bf16 (T, d); kn fp32 (d, E) = router kernel with unit columns):
//   r_t = 1 / sqrt(|x_t|^2 + 1e-6);  cos_te = r_t * x_t . kn_e;  pre = cos * temp
//   l_te = sanitize(clamp(pre, +-8), 1e3) + noise_te
//   top-k of l + expert_bias (selection only); gate = softmax over the selected l
//   p = softmax(l) (aux loss), lse = logsumexp(l) (z loss)
// and the batch statistics: sum_t p_t (E), sum_t lse_t^2, expert counts, max |pre|,
// and sum / max / min of |x_t|.
//
// The reference computes the router in fp32.  The three router GEMMs run on the
// tensor cores (m16n8k16 bf16, fp32 accumulate) with fp32 operands split into
// bf16 terms: x is exact in bf16 and kn = hi + mid + lo (three terms), so every
// product of the forward is exact and only the fp32 accumulation order differs from
// an fp32 GEMM.  The backward products use two-term splits (relative error ~2^-16).
//
// Backward: per token, dl from the gate softmax, the aux-loss softmax and the
// z-loss; dpre = dl masked by the clamp; dtemp = sum dpre * cos; dcos = dpre * temp;
// dx = sanitize(r * (dxn - xn (xn . dxn)), 1e3) with dxn = dcos kn^T (the grad
// sanitizer on the router input); dkn = sum_t x_t^T (r_t dcos_t).
//
// Experts are padded to EP = 16 * ceil(E / 16) <= 64 inside the kernels (zero
// kernel columns); the padded columns never reach an output.
#include "common.cuh"
#include "launchers.h"
#include "mma.cuh"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

constexpr int TOKC = 64;   // tokens per CTA (4 warps x 16)
constexpr int DS = 64;     // d slice staged per step
constexpr int NT = 128;    // threads
constexpr int EMAX = 64;
constexpr int LDX = DS + 8;  // bf16 row stride of staged tiles (bank spread, 16-byte rows)

AHB_DEVICE void atomic_max_pos(float* a, float v) { atomicMax(reinterpret_cast<int*>(a), __float_as_int(v)); }
AHB_DEVICE void atomic_min_pos(float* a, float v) { atomicMin(reinterpret_cast<int*>(a), __float_as_int(v)); }

// ------------------------------------------------------------------ forward
// knT: 3 x (EP, d) bf16 (hi, mid, lo of kn^T).
AHB_DEVICE void cp16z(void* dst, const void* src, bool valid) {  // zero-filled when !valid
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(dst);
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(src), "r"(n) : "memory");
}
AHB_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
AHB_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int NTE>
__host__ __device__ constexpr size_t fwd_stage_bytes() { return (size_t)(TOKC + 3 * NTE * 8) * LDX * 2; }
template <int NTE>
__host__ __device__ constexpr size_t fwd_smem_bytes() {
  return 2 * fwd_stage_bytes<NTE>() > (size_t)TOKC * (NTE * 8 + 1) * 4 ? 2 * fwd_stage_bytes<NTE>()
                                                                       : (size_t)TOKC * (NTE * 8 + 1) * 4;
}

// The x and kn slices are double-buffered with cp.async: slice s+1 loads while slice s multiplies.
template <int NTE>
__global__ void __launch_bounds__(NT) router_fwd_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ knT, const float* __restrict__ temp_p,
    const float* __restrict__ bias, const float* __restrict__ noise, int64_t T, int d, int E, int k,
    float* __restrict__ logits, float* __restrict__ cosv, float* __restrict__ rn_out, int64_t* __restrict__ top_idx,
    float* __restrict__ gate, float* __restrict__ probs_sum, float* __restrict__ scal, float* __restrict__ counts) {
  constexpr int EP = NTE * 8;
  constexpr size_t STAGE = fwd_stage_bytes<NTE>();
  // two staged (x, kn) slices; after the loop the same memory holds the logits rows
  extern __shared__ __align__(16) unsigned char raw[];
  float(*cs)[EP + 1] = reinterpret_cast<float(*)[EP + 1]>(raw);
  __shared__ float ssh[TOKC];
  __shared__ float psum[EMAX], csum[EMAX];
  const int64_t t0 = (int64_t)blockIdx.x * TOKC;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  auto xs_of = [&](int sl) { return reinterpret_cast<bf16*>(raw + sl * STAGE); };
  auto ks_of = [&](int sl) { return xs_of(sl) + TOKC * LDX; };
  auto issue = [&](int c0, int sl) {
    bf16* xs = xs_of(sl);
    bf16* ks = ks_of(sl);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = tid + NT * q, r = idx >> 3, c8 = (idx & 7) * 8;
      const int64_t t = t0 + r;
      cp16z(xs + r * LDX + c8, x + (t < T ? t : 0) * d + c0 + c8, t < T);
    }
    for (int idx = tid; idx < 3 * EP * 8; idx += NT) {
      const int s = idx / (EP * 8), rem = idx % (EP * 8), e = rem >> 3, c8 = (rem & 7) * 8;
      cp16z(ks + (s * EP + e) * LDX + c8, knT + ((int64_t)s * EP + e) * d + c0 + c8, true);
    }
    cp_commit();
  };
  float acc[NTE][4];
  zero_acc<NTE>(acc);
  float ss[4] = {0.f, 0.f, 0.f, 0.f};  // rows (tid >> 3) + 16 q of every x slice
  const int nsl = d / DS;
  issue(0, 0);
  for (int si = 0; si < nsl; ++si) {
    if (si + 1 < nsl) {
      issue((si + 1) * DS, (si + 1) & 1);  // the other stage was released by the previous barrier
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const bf16* xs = xs_of(si & 1);
    const bf16* ks = ks_of(si & 1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = tid + NT * q, r = idx >> 3, c8 = (idx & 7) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(xs + r * LDX + c8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        ss[q] += f.x * f.x + f.y * f.y;
      }
    }
#pragma unroll
    for (int s = 0; s < 3; ++s) warp_mma<NTE>(acc, RowA16{xs, LDX}, NKB16{ks + s * EP * LDX, LDX}, 16 * w, 0, 0, DS);
    __syncthreads();
  }
  for_acc<NTE>(acc, 16 * w, 0, [&](int r, int c, float& v) { cs[r][c] = v; });
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float v = ss[q];
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 7) == 0) ssh[(tid >> 3) + 16 * q] = v;
  }
  for (int e = tid; e < EMAX; e += NT) psum[e] = csum[e] = 0.f;
  __syncthreads();

  const float temp = *temp_p;
  float lse_sq = 0.f, pre_max = 0.f, nsum = 0.f, nmax = 0.f, nmin = 3.0e38f;
  for (int r = w; r < TOKC; r += NT / 32) {
    const int64_t t = t0 + r;
    if (t >= T) break;
    const float rn = rsqrtf(ssh[r] + 1e-6f);
    const float nrm = sqrtf(ssh[r]);
    nsum += nrm;
    nmax = fmaxf(nmax, nrm);
    nmin = fminf(nmin, nrm);
    if (lane == 0) rn_out[t] = rn;
    float l[2], b[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      l[h] = -INFINITY;
      b[h] = -INFINITY;
      if (e < E) {
        const float c = cs[r][e] * rn;
        const float pre = c * temp;
        pre_max = fmaxf(pre_max, fabsf(pre));
        float lv = sanitize(fminf(fmaxf(pre, -8.f), 8.f), 1e3f);
        if (noise) lv += noise[t * E + e];
        cosv[t * E + e] = c;
        logits[t * E + e] = lv;
        l[h] = lv;
        b[h] = lv + bias[e];
      }
    }
    const float m = warp_max(fmaxf(l[0], l[1]));
    const float p0 = l[0] > -INFINITY ? __expf(l[0] - m) : 0.f, p1 = l[1] > -INFINITY ? __expf(l[1] - m) : 0.f;
    const float z = warp_sum(p0 + p1);
    const float lse = m + __logf(z);
    lse_sq += lse * lse;  // identical on every lane
    if (lane < E) atomicAdd(&psum[lane], p0 / z);
    if (lane + 32 < E) atomicAdd(&psum[lane + 32], p1 / z);
    // top-k of the biased logits (ties: lowest expert index); gate over the unbiased ones
    float sel_l[8];
    int sel_e[8];
    float gm = -INFINITY;
    for (int j = 0; j < k; ++j) {
      float bv = b[0];
      int be = lane;
      if (b[1] > bv) {
        bv = b[1];
        be = lane + 32;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ov > bv || (ov == bv && oe < be)) {
          bv = ov;
          be = oe;
        }
      }
      sel_e[j] = be;
      sel_l[j] = __shfl_sync(0xffffffffu, be < 32 ? l[0] : l[1], be & 31);
      if ((be & 31) == lane) b[be >> 5] = -INFINITY;
      gm = fmaxf(gm, sel_l[j]);
    }
    if (lane == 0) {
      float zs = 0.f;
      for (int j = 0; j < k; ++j) zs += __expf(sel_l[j] - gm);
      for (int j = 0; j < k; ++j) {
        top_idx[t * k + j] = sel_e[j];
        gate[t * k + j] = __expf(sel_l[j] - gm) / zs;
        atomicAdd(&csum[sel_e[j]], 1.f);
      }
    }
  }
  // every lane of a warp saw the same tokens: lane 0's per-token sums stand for the warp
  const float pm = warp_max(pre_max);
  if (lane == 0) {
    atomicAdd(scal + 0, lse_sq);
    atomic_max_pos(scal + 1, pm);
    atomicAdd(scal + 2, nsum);
    atomic_max_pos(scal + 3, nmax);
    atomic_min_pos(scal + 4, nmin);
  }
  __syncthreads();
  for (int e = tid; e < E; e += NT) {
    atomicAdd(probs_sum + e, psum[e]);
    atomicAdd(counts + e, csum[e]);
  }
}

// ------------------------------------------------------------------ backward: dcos, dtemp, dx
// kn2: 2 x (d, EP) bf16 (hi, mid of kn).  dcos_out (T, EP) fp32 with zero padding.
template <int NTE>
__global__ void __launch_bounds__(NT) router_bwd_tokens_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ kn2, const float* __restrict__ temp_p,
    const float* __restrict__ logits, const float* __restrict__ cosv, const float* __restrict__ rn_in,
    const int64_t* __restrict__ top_idx, const float* __restrict__ gate, const float* __restrict__ dgate,
    const float* __restrict__ dps, const float* __restrict__ dlse_sq_p, int64_t T, int d, int E, int k,
    float* __restrict__ dcos_out, float* __restrict__ dtemp, bf16* __restrict__ dx) {
  constexpr int EP = NTE * 8;
  constexpr int KS = (EP + 15) / 16;  // k-steps over the (padded) experts
  __shared__ float dc[TOKC][EMAX + 1];
  const int64_t t0 = (int64_t)blockIdx.x * TOKC;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const float temp = *temp_p;
  const float dlse_sq = dlse_sq_p ? *dlse_sq_p : 0.f;
  for (int i = tid; i < TOKC * (EMAX + 1); i += NT) (&dc[0][0])[i] = 0.f;
  __syncthreads();
  float dtp = 0.f;
  for (int r = w; r < TOKC; r += NT / 32) {
    const int64_t t = t0 + r;
    if (t >= T) break;
    float l[2], p[2], dl[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      l[h] = e < E ? logits[t * E + e] : -INFINITY;
    }
    const float m = warp_max(fmaxf(l[0], l[1]));
    p[0] = l[0] > -INFINITY ? __expf(l[0] - m) : 0.f;
    p[1] = l[1] > -INFINITY ? __expf(l[1] - m) : 0.f;
    const float z = warp_sum(p[0] + p[1]);
    const float lse = m + __logf(z);
    p[0] /= z;
    p[1] /= z;
    float pd = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      pd += e < E ? p[h] * dps[e] : 0.f;
    }
    pd = warp_sum(pd);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      dl[h] = e < E ? p[h] * (dps[e] - pd) + dlse_sq * 2.f * lse * p[h] : 0.f;
    }
    float gd = 0.f;
    for (int j = 0; j < k; ++j) gd += gate[t * k + j] * dgate[t * k + j];
    for (int j = 0; j < k; ++j) {
      const int e = (int)top_idx[t * k + j];
      const float v = gate[t * k + j] * (dgate[t * k + j] - gd);
      if ((e & 31) == lane) dl[e >> 5] += v;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      if (e < EP) {
        float d_c = 0.f;
        if (e < E) {
          const float c = cosv[t * E + e];
          const float dpre = fabsf(c * temp) <= 8.f ? dl[h] : 0.f;
          dtp += dpre * c;
          d_c = dpre * temp;
        }
        dc[r][e] = d_c;
        dcos_out[t * EP + e] = d_c;
      }
    }
  }
  dtp = warp_sum(dtp);
  if (lane == 0) atomicAdd(dtemp, dtp);
  __syncthreads();
  // dxn = dcos kn^T for the warp's 16 tokens: A = dcos (hi + lo), B(e, c) = kn[c][e] (hi + mid)
  uint32_t ahi[KS][4], alo[KS][4];
  {
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int kc[4][2] = {{g, 16 * s + 2 * tq}, {g + 8, 16 * s + 2 * tq}, {g, 16 * s + 2 * tq + 8},
                            {g + 8, 16 * s + 2 * tq + 8}};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = 16 * w + kc[i][0], cc = kc[i][1];
        const float v0 = cc < EP ? dc[rr][cc] : 0.f, v1 = cc + 1 < EP ? dc[rr][cc + 1] : 0.f;
        const __nv_bfloat162 hi = __floats2bfloat162_rn(v0, v1);
        const float2 hf = __bfloat1622float2(hi);
        ahi[s][i] = *reinterpret_cast<const uint32_t*>(&hi);
        alo[s][i] = pack2(v0 - hf.x, v1 - hf.y);
      }
    }
  }
  const int g = lane >> 2, tq = lane & 3;
  const int64_t ta = t0 + 16 * w + g, tb = ta + 8;
  const float rna = ta < T ? rn_in[ta] : 0.f, rnb = tb < T ? rn_in[tb] : 0.f;
  const bf16* khi = kn2;
  const bf16* kmid = kn2 + (int64_t)d * EP;
  float dot_a = 0.f, dot_b = 0.f;
  for (int pass = 0; pass < 2; ++pass) {
    for (int n0 = 0; n0 < d; n0 += 64) {
      float acc[8][4];
      zero_acc<8>(acc);
#pragma unroll
      for (int s = 0; s < KS; ++s) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = n0 + 8 * j + g;
          const int kk = 16 * s + 2 * tq;
          uint32_t bh[2], bm[2];
          bh[0] = kk < EP ? *reinterpret_cast<const uint32_t*>(khi + (int64_t)col * EP + kk) : 0u;
          bh[1] = kk + 8 < EP ? *reinterpret_cast<const uint32_t*>(khi + (int64_t)col * EP + kk + 8) : 0u;
          bm[0] = kk < EP ? *reinterpret_cast<const uint32_t*>(kmid + (int64_t)col * EP + kk) : 0u;
          bm[1] = kk + 8 < EP ? *reinterpret_cast<const uint32_t*>(kmid + (int64_t)col * EP + kk + 8) : 0u;
          mma16816(acc[j], ahi[s], bh);
          mma16816(acc[j], ahi[s], bm);
          mma16816(acc[j], alo[s], bh);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = n0 + 8 * j + 2 * tq;
        const float2 xa = ta < T ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x + ta * d + c))
                                 : make_float2(0.f, 0.f);
        const float2 xb = tb < T ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x + tb * d + c))
                                 : make_float2(0.f, 0.f);
        if (pass == 0) {
          dot_a += xa.x * acc[j][0] + xa.y * acc[j][1];
          dot_b += xb.x * acc[j][2] + xb.y * acc[j][3];
        } else {
          if (ta < T)
            *reinterpret_cast<__nv_bfloat162*>(dx + ta * d + c) = __floats2bfloat162_rn(
                sanitize(rna * acc[j][0] - xa.x * rna * rna * rna * dot_a, 1e3f),
                sanitize(rna * acc[j][1] - xa.y * rna * rna * rna * dot_a, 1e3f));
          if (tb < T)
            *reinterpret_cast<__nv_bfloat162*>(dx + tb * d + c) = __floats2bfloat162_rn(
                sanitize(rnb * acc[j][2] - xb.x * rnb * rnb * rnb * dot_b, 1e3f),
                sanitize(rnb * acc[j][3] - xb.y * rnb * rnb * rnb * dot_b, 1e3f));
        }
      }
    }
    if (pass == 0) {  // the 4 lanes of a row share it
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        dot_a += __shfl_xor_sync(0xffffffffu, dot_a, o);
        dot_b += __shfl_xor_sync(0xffffffffu, dot_b, o);
      }
    }
  }
}

// ------------------------------------------------------------------ backward: dkn
// dkn[c][e] += sum_t x[t][c] (r_t dcos[t][e]); CTA = 64 columns of d (4 warps x 16) x a token range.
template <int NTE>
__global__ void __launch_bounds__(NT) router_bwd_kn_kernel(const bf16* __restrict__ x,
                                                          const float* __restrict__ rn_in,
                                                          const float* __restrict__ dcos, int64_t T, int d,
                                                          int E, int64_t tok_per_cta, float* __restrict__ dkn) {
  constexpr int EP = NTE * 8;
  constexpr int TC = 32;  // tokens per staged chunk
  __shared__ __align__(16) bf16 xs[TC * LDX];
  __shared__ bf16 bh[TC][EP + 2], bl[TC][EP + 2];
  const int c0 = blockIdx.x * 64;
  const int64_t ta = (int64_t)blockIdx.y * tok_per_cta;
  const int64_t tb = ta + tok_per_cta < T ? ta + tok_per_cta : T;
  const int tid = threadIdx.x, w = tid >> 5;
  float acc[NTE][4];
  zero_acc<NTE>(acc);
  for (int64_t q0 = ta; q0 < tb; q0 += TC) {
    __syncthreads();
    for (int idx = tid; idx < TC * 8; idx += NT) {
      const int r = idx >> 3, c8 = (idx & 7) * 8;
      const int64_t t = q0 + r;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (t < tb) u = *reinterpret_cast<const uint4*>(x + t * d + c0 + c8);
      *reinterpret_cast<uint4*>(xs + r * LDX + c8) = u;
    }
    for (int idx = tid; idx < TC * EP; idx += NT) {
      const int r = idx / EP, e = idx % EP;
      const int64_t t = q0 + r;
      const float v = t < tb ? dcos[t * EP + e] * rn_in[t] : 0.f;
      const bf16 h = __float2bfloat16_rn(v);
      bh[r][e] = h;
      bl[r][e] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
    __syncthreads();
    // A(m = column, k = token) = xs[k][m]; B(k = token, n = expert) = b[k][n]
    warp_mma<NTE>(acc, ColA16{xs, LDX}, KNB16{&bh[0][0], EP + 2}, 16 * w, 0, 0, TC);
    warp_mma<NTE>(acc, ColA16{xs, LDX}, KNB16{&bl[0][0], EP + 2}, 16 * w, 0, 0, TC);
  }
  for_acc<NTE>(acc, 16 * w, 0, [&](int r, int c, float& v) {
    if (c < E) atomicAdd(dkn + (int64_t)(c0 + r) * E + c, v);
  });
}

int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

int ahb_router_supported(int d, int E, int k) {
  return d % 64 == 0 && E >= 2 && E <= EMAX && k >= 1 && k <= 8 && k <= E;
}

int ahb_router_padded_experts(int E) { return (E + 15) / 16 * 16; }

void ahb_router_fwd(const void* x, const void* knT3, const float* temp, const float* bias, const float* noise,
                    int64_t T, int d, int E, int k, float* logits, float* cosv, float* rn, int64_t* top_idx,
                    float* gate, float* probs_sum, float* scal, float* counts, cudaStream_t st) {
  if (T <= 0) return;
  const int grid = (int)((T + TOKC - 1) / TOKC);
  const int EP = ahb_router_padded_experts(E);
#define RF(N)                                                                                                   \
  do {                                                                                                          \
    static bool init = false;                                                                                   \
    if (!init) {                                                                                                \
      cudaFuncSetAttribute(router_fwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,                    \
                           (int)fwd_smem_bytes<N>());                                                           \
      init = true;                                                                                              \
    }                                                                                                           \
    router_fwd_kernel<N><<<grid, NT, fwd_smem_bytes<N>(), st>>>((const bf16*)x, (const bf16*)knT3, temp, bias,   \
                                                               noise, T, d, E, k, logits, cosv, rn, top_idx, gate, \
                                                               probs_sum, scal, counts);                        \
  } while (0)
  if (EP == 16) RF(2); else if (EP == 32) RF(4); else if (EP == 48) RF(6); else RF(8);
#undef RF
}

void ahb_router_bwd(const void* x, const void* kn2, const float* temp, const float* logits, const float* cosv,
                    const float* rn, const int64_t* top_idx, const float* gate, const float* dgate, const float* dps,
                    const float* dlse_sq, int64_t T, int d, int E, int k, float* dcos, float* dtemp, void* dx,
                    float* dkn, cudaStream_t st) {
  if (T <= 0) return;
  const int grid = (int)((T + TOKC - 1) / TOKC);
  const int EP = ahb_router_padded_experts(E);
#define RB(N) router_bwd_tokens_kernel<N><<<grid, NT, 0, st>>>((const bf16*)x, (const bf16*)kn2, temp, logits, cosv, \
    rn, top_idx, gate, dgate, dps, dlse_sq, T, d, E, k, dcos, dtemp, (bf16*)dx)
  if (EP == 16) RB(2); else if (EP == 32) RB(4); else if (EP == 48) RB(6); else RB(8);
#undef RB
  const int nx = d / 64;
  int ny = (2 * sm_count() + nx - 1) / nx;
  const int64_t per = ((T + ny - 1) / ny + 31) / 32 * 32;
  ny = (int)((T + per - 1) / per);
#define RK(N) router_bwd_kn_kernel<N><<<dim3(nx, ny), NT, 0, st>>>((const bf16*)x, rn, dcos, T, d, E, per, dkn)
  if (EP == 16) RK(2); else if (EP == 32) RK(4); else if (EP == 48) RK(6); else RK(8);
#undef RK
}
