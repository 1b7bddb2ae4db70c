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
// kn2: 2 x (d, EP) bf16 (hi, mid of kn).  bhl_out (T, 2 EP) bf16: the hi and lo terms of r_t dcos_t
// (the operand of the dkn kernel), zero on padded experts.
//
// Per token: dl, dcos, dtemp as in the forward's statistics; then dx = sanitize(r dxn - x r^2 S, 1e3)
// with dxn = dcos kn^T and S = sum_e dcos_e cos_e (= r x . dxn, since cos_e = r x . kn_e: the dot
// product needs no second pass over d).  The d columns run in slices of 64: the slice of kn (hi and
// mid) and of x are staged by cp.async one slice ahead, dx goes out through a shared tile as 16-byte
// row segments.
constexpr int RB_SL = 64;           // d columns per slice
constexpr int RB_XS = RB_SL + 8;    // bf16 stride of the x / dx tiles (16-byte rows, spread banks)

template <int NTE>
struct RbLayout {
  static constexpr int EP = NTE * 8;
  static constexpr int KS = EP + 8;  // bf16 stride of a staged kn row
  static constexpr size_t DC = 0;                                         // float [TOKC][EMAX + 1]
  static constexpr size_t SS = DC + (size_t)TOKC * (EMAX + 1) * 4;        // float [TOKC]
  static constexpr size_t KN = SS + (size_t)TOKC * 4;                     // bf16 [2 buf][2 term][RB_SL][KS]
  static constexpr size_t XT = KN + (size_t)2 * 2 * RB_SL * KS * 2;       // bf16 [2 buf][TOKC][RB_XS]
  static constexpr size_t OT = XT + (size_t)2 * TOKC * RB_XS * 2;         // bf16 [TOKC][RB_XS]
  static constexpr size_t BYTES = OT + (size_t)TOKC * RB_XS * 2;
};

template <int NTE>
__global__ void __launch_bounds__(NT) router_bwd_tokens_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ kn2, const float* __restrict__ temp_p,
    const float* __restrict__ logits, const float* __restrict__ cosv, const float* __restrict__ rn_in,
    const int64_t* __restrict__ top_idx, const float* __restrict__ gate, const float* __restrict__ dgate,
    const float* __restrict__ dps, const float* __restrict__ dlse_sq_p, int64_t T, int d, int E, int k,
    bf16* __restrict__ bhl_out, float* __restrict__ dtemp, bf16* __restrict__ dx) {
  using Lay = RbLayout<NTE>;
  constexpr int EP = Lay::EP;
  constexpr int KSTEPS = (EP + 15) / 16;  // k-steps over the (padded) experts
  extern __shared__ __align__(16) unsigned char rb_smem[];
  float(*dc)[EMAX + 1] = reinterpret_cast<float(*)[EMAX + 1]>(rb_smem + Lay::DC);
  float* Srow = reinterpret_cast<float*>(rb_smem + Lay::SS);
  bf16* knt = reinterpret_cast<bf16*>(rb_smem + Lay::KN);
  bf16* xt = reinterpret_cast<bf16*>(rb_smem + Lay::XT);
  bf16* ot = reinterpret_cast<bf16*>(rb_smem + Lay::OT);
  const int64_t t0 = (int64_t)blockIdx.x * TOKC;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const float temp = *temp_p;
  const float dlse_sq = dlse_sq_p ? *dlse_sq_p : 0.f;
  const int nsl = d / RB_SL;
  // stage slice `sl` of kn (rows c, hi and mid) and of x (the CTA's 64 tokens) into buffer sl & 1
  auto issue = [&](int sl) {
    bf16* kb = knt + (size_t)(sl & 1) * 2 * RB_SL * Lay::KS;
    bf16* xb = xt + (size_t)(sl & 1) * TOKC * RB_XS;
    constexpr int KCH = EP / 8;  // 16-byte chunks per kn row
    for (int i = tid; i < 2 * RB_SL * KCH; i += NT) {
      const int term = i / (RB_SL * KCH), r = (i / KCH) % RB_SL, q = i % KCH;
      const bf16* src = kn2 + (int64_t)term * d * EP + (int64_t)(sl * RB_SL + r) * EP + 8 * q;
      cp16z(kb + (term * RB_SL + r) * Lay::KS + 8 * q, src, true);
    }
    for (int i = tid; i < TOKC * (RB_SL / 8); i += NT) {
      const int r = i / (RB_SL / 8), q = i % (RB_SL / 8);
      const int64_t t = t0 + r;
      cp16z(xb + r * RB_XS + 8 * q, x + (t < T ? t : 0) * d + sl * RB_SL + 8 * q, t < T);
    }
    cp_commit();
  };
  issue(0);  // the first slice loads while the per-token part runs
  for (int i = tid; i < TOKC * (EMAX + 1); i += NT) (&dc[0][0])[i] = 0.f;
  __syncthreads();
  float dtp = 0.f;
  for (int r = w; r < TOKC; r += NT / 32) {
    const int64_t t = t0 + r;
    if (t >= T) {
      if (lane == 0) Srow[r] = 0.f;
      continue;
    }
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
    const float rt = rn_in[t];
    float sdot = 0.f;
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
          sdot += d_c * c;
        }
        dc[r][e] = d_c;
        const float v = rt * d_c;
        const bf16 hi = __float2bfloat16_rn(v);
        bhl_out[t * 2 * EP + e] = hi;
        bhl_out[t * 2 * EP + EP + e] = __float2bfloat16_rn(v - __bfloat162float(hi));
      }
    }
    sdot = warp_sum(sdot);
    if (lane == 0) Srow[r] = sdot;
  }
  dtp = warp_sum(dtp);
  if (lane == 0) atomicAdd(dtemp, dtp);
  __syncthreads();
  // A = dcos (hi + lo) of the warp's 16 tokens; B(e, c) = kn[c][e] (hi + mid)
  uint32_t ahi[KSTEPS][4], alo[KSTEPS][4];
  const int g = lane >> 2, tq = lane & 3;
  {
#pragma unroll
    for (int s = 0; s < KSTEPS; ++s) {
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
  const int ra = 16 * w + g, rb = ra + 8;
  const float rna = t0 + ra < T ? rn_in[t0 + ra] : 0.f, rnb = t0 + rb < T ? rn_in[t0 + rb] : 0.f;
  const float qa = rna * rna * Srow[ra], qb = rnb * rnb * Srow[rb];
  for (int sl = 0; sl < nsl; ++sl) {
    if (sl + 1 < nsl) {
      issue(sl + 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const bf16* kb = knt + (size_t)(sl & 1) * 2 * RB_SL * Lay::KS;
    const bf16* xb = xt + (size_t)(sl & 1) * TOKC * RB_XS;
    float acc[8][4];
    zero_acc<8>(acc);
#pragma unroll
    for (int s = 0; s < KSTEPS; ++s) {
      const int kk = 16 * s + 2 * tq;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = 8 * j + g;
        const bf16* rh = kb + c * Lay::KS;
        const bf16* rm = kb + (RB_SL + c) * Lay::KS;
        uint32_t bh[2], bm[2];
        bh[0] = kk < EP ? *reinterpret_cast<const uint32_t*>(rh + kk) : 0u;
        bh[1] = kk + 8 < EP ? *reinterpret_cast<const uint32_t*>(rh + kk + 8) : 0u;
        bm[0] = kk < EP ? *reinterpret_cast<const uint32_t*>(rm + kk) : 0u;
        bm[1] = kk + 8 < EP ? *reinterpret_cast<const uint32_t*>(rm + kk + 8) : 0u;
        mma16816(acc[j], ahi[s], bh);
        mma16816(acc[j], ahi[s], bm);
        mma16816(acc[j], alo[s], bh);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = 8 * j + 2 * tq;
      const float2 xa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xb + ra * RB_XS + c));
      const float2 xb2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xb + rb * RB_XS + c));
      *reinterpret_cast<__nv_bfloat162*>(ot + ra * RB_XS + c) = __floats2bfloat162_rn(
          sanitize(rna * acc[j][0] - xa.x * qa, 1e3f), sanitize(rna * acc[j][1] - xa.y * qa, 1e3f));
      *reinterpret_cast<__nv_bfloat162*>(ot + rb * RB_XS + c) = __floats2bfloat162_rn(
          sanitize(rnb * acc[j][2] - xb2.x * qb, 1e3f), sanitize(rnb * acc[j][3] - xb2.y * qb, 1e3f));
    }
    __syncthreads();  // the dx tile is complete; this slice's buffers may be refilled
    for (int i = tid; i < TOKC * (RB_SL / 8); i += NT) {
      const int r = i / (RB_SL / 8), q = i % (RB_SL / 8);
      const int64_t t = t0 + r;
      if (t < T)
        *reinterpret_cast<uint4*>(dx + t * d + sl * RB_SL + 8 * q) =
            *reinterpret_cast<const uint4*>(ot + r * RB_XS + 8 * q);
    }
  }
}

// ------------------------------------------------------------------ backward: dkn
// dkn[c][e] += sum_t x[t][c] (r_t dcos[t][e]) with r dcos as bf16 hi + lo terms (written by the
// tokens kernel); CTA = 64 columns of d (4 warps x 16) x a token range, chunks of 64 tokens of x and
// of the terms staged by cp.async one chunk ahead.
constexpr int RK_TC = 64;

template <int NTE>
struct RkLayout {
  static constexpr int EP = NTE * 8;
  static constexpr int BS = EP + 8;  // bf16 stride of a staged term row
  static constexpr size_t XS = 0;                                      // bf16 [2][RK_TC][RB_XS]
  static constexpr size_t BT = XS + (size_t)2 * RK_TC * RB_XS * 2;     // bf16 [2][2 term][RK_TC][BS]
  static constexpr size_t BYTES = BT + (size_t)2 * 2 * RK_TC * BS * 2;
};

template <int NTE>
__global__ void __launch_bounds__(NT) router_bwd_kn_kernel(const bf16* __restrict__ x, const bf16* __restrict__ bhl,
                                                          int64_t T, int d, int E, int64_t tok_per_cta,
                                                          float* __restrict__ dkn) {
  using Lay = RkLayout<NTE>;
  constexpr int EP = Lay::EP;
  extern __shared__ __align__(16) unsigned char rk_smem[];
  bf16* xs = reinterpret_cast<bf16*>(rk_smem + Lay::XS);
  bf16* bt = reinterpret_cast<bf16*>(rk_smem + Lay::BT);
  const int c0 = blockIdx.x * 64;
  const int64_t ta = (int64_t)blockIdx.y * tok_per_cta;
  const int64_t tb = ta + tok_per_cta < T ? ta + tok_per_cta : T;
  const int tid = threadIdx.x, w = tid >> 5;
  const int nch = (int)((tb - ta + RK_TC - 1) / RK_TC);
  auto issue = [&](int ch) {
    const int64_t q0 = ta + (int64_t)ch * RK_TC;
    bf16* xb = xs + (size_t)(ch & 1) * RK_TC * RB_XS;
    bf16* bb = bt + (size_t)(ch & 1) * 2 * RK_TC * Lay::BS;
    for (int i = tid; i < RK_TC * 8; i += NT) {
      const int r = i >> 3, q = i & 7;
      const int64_t t = q0 + r;
      cp16z(xb + r * RB_XS + 8 * q, x + (t < tb ? t : ta) * d + c0 + 8 * q, t < tb);
    }
    constexpr int BCH = EP / 8;
    for (int i = tid; i < 2 * RK_TC * BCH; i += NT) {
      const int term = i / (RK_TC * BCH), r = (i / BCH) % RK_TC, q = i % BCH;
      const int64_t t = q0 + r;
      cp16z(bb + (term * RK_TC + r) * Lay::BS + 8 * q, bhl + (t < tb ? t : ta) * 2 * EP + term * EP + 8 * q,
            t < tb);
    }
    cp_commit();
  };
  float acc[NTE][4];
  zero_acc<NTE>(acc);
  if (nch > 0) issue(0);
  for (int ch = 0; ch < nch; ++ch) {
    if (ch + 1 < nch) {
      issue(ch + 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const bf16* xb = xs + (size_t)(ch & 1) * RK_TC * RB_XS;
    const bf16* bb = bt + (size_t)(ch & 1) * 2 * RK_TC * Lay::BS;
    // A(m = column, k = token) = xs[k][m]; B(k = token, n = expert) = term[k][n]
    warp_mma<NTE>(acc, ColA16{xb, RB_XS}, KNB16{bb, Lay::BS}, 16 * w, 0, 0, RK_TC);
    warp_mma<NTE>(acc, ColA16{xb, RB_XS}, KNB16{bb + RK_TC * Lay::BS, Lay::BS}, 16 * w, 0, 0, RK_TC);
    __syncthreads();  // both reads of this buffer are done before it is refilled
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
  // dcos: (T, EP) fp32 scratch, used here as (T, 2 EP) bf16 hi / lo terms of r dcos
  if (T <= 0) return;
  const int grid = (int)((T + TOKC - 1) / TOKC);
  const int EP = ahb_router_padded_experts(E);
  bf16* bhl = reinterpret_cast<bf16*>(dcos);
#define RB(N)                                                                                                      \
  do {                                                                                                             \
    static bool init = false;                                                                                      \
    if (!init) {                                                                                                   \
      cudaFuncSetAttribute(router_bwd_tokens_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,               \
                           (int)RbLayout<N>::BYTES);                                                               \
      init = true;                                                                                                 \
    }                                                                                                              \
    router_bwd_tokens_kernel<N><<<grid, NT, RbLayout<N>::BYTES, st>>>((const bf16*)x, (const bf16*)kn2, temp,      \
        logits, cosv, rn, top_idx, gate, dgate, dps, dlse_sq, T, d, E, k, bhl, dtemp, (bf16*)dx);                 \
  } while (0)
  if (EP == 16) RB(2); else if (EP == 32) RB(4); else if (EP == 48) RB(6); else RB(8);
#undef RB
  const int nx = d / 64;
  int ny = (2 * sm_count() + nx - 1) / nx;
  const int64_t per = ((T + ny - 1) / ny + RK_TC - 1) / RK_TC * RK_TC;
  ny = (int)((T + per - 1) / per);
#define RK(N)                                                                                                      \
  do {                                                                                                             \
    static bool init = false;                                                                                      \
    if (!init) {                                                                                                   \
      cudaFuncSetAttribute(router_bwd_kn_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,                   \
                           (int)RkLayout<N>::BYTES);                                                               \
      init = true;                                                                                                 \
    }                                                                                                              \
    router_bwd_kn_kernel<N><<<dim3(nx, ny), NT, RkLayout<N>::BYTES, st>>>((const bf16*)x, bhl, T, d, E, per, dkn); \
  } while (0)
  if (EP == 16) RK(2); else if (EP == 32) RK(4); else if (EP == 48) RK(6); else RK(8);
#undef RK
}
