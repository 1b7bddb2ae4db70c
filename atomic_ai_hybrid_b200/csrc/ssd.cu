// Mamba2 SSD with per-channel dt (headdim 64, d_state 128, chunk 64, B/C shared
// by all heads), following the reference's chunked form and clip discipline
// (reference `atomic_ops/mamba2_ssd_reference.py:56-148`):
//   dA = clip(dt*A_h, +-20) ; c = cumsum_t dA            (per channel p)
//   CB[i,j] = C_i . B_j ; dBx = dt*x
//   y_diag[i,p] = sum_{j<=i} e^{max(c_ip-c_jp,-20)} CB[i,j] dBx[j,p]
//   y_off[i,p]  = e^{max(c_ip,-20)} sum_s C[i,s] S_in[p,s]
//   S_end[p,s]  = sum_j e^{max(cL_p-c_jp,-20)} dBx[j,p] B[j,s]
//   S_in(next)  = S_in e^{max(cL_p,-20)} + S_end
//
// sm_100a layout: ssd_state_fwd / ssd_out_fwd / ssd_bwd_chunk use one CTA per
// (chunk, batch) that loops over the heads, so C B^T and the B/C tiles are read
// once per chunk and the B/C gradients of all heads accumulate in registers
// (no atomics).  ssd_scan carries the chunk states: each thread owns one (p, s)
// state element of one head and walks the chunks (forward or reverse).
// Pairwise decays inside a chunk use the reference-row factorisation of the
// GDN kernels (both factors <= 1); diagonal 16x16 blocks are exact.
#include "common.cuh"
#include "mma.cuh"
#include "launchers.h"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

constexpr int C = 64;    // chunk
constexpr int P = 64;    // head dim
constexpr int N = 128;   // state dim
constexpr int LDN = N + 8;   // bf16 stride for C x N / P x N tiles
constexpr int LDP = P + 8;   // bf16 stride for C x P tiles
constexpr int LDPF = P + 4;  // fp32 stride for C x P tiles
constexpr int LDCC = C + 4;  // fp32 stride for C x C tiles

AHB_DEVICE float bf(bf16 x) { return __bfloat162float(x); }
AHB_DEVICE void st2(bf16* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack2(a, b); }

struct SIdx {
  int64_t L, H, NC;
  AHB_DEVICE int64_t xp(int b, int64_t t, int h) const { return ((b * L + t) * H + h) * P; }  // (B,L,H,P)
  AHB_DEVICE int64_t bn(int b, int64_t t) const { return (b * L + t) * N; }                  // (B,L,N)
  AHB_DEVICE int64_t ch(int b, int h, int n) const { return ((int64_t)b * H + h) * NC + n; }
};

AHB_DEVICE void load_bn_tile(bf16* dst, const bf16* src, const SIdx& ix, int b, int n) {
  for (int i = threadIdx.x; i < C * (N / 8); i += blockDim.x) {
    int r = i / (N / 8), c8 = (i % (N / 8)) * 8;
    *reinterpret_cast<uint4*>(dst + r * LDN + c8) =
        *reinterpret_cast<const uint4*>(src + ix.bn(b, (int64_t)n * C + r) + c8);
  }
}
AHB_DEVICE void load_xp_tile(bf16* dst, const bf16* src, const SIdx& ix, int b, int n, int h) {
  for (int i = threadIdx.x; i < C * (P / 8); i += blockDim.x) {
    int r = i / (P / 8), c8 = (i % (P / 8)) * 8;
    *reinterpret_cast<uint4*>(dst + r * LDP + c8) =
        *reinterpret_cast<const uint4*>(src + ix.xp(b, (int64_t)n * C + r, h) + c8);
  }
}
// state tile image (bf16, rows s = 0..127, columns p = 0..63, 128-byte swizzle) -> smem [P][LDN]
AHB_DEVICE void load_state_bf(bf16* dst, const unsigned char* img) {
  for (int u = threadIdx.x; u < N * (P / 8); u += blockDim.x) {
    const int s = u >> 3, c8 = (u & 7) << 3;
    const int off = (s >> 3) * 1024 + (s & 7) * 128 + (((c8 >> 3) ^ (s & 7)) << 4);
    const uint4 w = *reinterpret_cast<const uint4*>(img + off);
    const bf16* e = reinterpret_cast<const bf16*>(&w);
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[(c8 + k) * LDN + s] = e[k];
  }
}
// c = cumsum(clip(dt*A, +-20)), clipped to +-1e4 (reference sanitize)
AHB_DEVICE void cum_decay(float* cum, const bf16* dt_s, float A) {
  __syncthreads();
  if (threadIdx.x < P) {
    float s = 0.f;
    for (int r = 0; r < C; ++r) {
      s += fminf(fmaxf(bf(dt_s[r * LDP + threadIdx.x]) * A, -20.f), 20.f);
      cum[r * LDPF + threadIdx.x] = fminf(fmaxf(s, -1e4f), 1e4f);
    }
  }
  __syncthreads();
}
// triangular pair index -> (i, j), i >= j, within 16
AHB_DEVICE void tri_ij(int p, int& i, int& j) {
  i = (int)((sqrtf(8.f * p + 1.f) - 1.f) * 0.5f);
  while ((i + 1) * (i + 2) / 2 <= p) ++i;
  while (i * (i + 1) / 2 > p) --i;
  j = p - i * (i + 1) / 2;
}

AHB_DEVICE float dbx(const bf16* x_s, const bf16* dt_s, int r, int p) {
  return bf(x_s[r * LDP + p]) * bf(dt_s[r * LDP + p]);
}

// y_diag for the warp's tile: rows [16I, 16I+16), cols [n0, n0+8*NT)
// Whether a 16-row diagonal block may be factorised at its first row: the largest
// per-channel decay across its rows (c_r0 - c_r0+15) must keep e^{span} far from overflow.
// Every lane of the calling warp gets the answer.
AHB_DEVICE bool block_span_ok(const float* cum, int I) {
  const int lane = threadIdx.x & 31;
  const float* a = cum + 16 * I * LDPF;
  const float* z = cum + (16 * I + 15) * LDPF;
  float span = fmaxf(a[lane] - z[lane], a[lane + 32] - z[lane + 32]);
  span = warp_max(span);
  return span <= 60.f;
}

template <int NT>
AHB_DEVICE void ydiag_tile(float (*acc)[4], const float* cb_s, const bf16* x_s, const bf16* dt_s, const float* cum,
                           int I, int n0) {
  const int r0 = 16 * I;
  zero_acc<NT>(acc);
  // the diagonal block is factorised at row r0 too (B carries e^{c_r0 - c_j} <= e^{span}) unless
  // its decay span is too wide; then it is summed exactly below
  const bool fact = block_span_ok(cum, I);
  const float* cr = cum + r0 * LDPF;
  auto fbf = [&](int kj, int np) -> float2 {
    return make_float2(dbx(x_s, dt_s, kj, np) * __expf(cr[np] - cum[kj * LDPF + np]),
                       dbx(x_s, dt_s, kj + 1, np) * __expf(cr[np] - cum[(kj + 1) * LDPF + np]));
  };
  if (I > 0) {
    auto fb = [&](int kj, int np) -> uint32_t {
      const float2 v = fbf(kj, np);
      return pack2(v.x, v.y);
    };
    warp_mma<NT>(acc, RowA32{cb_s, LDCC}, fb, r0, n0, 0, r0);
  }
  if (fact) {  // the diagonal block: two-term bf16 operands keep it close to fp32
    auto fa = [&](int r, int kj) -> float2 {
      return make_float2(kj <= r ? cb_s[r * LDCC + kj] : 0.f, kj + 1 <= r ? cb_s[r * LDCC + kj + 1] : 0.f);
    };
    warp_mma_split<NT>(acc, fa, fbf, r0, n0, r0, r0 + 16);
  }
  if (I > 0 || fact)
    for_acc<NT>(acc, r0, n0, [&](int r, int c, float& v) { v *= __expf(cum[r * LDPF + c] - cr[c]); });
  if (fact) return;
  for_acc<NT>(acc, r0, n0, [&](int r, int c, float& v) {
    float s = 0.f;
    const float ci = cum[r * LDPF + c];
    for (int j = r0; j <= r; ++j)
      s += cb_s[r * LDCC + j] * dbx(x_s, dt_s, j, c) * __expf(fmaxf(ci - cum[j * LDPF + c], -20.f));
    v += s;
  });
}

// y_off tile: e^{max(c,-20)} * (C S^T)
template <int NT>
AHB_DEVICE void yoff_tile(float (*acc)[4], const bf16* c_s, const bf16* sin_s, const float* cum, int I, int n0) {
  zero_acc<NT>(acc);
  warp_mma<NT>(acc, RowA16{c_s, LDN}, NKB16{sin_s, LDN}, 16 * I, n0, 0, N);
  for_acc<NT>(acc, 16 * I, n0, [&](int r, int c, float& v) { v *= __expf(fmaxf(cum[r * LDPF + c], -20.f)); });
}

// C B^T (C x C), sanitized
AHB_DEVICE void compute_cb(float* cb_s, const bf16* c_s, const bf16* b_s) {
  const int warp = threadIdx.x >> 5;
  float acc[2][4];
  zero_acc<2>(acc);
  warp_mma<2>(acc, RowA16{c_s, LDN}, NKB16{b_s, LDN}, 16 * (warp & 3), 16 * (warp >> 2), 0, N);
  for_acc<2>(acc, 16 * (warp & 3), 16 * (warp >> 2),
             [&](int r, int c, float& v) { cb_s[r * LDCC + c] = sanitize(v, 1e4f); });
}

// ============================================================ backward: per chunk, all heads
// smem: b, c bf16 [C][LDN]; cb, dcb f32 [C][LDCC]; x, dt, dy bf16 [C][LDP]; cum, dc, ddbx f32 [C][LDPF];
//       sin, dse bf16 [P][LDN]
constexpr size_t SMEM_BWD =
    2 * C * LDN * 2 + 2 * C * LDCC * 4 + 3 * C * LDP * 2 + 3 * C * LDPF * 4 + 2 * P * LDN * 2 + P * 4;

__global__ void __launch_bounds__(512, 1) ssd_bwd_chunk_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ dt, const float* __restrict__ A,
    const bf16* __restrict__ Bm, const bf16* __restrict__ Cm, const bf16* __restrict__ dy,
    const unsigned char* __restrict__ sin_t, const unsigned char* __restrict__ dse_t, int L, int H, bf16* __restrict__ dx,
    bf16* __restrict__ ddt, float* __restrict__ dB, float* __restrict__ dC, float* __restrict__ dA) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* b_s = reinterpret_cast<bf16*>(smem);
  bf16* c_s = b_s + C * LDN;
  float* cb_s = reinterpret_cast<float*>(c_s + C * LDN);
  float* dcb_s = cb_s + C * LDCC;
  bf16* x_s = reinterpret_cast<bf16*>(dcb_s + C * LDCC);
  bf16* dt_s = x_s + C * LDP;
  bf16* dy_s = dt_s + C * LDP;
  float* cum = reinterpret_cast<float*>(dy_s + C * LDP);
  float* dc_s = cum + C * LDPF;
  float* ddbx_s = dc_s + C * LDPF;
  bf16* sin_s = reinterpret_cast<bf16*>(ddbx_s + C * LDPF);
  bf16* dse_s = sin_s + P * LDN;
  float* dcl_s = reinterpret_cast<float*>(dse_s + P * LDN);

  __shared__ int exact_s[4];
  const int n = blockIdx.x, b = blockIdx.y, NC = gridDim.x;
  const SIdx ix{L, H, NC};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  load_bn_tile(b_s, Bm, ix, b, n);
  load_bn_tile(c_s, Cm, ix, b, n);
  __syncthreads();
  compute_cb(cb_s, c_s, b_s);
  // dB / dC accumulators: warp tile rows [16*(warp&3)), cols [64*(warp>>2)), 8 n-tiles
  const int mt = warp & 3, nq = warp >> 2;
  float dBa[4][4], dCa[4][4];
  zero_acc<4>(dBa);
  zero_acc<4>(dCa);
  const int hpg = H / gridDim.z, h0 = blockIdx.z * hpg;
  for (int h = h0; h < h0 + hpg; ++h) {
    const int64_t cbi = ix.ch(b, h, n);
    const float Ah = A[h];
    load_xp_tile(x_s, x, ix, b, n, h);
    load_xp_tile(dt_s, dt, ix, b, n, h);
    load_xp_tile(dy_s, dy, ix, b, n, h);
    load_state_bf(sin_s, sin_t + cbi * (P * N * 2));
    load_state_bf(dse_s, dse_t + cbi * (P * N * 2));
    if (tid < P) dcl_s[tid] = 0.f;
    cum_decay(cum, dt_s, Ah);
    const float* cl = cum + (C - 1) * LDPF;
    if (warp < 4) {
      const bool ok = block_span_ok(cum, warp);
      if (lane == 0) exact_s[warp] = !ok;
    }
    __syncthreads();
    // (1) dCB[i,j] = sum_p dy[i,p] e^{c_i-c_j} dBx[j,p]   (j <= i); diagonal blocks factorised
    //     at row r0 like the others unless their decay span is too wide (exact pass below)
    {
      const int I = mt, r0 = 16 * I;
      float acc[2][4];
      zero_acc<2>(acc);
      const int n0 = 16 * nq;  // j columns [n0, n0+16)
      if (n0 < r0 || (n0 == r0 && !exact_s[I])) {
        const float* cr = cum + r0 * LDPF;
        auto faf = [&](int ri, int kp) -> float2 {
          return make_float2(bf(dy_s[ri * LDP + kp]) * __expf(cum[ri * LDPF + kp] - cr[kp]),
                             bf(dy_s[ri * LDP + kp + 1]) * __expf(cum[ri * LDPF + kp + 1] - cr[kp + 1]));
        };
        auto fbf = [&](int kp, int nj) -> float2 {
          return make_float2(dbx(x_s, dt_s, nj, kp) * __expf(cr[kp] - cum[nj * LDPF + kp]),
                             dbx(x_s, dt_s, nj, kp + 1) * __expf(cr[kp + 1] - cum[nj * LDPF + kp + 1]));
        };
        if (n0 == r0) {  // diagonal block: two-term operands (its sums feed the cancelling dA)
          warp_mma_split<2>(acc, faf, fbf, r0, n0, 0, P);
        } else {
          auto fa = [&](int ri, int kp) -> uint32_t { const float2 v = faf(ri, kp); return pack2(v.x, v.y); };
          auto fb = [&](int kp, int nj) -> uint32_t { const float2 v = fbf(kp, nj); return pack2(v.x, v.y); };
          warp_mma<2>(acc, fa, fb, r0, n0, 0, P);
        }
      }
      const bool fact_diag = n0 == r0 && !exact_s[I];
      for_acc<2>(acc, r0, n0, [&](int r, int c, float& v) {
        if (fact_diag) {
          dcb_s[r * LDCC + c] = c <= r ? v : 0.f;
        } else {
          const bool diag = c >= r0 && c < r0 + 16 && c <= r;  // written by the exact pass below
          if (!diag) dcb_s[r * LDCC + c] = c >= r0 ? 0.f : v;
        }
      });
    }
    // exact per-channel sums of the diagonal 16x16 blocks with a wide decay span: one (i, j) pair per thread
    for (int q = tid; q < 4 * 136; q += blockDim.x) {
      if (!exact_s[q / 136]) continue;
      int i, j;
      tri_ij(q % 136, i, j);
      const int r = 16 * (q / 136) + i, c = 16 * (q / 136) + j;
      float sacc = 0.f;
#pragma unroll 8
      for (int p = 0; p < P; ++p)
        sacc += bf(dy_s[r * LDP + p]) * dbx(x_s, dt_s, c, p) *
                __expf(fmaxf(cum[r * LDPF + p] - cum[c * LDPF + p], -20.f));
      dcb_s[r * LDCC + c] = sacc;
    }
    __syncthreads();
    // (2) dC += dCB B + (dy e^c) S_in^T ;  (3) dB += dCB^T C + (dBx e^{cL-c}) dS_end^T
    {
      const int m0 = 16 * mt, n0 = 32 * nq;
      warp_mma<4>(dCa, RowA32{dcb_s, LDCC}, KNB16{b_s, LDN}, m0, n0, 0, m0 + 16);
      auto fa_dy = [&](int ri, int kp) -> uint32_t {
        return pack2(bf(dy_s[ri * LDP + kp]) * __expf(fmaxf(cum[ri * LDPF + kp], -20.f)),
                     bf(dy_s[ri * LDP + kp + 1]) * __expf(fmaxf(cum[ri * LDPF + kp + 1], -20.f)));
      };
      warp_mma<4>(dCa, fa_dy, KNB16{sin_s, LDN}, m0, n0, 0, P);
      warp_mma<4>(dBa, ColA32{dcb_s, LDCC}, KNB16{c_s, LDN}, m0, n0, m0, C);
      auto fa_bx = [&](int rj, int kp) -> uint32_t {
        return pack2(dbx(x_s, dt_s, rj, kp) * __expf(fmaxf(cl[kp] - cum[rj * LDPF + kp], -20.f)),
                     dbx(x_s, dt_s, rj, kp + 1) * __expf(fmaxf(cl[kp + 1] - cum[rj * LDPF + kp + 1], -20.f)));
      };
      warp_mma<4>(dBa, fa_bx, KNB16{dse_s, LDN}, m0, n0, 0, P);
    }
    // (4)+(5) per (t,p) tile: y_diag, y_off, ddBx (diag part, state part) -> dc, ddBx
    {
      const int I = mt, n0 = 16 * nq, r0 = 16 * I;
      float yd[2][4], yo[2][4], dd[2][4], ds[2][4];
      ydiag_tile<2>(yd, cb_s, x_s, dt_s, cum, I, n0);
      yoff_tile<2>(yo, c_s, sin_s, cum, I, n0);
      // ddBx_diag[j,p] = sum_{i>=j} CB[i,j] dy[i,p] e^{c_i-c_j}  (own block factorised unless exact)
      zero_acc<2>(dd);
      const bool exact_i = exact_s[I];
      for (int I2 = exact_i ? I + 1 : I; I2 < 4; ++I2) {
        const int r2 = 16 * I2;
        const float* cr = cum + r2 * LDPF;
        auto faf = [&](int rj, int ki) -> float2 {
          const int i0 = r2 + ki;
          return make_float2(i0 >= rj ? cb_s[i0 * LDCC + rj] : 0.f, i0 + 1 >= rj ? cb_s[(i0 + 1) * LDCC + rj] : 0.f);
        };
        auto fa = [&](int rj, int ki) -> uint32_t { const float2 v = faf(rj, ki); return pack2(v.x, v.y); };
        auto fbf = [&](int ki, int np) -> float2 {
          return make_float2(bf(dy_s[(r2 + ki) * LDP + np]) * __expf(cum[(r2 + ki) * LDPF + np] - cr[np]),
                             bf(dy_s[(r2 + ki + 1) * LDP + np]) * __expf(cum[(r2 + ki + 1) * LDPF + np] - cr[np]));
        };
        auto fb = [&](int ki, int np) -> uint32_t { const float2 v = fbf(ki, np); return pack2(v.x, v.y); };
        float tacc[2][4];
        zero_acc<2>(tacc);
        if (I2 == I)  // own block: two-term operands
          warp_mma_split<2>(tacc, faf, fbf, r0, n0, 0, 16);
        else
          warp_mma<2>(tacc, fa, fb, r0, n0, 0, 16);
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            int r = r0 + g + (e >> 1) * 8, c = n0 + 8 * j + 2 * t + (e & 1);
            dd[j][e] += tacc[j][e] * __expf(cr[c] - cum[r * LDPF + c]);
          }
      }
      for_acc<2>(dd, r0, n0, [&](int r, int c, float& v) {
        float s = 0.f;
        const float cj = cum[r * LDPF + c];
        for (int i = r; exact_i && i < r0 + 16; ++i)
          s += cb_s[i * LDCC + r] * bf(dy_s[i * LDP + c]) * __expf(fmaxf(cum[i * LDPF + c] - cj, -20.f));
        v += s;
      });
      // ddBx_state[j,p] = e^{cL-c_j} sum_s B[j,s] dS_end[p,s]
      zero_acc<2>(ds);
      warp_mma<2>(ds, RowA16{b_s, LDN}, NKB16{dse_s, LDN}, r0, n0, 0, N);
      const int g = lane >> 2, t = lane & 3;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = r0 + g + (e >> 1) * 8, c = n0 + 8 * j + 2 * t + (e & 1);
          const float cr = cum[r * LDPF + c];
          const float dlt = cl[c] - cr;
          const float eds = __expf(fmaxf(dlt, -20.f));
          const float dsv = ds[j][e] * eds;
          const float bxv = dbx(x_s, dt_s, r, c);
          const float dyv = bf(dy_s[r * LDP + c]);
          float dcv = dyv * yd[j][e] - bxv * dd[j][e];
          if (cr > -20.f) dcv += dyv * yo[j][e];
          if (dlt > -20.f) {
            dcv -= bxv * dsv;
            atomicAdd(dcl_s + c, bxv * dsv);
          }
          dc_s[r * LDPF + c] = dcv;
          ddbx_s[r * LDPF + c] = dd[j][e] + dsv;
        }
    }
    __syncthreads();
    // dcL (last row): sum_j dBx ddBx_state (accumulated above into dcl_s) + state carry
    {
      const int p = tid >> 3, q8 = tid & 7;
      float s_car = 0.f;
      for (int s2 = q8 * 16; s2 < q8 * 16 + 16; ++s2) s_car += bf(dse_s[p * LDN + s2]) * bf(sin_s[p * LDN + s2]);
      s_car += __shfl_xor_sync(0xffffffffu, s_car, 1);
      s_car += __shfl_xor_sync(0xffffffffu, s_car, 2);
      s_car += __shfl_xor_sync(0xffffffffu, s_car, 4);
      if (q8 == 0) {
        float add = dcl_s[p];
        if (cl[p] > -20.f) add += s_car * __expf(cl[p]);
        dc_s[(C - 1) * LDPF + p] += add;
      }
    }
    __syncthreads();
    // reverse cumsum of dc -> d(dA); outputs dx, ddt; dA_h
    float dAh = 0.f;
    if (tid < P) {
      const int p = tid;
      float s = 0.f;
      for (int r = C - 1; r >= 0; --r) {
        s += dc_s[r * LDPF + p];
        const float dtv = bf(dt_s[r * LDP + p]);
        const float pre = dtv * Ah;
        const float g = (pre > -20.f && pre < 20.f) ? s : 0.f;
        dc_s[r * LDPF + p] = g * Ah;  // contribution to ddt
        dAh += g * dtv;
      }
    }
    __syncthreads();
    for (int i = tid; i < C * P; i += blockDim.x) {
      const int r = i / P, p = i % P;
      const float dd = ddbx_s[r * LDPF + p];
      const int64_t gi = ix.xp(b, (int64_t)n * C + r, h) + p;
      dx[gi] = __float2bfloat16_rn(dd * bf(dt_s[r * LDP + p]));
      ddt[gi] = __float2bfloat16_rn(dd * bf(x_s[r * LDP + p]) + dc_s[r * LDPF + p]);
    }
    dAh = warp_sum(dAh);
    if (lane == 0 && tid < P) atomicAdd(dA + h, dAh);
    __syncthreads();
  }
  // partial dB, dC of this head group: (G, B, L, N)
  const int m0 = 16 * mt, n0 = 32 * nq;
  const int64_t goff = (int64_t)blockIdx.z * ix.L * N * gridDim.y;
  for_acc<4>(dBa, m0, n0, [&](int r, int c, float& v) { dB[goff + ix.bn(b, (int64_t)n * C + r) + c] = v; });
  for_acc<4>(dCa, m0, n0, [&](int r, int c, float& v) { dC[goff + ix.bn(b, (int64_t)n * C + r) + c] = v; });
}

// out[i] = sum_g part[g * n + i]
__global__ void sum_groups_kernel(const float* __restrict__ part, int G, int64_t n, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int g = 0; g < G; ++g) s += part[g * n + i];
    out[i] = s;
  }
}

int head_groups(int H) {
  for (int g : {8, 4, 2}) if (H % g == 0) return g;
  return 1;
}

template <class K>
void set_smem(K kernel, size_t bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

int ahb_ssd_head_groups(int H) { return head_groups(H); }

// dB_part / dC_part: (G, B, L, N) fp32 scratch with G = ahb_ssd_head_groups(H); the sums over
// head groups are written to dB / dC.  sin_t / dse_t: per chunk-head state and state-gradient
// tile images (bf16, rows s, columns p) from ahb_ssd_fwd_tc / ahb_ssd_state_bwd_tc.
void ahb_ssd_bwd_chunk(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, const void* dy,
                       int B, int L, int H, const void* sin_t, const void* dse_t, void* dx, void* ddt, float* dB,
                       float* dC, float* dA, float* dB_part, float* dC_part, cudaStream_t st) {
  static bool init = false;
  if (!init) {
    set_smem(ssd_bwd_chunk_kernel, SMEM_BWD);
    init = true;
  }
  const int NC = L / C;
  const int G = head_groups(H);
  ssd_bwd_chunk_kernel<<<dim3(NC, B, G), 512, SMEM_BWD, st>>>((const bf16*)x, (const bf16*)dt, A, (const bf16*)Bm,
                                                             (const bf16*)Cm, (const bf16*)dy,
                                                             (const unsigned char*)sin_t,
                                                             (const unsigned char*)dse_t, L, H, (bf16*)dx, (bf16*)ddt,
                                                             dB_part, dC_part, dA);
  const int64_t n = (int64_t)B * L * N;
  const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  sum_groups_kernel<<<blocks, 256, 0, st>>>(dB_part, G, n, dB);
  sum_groups_kernel<<<blocks, 256, 0, st>>>(dC_part, G, n, dC);
}
