// Causal flash attention for the MLA sublayer (reference `model.py:326-359`, the
// TPU Pallas flash_attention with causal=True), bf16 in / out, fp32 softmax.
//
// Layout: q, k, v, o (BH, L, D) row-major, D in {64, 96, 128}; 64-row tiles.
// Forward: one CTA (4 warps x 16 query rows) per (query tile, batch*head); key
// tiles up to the diagonal are staged in shared memory; S = Q K^T, online softmax
// in registers, O += P V with P re-used from the S accumulators as the A operand.
// Writes O and the row log-sum-exp for the backward.
// Backward: one CTA (4 warps x 16 keys) per (key tile, batch*head); for every
// query tile at or after it: P^T = exp(K Q^T * scale - lse), dV += P^T dO,
// dP^T = V dO^T, dS^T = P^T (dP^T - delta), dK += dS^T Q; dS goes through shared
// memory for dQ += dS K, accumulated in fp32 with atomics.  delta = rowsum(dO o O)
// is computed beforehand.
#include "common.cuh"
#include "launchers.h"
#include "mma.cuh"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

constexpr int BT = 64;  // rows per tile
constexpr int NT = 128;

// copy a (rows x D) bf16 tile (rows of a (L, D) matrix starting at row r0) into smem; rows >= L are zero
template <int D>
AHB_DEVICE void load_tile(bf16* s, const bf16* g, int r0, int L) {
  constexpr int LD = (D + 8);
  constexpr int V8 = D / 8;
  for (int i = threadIdx.x; i < BT * V8; i += NT) {
    const int r = i / V8, c = (i % V8) * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (r0 + r < L) u = *reinterpret_cast<const uint4*>(g + (int64_t)(r0 + r) * D + c);
    *reinterpret_cast<uint4*>(s + r * LD + c) = u;
  }
}

template <int D>
__global__ void __launch_bounds__(NT) attn_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                      const bf16* __restrict__ v, int L, float scale,
                                                      bf16* __restrict__ o, float* __restrict__ lse) {
  constexpr int LD = (D + 8);
  constexpr int KD = D / 16;  // k-steps over the head dim
  constexpr int ND = D / 8;   // n-tiles over the head dim
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* q_s = reinterpret_cast<bf16*>(smem);
  bf16* k_s = q_s + BT * LD;
  bf16* v_s = k_s + BT * LD;
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int64_t base = (int64_t)bh * L * D;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int q0 = qt * BT;
  load_tile<D>(q_s, q + base, q0, L);
  __syncthreads();
  uint32_t qa[KD][4];
#pragma unroll
  for (int s = 0; s < KD; ++s) load_a(qa[s], RowA16{q_s, LD}, 16 * w, 16 * s);
  float oacc[ND][4];
  zero_acc<ND>(oacc);
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int r_a = q0 + 16 * w + g, r_b = r_a + 8;  // this thread's two query rows
  for (int kt = 0; kt <= qt; ++kt) {
    __syncthreads();
    load_tile<D>(k_s, k + base, kt * BT, L);
    load_tile<D>(v_s, v + base, kt * BT, L);
    __syncthreads();
    float sacc[8][4];
    zero_acc<8>(sacc);
#pragma unroll
    for (int s = 0; s < KD; ++s) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t b[2];
        load_b(b, NKB16{k_s, LD}, 16 * s, 8 * j);
        mma16816(sacc[j], qa[s], b);
      }
    }
    // scale, causal / length mask, row max
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = kt * BT + 8 * j + 2 * t + (e & 1);
        const int row = e < 2 ? r_a : r_b;
        float sv = sacc[j][e] * scale;
        if (col > row || col >= L) sv = -INFINITY;
        sacc[j][e] = sv;
        mx[e >> 1] = fmaxf(mx[e >> 1], sv);
      }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mn = fmaxf(m[h], mx[h]);
      corr[h] = m[h] == -INFINITY ? 0.f : __expf(m[h] - mn);
      m[h] = mn;
      l[h] *= corr[h];
    }
#pragma unroll
    for (int j = 0; j < ND; ++j) {
      oacc[j][0] *= corr[0];
      oacc[j][1] *= corr[0];
      oacc[j][2] *= corr[1];
      oacc[j][3] *= corr[1];
    }
    // P = exp(S - m) -> bf16 A fragments (key pairs of two S tiles per 16-key step)
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = m[0] == -INFINITY ? 0.f : __expf(sacc[j][0] - m[0]);
      const float p1 = m[0] == -INFINITY ? 0.f : __expf(sacc[j][1] - m[0]);
      const float p2 = m[1] == -INFINITY ? 0.f : __expf(sacc[j][2] - m[1]);
      const float p3 = m[1] == -INFINITY ? 0.f : __expf(sacc[j][3] - m[1]);
      l[0] += p0 + p1;
      l[1] += p2 + p3;
      const int s = j >> 1, hi = j & 1;
      pa[s][hi * 2 + 0] = pack2(p0, p1);
      pa[s][hi * 2 + 1] = pack2(p2, p3);
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int j = 0; j < ND; ++j) {
        uint32_t b[2];
        load_b(b, KNB16{v_s, LD}, 16 * s, 8 * j);
        mma16816(oacc[j], pa[s], b);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  const float inv_a = l[0] > 0.f ? 1.f / l[0] : 0.f, inv_b = l[1] > 0.f ? 1.f / l[1] : 0.f;
#pragma unroll
  for (int j = 0; j < ND; ++j) {
    const int c = 8 * j + 2 * t;
    if (r_a < L)
      *reinterpret_cast<__nv_bfloat162*>(o + base + (int64_t)r_a * D + c) =
          __floats2bfloat162_rn(oacc[j][0] * inv_a, oacc[j][1] * inv_a);
    if (r_b < L)
      *reinterpret_cast<__nv_bfloat162*>(o + base + (int64_t)r_b * D + c) =
          __floats2bfloat162_rn(oacc[j][2] * inv_b, oacc[j][3] * inv_b);
  }
  if (t == 0) {
    if (r_a < L) lse[(int64_t)bh * L + r_a] = m[0] + __logf(l[0]);
    if (r_b < L) lse[(int64_t)bh * L + r_b] = m[1] + __logf(l[1]);
  }
}

template <int D>
__global__ void __launch_bounds__(NT) attn_bwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                      const bf16* __restrict__ v, const bf16* __restrict__ dout,
                                                      const float* __restrict__ lse, const float* __restrict__ delta,
                                                      int L, float scale, float* __restrict__ dq,
                                                      bf16* __restrict__ dk, bf16* __restrict__ dv) {
  constexpr int LD = (D + 8);
  constexpr int ND = D / 8;
  constexpr int LDS = BT + 8;
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* k_s = reinterpret_cast<bf16*>(smem);
  bf16* v_s = k_s + BT * LD;
  bf16* q_s = v_s + BT * LD;
  bf16* do_s = q_s + BT * LD;
  bf16* ds_s = do_s + BT * LD;                                   // dS^T [key][query]
  float* lse_s = reinterpret_cast<float*>(ds_s + BT * LDS);
  float* dl_s = lse_s + BT;
  const int kt = blockIdx.x, bh = blockIdx.y;
  const int64_t base = (int64_t)bh * L * D;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int k0 = kt * BT;
  load_tile<D>(k_s, k + base, k0, L);
  load_tile<D>(v_s, v + base, k0, L);
  float dka[ND][4], dva[ND][4];
  zero_acc<ND>(dka);
  zero_acc<ND>(dva);
  const int key_a = k0 + 16 * w + g, key_b = key_a + 8;
  const int nqt = (L + BT - 1) / BT;
  for (int qt = kt; qt < nqt; ++qt) {
    const int q0 = qt * BT;
    __syncthreads();
    load_tile<D>(q_s, q + base, q0, L);
    load_tile<D>(do_s, dout + base, q0, L);
    for (int i = threadIdx.x; i < BT; i += NT) {
      const bool in = q0 + i < L;
      lse_s[i] = in ? lse[(int64_t)bh * L + q0 + i] : INFINITY;
      dl_s[i] = in ? delta[(int64_t)bh * L + q0 + i] : 0.f;
    }
    __syncthreads();
    // S^T = K Q^T (16 keys x 64 queries per warp) -> P^T
    float st[8][4];
    zero_acc<8>(st);
    warp_mma<8>(st, RowA16{k_s, LD}, NKB16{q_s, LD}, 16 * w, 0, 0, D);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = 8 * j + 2 * t + (e & 1);
        const int key = e < 2 ? key_a : key_b;
        const float p = (q0 + qi < key || key >= L) ? 0.f : __expf(st[j][e] * scale - lse_s[qi]);
        st[j][e] = p;
      }
    }
    // dV += P^T dO
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int s = j >> 1, hi = j & 1;
      pa[s][hi * 2 + 0] = pack2(st[j][0], st[j][1]);
      pa[s][hi * 2 + 1] = pack2(st[j][2], st[j][3]);
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int j = 0; j < ND; ++j) {
        uint32_t b[2];
        load_b(b, KNB16{do_s, LD}, 16 * s, 8 * j);
        mma16816(dva[j], pa[s], b);
      }
    }
    // dP^T = V dO^T ; dS^T = P^T (dP^T - delta)
    float dp[8][4];
    zero_acc<8>(dp);
    warp_mma<8>(dp, RowA16{v_s, LD}, NKB16{do_s, LD}, 16 * w, 0, 0, D);
    uint32_t da[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float dsv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = 8 * j + 2 * t + (e & 1);
        dsv[e] = st[j][e] * (dp[j][e] - dl_s[qi]);
      }
      const int s = j >> 1, hi = j & 1;
      da[s][hi * 2 + 0] = pack2(dsv[0], dsv[1]);
      da[s][hi * 2 + 1] = pack2(dsv[2], dsv[3]);
      const int qc = 8 * j + 2 * t;
      *reinterpret_cast<__nv_bfloat162*>(ds_s + (16 * w + g) * LDS + qc) = __floats2bfloat162_rn(dsv[0], dsv[1]);
      *reinterpret_cast<__nv_bfloat162*>(ds_s + (16 * w + g + 8) * LDS + qc) = __floats2bfloat162_rn(dsv[2], dsv[3]);
    }
    // dK += dS^T Q
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int j = 0; j < ND; ++j) {
        uint32_t b[2];
        load_b(b, KNB16{q_s, LD}, 16 * s, 8 * j);
        mma16816(dka[j], da[s], b);
      }
    }
    __syncthreads();
    // dQ[q, :] += sum_key dS[q, key] K[key, :]  (warp: 16 queries, head dim in two halves)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float dqa[ND / 2][4];
      zero_acc<ND / 2>(dqa);
      warp_mma<ND / 2>(dqa, ColA16{ds_s, LDS}, KNB16{k_s, LD}, 16 * w, half * (D / 2), 0, BT);
      for_acc<ND / 2>(dqa, 16 * w, half * (D / 2), [&](int r, int c, float& val) {
        if (q0 + r < L) atomicAdd(dq + base + (int64_t)(q0 + r) * D + c, val * scale);
      });
    }
  }
#pragma unroll
  for (int j = 0; j < ND; ++j) {
    const int c = 8 * j + 2 * t;
    if (key_a < L) {
      *reinterpret_cast<__nv_bfloat162*>(dk + base + (int64_t)key_a * D + c) =
          __floats2bfloat162_rn(dka[j][0] * scale, dka[j][1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dv + base + (int64_t)key_a * D + c) =
          __floats2bfloat162_rn(dva[j][0], dva[j][1]);
    }
    if (key_b < L) {
      *reinterpret_cast<__nv_bfloat162*>(dk + base + (int64_t)key_b * D + c) =
          __floats2bfloat162_rn(dka[j][2] * scale, dka[j][3] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dv + base + (int64_t)key_b * D + c) =
          __floats2bfloat162_rn(dva[j][2], dva[j][3]);
    }
  }
}

template <int D>
size_t fwd_smem() { return (size_t)3 * BT * (D + 8) * 2; }
template <int D>
size_t bwd_smem() { return (size_t)4 * BT * (D + 8) * 2 + (size_t)BT * (BT + 8) * 2 + 2 * BT * 4; }

template <int D>
int launch_fwd(const void* q, const void* k, const void* v, int BH, int L, float scale, void* o, float* lse,
               cudaStream_t st) {
  static bool init = false;
  const size_t sm = fwd_smem<D>();
  if (!init) {
    if (cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
      return -1;
    init = true;
  }
  attn_fwd_kernel<D><<<dim3((L + BT - 1) / BT, BH), NT, sm, st>>>((const bf16*)q, (const bf16*)k, (const bf16*)v, L,
                                                                  scale, (bf16*)o, lse);
  return 0;
}

template <int D>
int launch_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
               int BH, int L, float scale, float* dq, void* dk, void* dv, cudaStream_t st) {
  static bool init = false;
  const size_t sm = bwd_smem<D>();
  if (!init) {
    if (cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
      return -1;
    init = true;
  }
  attn_bwd_kernel<D><<<dim3((L + BT - 1) / BT, BH), NT, sm, st>>>((const bf16*)q, (const bf16*)k, (const bf16*)v,
                                                                  (const bf16*)dout, lse, delta, L, scale, dq,
                                                                  (bf16*)dk, (bf16*)dv);
  return 0;
}

}  // namespace

int ahb_attn_supported(int D) { return D == 64 || D == 96 || D == 128; }

int ahb_attn_fwd(const void* q, const void* k, const void* v, int BH, int L, int D, float scale, void* o, float* lse,
                 cudaStream_t st) {
  switch (D) {
    case 64: return launch_fwd<64>(q, k, v, BH, L, scale, o, lse, st);
    case 96: return launch_fwd<96>(q, k, v, BH, L, scale, o, lse, st);
    case 128: return launch_fwd<128>(q, k, v, BH, L, scale, o, lse, st);
    default: return -2;
  }
}

int ahb_attn_bwd(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
                 int BH, int L, int D, float scale, float* dq, void* dk, void* dv, cudaStream_t st) {
  switch (D) {
    case 64: return launch_bwd<64>(q, k, v, dout, lse, delta, BH, L, scale, dq, dk, dv, st);
    case 96: return launch_bwd<96>(q, k, v, dout, lse, delta, BH, L, scale, dq, dk, dv, st);
    case 128: return launch_bwd<128>(q, k, v, dout, lse, delta, BH, L, scale, dq, dk, dv, st);
    default: return -2;
  }
}
