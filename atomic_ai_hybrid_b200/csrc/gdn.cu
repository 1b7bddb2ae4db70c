// GDN-2 chunk-parallel backward kernels (head dim 128, chunk 64, per-channel gates).
//
// Chunked WY form and its forward kernels: gdn_tc.cu.  Backward (reference B1..B6,
// `atomic_ops/kernel_bwd_b*.py`, `kernel_trainable_B6.py`), after the reverse state
// recurrence (gdn_tc.cu: dh per chunk, dv_new):
//   gdn_bwd_states (products with h/dh: qg/kg chains, dw~, dAqk)
//   -> gdn_bwd_wy (through A: dw, dv, d(bk), dAkk)
//   -> gdn_bwd_intra (through Aqk/Akk + assembly + reverse cumsum for dg).
// Pairwise decays use a reference row r between j and i (r = first row of i's 16-row block),
// so both factors e^{gc_i-gc_r} and e^{gc_r-gc_j} stay <= 1 off the diagonal blocks.
#include "common.cuh"
#include "mma.cuh"
#include "launchers.h"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

constexpr int C = 64;       // chunk length
constexpr int D = 128;      // head dim (dk = dv)
constexpr int LDB = D + 8;  // bf16 row stride of C x D tiles
constexpr int LDF = D + 4;  // fp32 row stride of C x D tiles
constexpr int LDC = C + 4;  // fp32 row stride of C x C tiles
constexpr int NTH = 512;    // threads of the chunk-parallel kernels (16 warps: 4 row tiles x 4 column quarters)

AHB_DEVICE float bf(bf16 x) { return __bfloat162float(x); }
AHB_DEVICE float guard(float x) {  // nan_to_num(nan=0, +-inf -> +-1e4)
  if (x != x) return 0.f;
  return fminf(fmaxf(x, -1e4f), 1e4f);
}

// row index helpers
struct Idx {
  int64_t L, H, NC;
  AHB_DEVICE int64_t seq(int b, int64_t t, int h) const { return ((b * L + t) * H + h) * D; }  // (B,L,H,D)
  AHB_DEVICE int64_t chunk(int b, int h, int n) const { return ((int64_t)b * H + h) * NC + n; }
};

// Load a C x D bf16 tile of a (B,L,H,D) tensor into smem (row stride LDB).
AHB_DEVICE void load_seq_tile(bf16* dst, const bf16* src, const Idx& ix, int b, int n, int h, int nthreads) {
  for (int i = threadIdx.x; i < C * (D / 8); i += nthreads) {
    int r = i / (D / 8), c8 = (i % (D / 8)) * 8;
    *reinterpret_cast<uint4*>(dst + r * LDB + c8) =
        *reinterpret_cast<const uint4*>(src + ix.seq(b, (int64_t)n * C + r, h) + c8);
  }
}
// Load g (fp32, (B,L,H,D)) chunk and write its inclusive cumsum over rows into gc (stride LDF).
AHB_DEVICE void load_gc(float* gc, const float* g, const Idx& ix, int b, int n, int h, int nthreads) {
  for (int i = threadIdx.x; i < C * (D / 4); i += nthreads) {
    int r = i / (D / 4), c4 = (i % (D / 4)) * 4;
    *reinterpret_cast<float4*>(gc + r * LDF + c4) =
        *reinterpret_cast<const float4*>(g + ix.seq(b, (int64_t)n * C + r, h) + c4);
  }
  __syncthreads();
  if (threadIdx.x < D) {
    float s = 0.f;
    for (int r = 0; r < C; ++r) {
      s += gc[r * LDF + threadIdx.x];
      gc[r * LDF + threadIdx.x] = s;
    }
  }
  __syncthreads();
}
// contiguous C x D tile (chunk-major tensors) -> smem
AHB_DEVICE void load_chunk_tile(bf16* dst, const bf16* src, int nthreads) {
  for (int i = threadIdx.x; i < C * (D / 8); i += nthreads) {
    int r = i / (D / 8), c8 = (i % (D / 8)) * 8;
    *reinterpret_cast<uint4*>(dst + r * LDB + c8) = *reinterpret_cast<const uint4*>(src + r * D + c8);
  }
}
AHB_DEVICE void load_chunk_tile_f32(float* dst, int ld, const float* src, int rows, int cols, int nthreads) {
  for (int i = threadIdx.x; i < rows * (cols / 4); i += nthreads) {
    int r = i / (cols / 4), c4 = (i % (cols / 4)) * 4;
    *reinterpret_cast<float4*>(dst + r * ld + c4) = *reinterpret_cast<const float4*>(src + r * cols + c4);
  }
}

// Store an accumulator tile (NT n-tiles) as bf16 pairs: dst[row*ld + col]
template <int NT, class F>
AHB_DEVICE void store_pairs(float (*acc)[4], int m0, int n0, F&& put) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int c = n0 + 8 * j + 2 * t;
    put(m0 + g, c, acc[j][0], acc[j][1]);
    put(m0 + g + 8, c, acc[j][2], acc[j][3]);
  }
}

AHB_DEVICE void st_bf16x2(bf16* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack2(a, b); }

// ============================================================ backward: products with the states
// smem: h, dh bf16 [D][LDB]; do, vn, dvn, q, k bf16 [C][LDB]; gc f32 [C][LDF]; red f32 [D]
constexpr size_t SMEM_BWD_STATES = 2 * D * LDB * 2 + 5 * C * LDB * 2 + C * LDF * 4 + D * 4;

__global__ void __launch_bounds__(NTH, 1) gdn_bwd_states_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const float* __restrict__ g,
    const bf16* __restrict__ dout, const bf16* __restrict__ h_store, const bf16* __restrict__ dh_store,
    const bf16* __restrict__ vn_store, const bf16* __restrict__ dvn_store, float scale, int L, int H,
    float* __restrict__ dq_p, float* __restrict__ dk_p, float* __restrict__ dgc_p, float* __restrict__ dwt_o,
    float* __restrict__ dgcl_o, float* __restrict__ daqk_o) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* h_s = reinterpret_cast<bf16*>(smem);
  bf16* dh_s = h_s + D * LDB;
  bf16* do_s = dh_s + D * LDB;
  bf16* vn_s = do_s + C * LDB;
  bf16* dvn_s = vn_s + C * LDB;
  bf16* q_s = dvn_s + C * LDB;
  bf16* k_s = q_s + C * LDB;
  float* gc_s = reinterpret_cast<float*>(k_s + C * LDB);
  float* red_s = gc_s + C * LDF;

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const Idx ix{L, H, NC};
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t cb = ix.chunk(b, h, n);
  for (int i = tid; i < D * (D / 8); i += NTH) {
    int r = i / (D / 8), c8 = (i % (D / 8)) * 8;
    *reinterpret_cast<uint4*>(h_s + r * LDB + c8) = *reinterpret_cast<const uint4*>(h_store + cb * D * D + r * D + c8);
    *reinterpret_cast<uint4*>(dh_s + r * LDB + c8) =
        *reinterpret_cast<const uint4*>(dh_store + cb * D * D + r * D + c8);
  }
  load_seq_tile(do_s, dout, ix, b, n, h, NTH);
  load_seq_tile(q_s, q, ix, b, n, h, NTH);
  load_seq_tile(k_s, k, ix, b, n, h, NTH);
  load_chunk_tile(vn_s, vn_store + cb * C * D, NTH);
  load_chunk_tile(dvn_s, dvn_store + cb * C * D, NTH);
  if (tid < D) red_s[tid] = 0.f;
  load_gc(gc_s, g, ix, b, n, h, NTH);

  const int mt = warp & 3, nq = warp >> 2;
  const int m0 = 16 * mt, n0 = 32 * nq;
  float acc[4][4], dg[4][4];
  zero_acc<4>(dg);
  // P1 = do h^T  -> dq_p = scale P1 e^gc ; dgc += dq_p q
  zero_acc<4>(acc);
  warp_mma<4>(acc, RowA16{do_s, LDB}, NKB16{h_s, LDB}, m0, n0, 0, D);
  {
    const int lane = tid & 31, gq = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int r = m0 + gq + (e >> 1) * 8, c = n0 + 8 * j + 2 * t + (e & 1);
        float x = scale * acc[j][e] * __expf(gc_s[r * LDF + c]);
        dq_p[cb * C * D + r * D + c] = x;
        dg[j][e] += x * bf(q_s[r * LDB + c]);
      }
  }
  // P2 = vn dh^T -> dk_p = P2 e^{gcl-gc}; dgc -= P2 kg; dgcl += P2 kg
  zero_acc<4>(acc);
  warp_mma<4>(acc, RowA16{vn_s, LDB}, NKB16{dh_s, LDB}, m0, n0, 0, D);
  {
    const int lane = tid & 31, gq = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int r = m0 + gq + (e >> 1) * 8, c = n0 + 8 * j + 2 * t + (e & 1);
        float ex = __expf(gc_s[(C - 1) * LDF + c] - gc_s[r * LDF + c]);
        float x = acc[j][e];
        dk_p[cb * C * D + r * D + c] = x * ex;
        float t2 = x * ex * bf(k_s[r * LDB + c]);
        dg[j][e] -= t2;
        atomicAdd(red_s + c, t2);
      }
  }
  // P3 = dvn h^T -> dwt = -P3
  zero_acc<4>(acc);
  warp_mma<4>(acc, RowA16{dvn_s, LDB}, NKB16{h_s, LDB}, m0, n0, 0, D);
  store_pairs<4>(acc, m0, n0, [&](int r, int c, float x0, float x1) {
    *reinterpret_cast<float2*>(dwt_o + cb * C * D + r * D + c) = make_float2(-x0, -x1);
  });
  store_pairs<4>(dg, m0, n0, [&](int r, int c, float x0, float x1) {
    *reinterpret_cast<float2*>(dgc_p + cb * C * D + r * D + c) = make_float2(x0, x1);
  });
  // dAqk = do vn^T (causal), unscaled
  {
    float a4[2][4];
    zero_acc<2>(a4);
    warp_mma<2>(a4, RowA16{do_s, LDB}, NKB16{vn_s, LDB}, m0, 16 * nq, 0, D);
    store_pairs<2>(a4, m0, 16 * nq, [&](int r, int c, float x0, float x1) {
      *reinterpret_cast<float2*>(daqk_o + cb * C * C + r * C + c) =
          make_float2(c <= r ? x0 : 0.f, c + 1 <= r ? x1 : 0.f);
    });
  }
  // dgcl += e^{gcl} sum_v dh h
  {
    const int d = tid >> 2, quarter = tid & 3;
    float s = 0.f;
    for (int vv = quarter * 32; vv < quarter * 32 + 32; ++vv) s += bf(dh_s[d * LDB + vv]) * bf(h_s[d * LDB + vv]);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    __syncthreads();
    if (quarter == 0) dgcl_o[cb * D + d] = red_s[d] + __expf(gc_s[(C - 1) * LDF + d]) * s;
  }
}

// ============================================================ backward through the WY representation
// smem: k, b, w, v, du bf16 [C][LDB]; gc, dwt f32 [C][LDF]; a, da, t f32 [C][LDC]
constexpr size_t SMEM_BWD_WY = 5 * C * LDB * 2 + 2 * C * LDF * 4 + 3 * C * LDC * 4;

__global__ void __launch_bounds__(NTH, 1) gdn_bwd_wy_kernel(
    const bf16* __restrict__ k, const bf16* __restrict__ v, const float* __restrict__ g,
    const bf16* __restrict__ bg, const bf16* __restrict__ wg, const float* __restrict__ a_store,
    const bf16* __restrict__ dvn_store, const float* __restrict__ dwt, int L, int H, bf16* __restrict__ dv_o,
    bf16* __restrict__ dw_o, float* __restrict__ dbk_o, float* __restrict__ dgc_o, float* __restrict__ dakk_o) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* k_s = reinterpret_cast<bf16*>(smem);
  bf16* b_s = k_s + C * LDB;
  bf16* w_s = b_s + C * LDB;
  bf16* v_s = w_s + C * LDB;
  bf16* du_s = v_s + C * LDB;
  float* gc_s = reinterpret_cast<float*>(du_s + C * LDB);
  float* dwt_s = gc_s + C * LDF;
  float* a_s = dwt_s + C * LDF;
  float* da_s = a_s + C * LDC;
  float* t_s = da_s + C * LDC;

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const Idx ix{L, H, NC};
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t cb = ix.chunk(b, h, n);
  load_seq_tile(k_s, k, ix, b, n, h, NTH);
  load_seq_tile(b_s, bg, ix, b, n, h, NTH);
  load_seq_tile(w_s, wg, ix, b, n, h, NTH);
  load_seq_tile(v_s, v, ix, b, n, h, NTH);
  load_chunk_tile(du_s, dvn_store + cb * C * D, NTH);
  load_chunk_tile_f32(dwt_s, LDF, dwt + cb * C * D, C, D, NTH);
  load_chunk_tile_f32(a_s, LDC, a_store + cb * C * C, C, C, NTH);
  load_gc(gc_s, g, ix, b, n, h, NTH);

  const int mt = warp & 3, nq = warp >> 2;
  // dA (strictly lower) = du (w v)^T + dwt (bk e^gc)^T
  {
    auto fb_wv = [&](int kv, int nj) -> uint32_t {
      return pack2(bf(w_s[nj * LDB + kv]) * bf(v_s[nj * LDB + kv]),
                   bf(w_s[nj * LDB + kv + 1]) * bf(v_s[nj * LDB + kv + 1]));
    };
    auto fb_bke = [&](int kd, int nj) -> uint32_t {
      const float* gj = gc_s + nj * LDF;
      return pack2(bf(b_s[nj * LDB + kd]) * bf(k_s[nj * LDB + kd]) * __expf(gj[kd]),
                   bf(b_s[nj * LDB + kd + 1]) * bf(k_s[nj * LDB + kd + 1]) * __expf(gj[kd + 1]));
    };
    float acc[2][4];
    zero_acc<2>(acc);
    warp_mma<2>(acc, RowA16{du_s, LDB}, fb_wv, 16 * mt, 16 * nq, 0, D);
    warp_mma<2>(acc, RowA32{dwt_s, LDF}, fb_bke, 16 * mt, 16 * nq, 0, D);
    for_acc<2>(acc, 16 * mt, 16 * nq, [&](int r, int c, float& x) { da_s[r * LDC + c] = c < r ? x : 0.f; });
  }
  // d(wv) = A^T du -> dw, dv ; d(bke) = A^T dwt -> dbk_wy, dgc_wy
  {
    const int m0 = 16 * mt, n0 = 32 * nq;
    float acc[4][4];
    zero_acc<4>(acc);
    warp_mma<4>(acc, ColA32{a_s, LDC}, KNB16{du_s, LDB}, m0, n0, m0, C);
    store_pairs<4>(acc, m0, n0, [&](int r, int c, float x0, float x1) {
      int64_t gi = ix.seq(b, (int64_t)n * C + r, h) + c;
      st_bf16x2(dw_o + gi, x0 * bf(v_s[r * LDB + c]), x1 * bf(v_s[r * LDB + c + 1]));
      st_bf16x2(dv_o + gi, x0 * bf(w_s[r * LDB + c]), x1 * bf(w_s[r * LDB + c + 1]));
    });
    zero_acc<4>(acc);
    warp_mma<4>(acc, ColA32{a_s, LDC}, KNB32{dwt_s, LDF}, m0, n0, m0, C);
    store_pairs<4>(acc, m0, n0, [&](int r, int c, float x0, float x1) {
      float e0 = __expf(gc_s[r * LDF + c]), e1 = __expf(gc_s[r * LDF + c + 1]);
      float d0 = x0 * e0, d1 = x1 * e1;
      *reinterpret_cast<float2*>(dbk_o + cb * C * D + r * D + c) = make_float2(d0, d1);
      float bk0 = bf(b_s[r * LDB + c]) * bf(k_s[r * LDB + c]);
      float bk1 = bf(b_s[r * LDB + c + 1]) * bf(k_s[r * LDB + c + 1]);
      *reinterpret_cast<float2*>(dgc_o + cb * C * D + r * D + c) = make_float2(d0 * bk0, d1 * bk1);
    });
  }
  __syncthreads();
  // T = dA A^T
  {
    float acc[2][4];
    zero_acc<2>(acc);
    warp_mma<2>(acc, RowA32{da_s, LDC}, NKB32{a_s, LDC}, 16 * mt, 16 * nq, 0, 16 * (mt + 1));
    for_acc<2>(acc, 16 * mt, 16 * nq, [&](int r, int c, float& x) { t_s[r * LDC + c] = x; });
  }
  __syncthreads();
  // dAkk = -(A^T T), strictly lower
  {
    float acc[2][4];
    zero_acc<2>(acc);
    warp_mma<2>(acc, ColA32{a_s, LDC}, KNB32{t_s, LDC}, 16 * mt, 16 * nq, 16 * mt, C);
    store_pairs<2>(acc, 16 * mt, 16 * nq, [&](int r, int c, float x0, float x1) {
      *reinterpret_cast<float2*>(dakk_o + cb * C * C + r * C + c) =
          make_float2(c < r ? -x0 : 0.f, c + 1 < r ? -x1 : 0.f);
    });
  }
}

// ============================================================ backward through Aqk / Akk + assembly
// smem: q, k, b bf16 [C][LDB]; gc, dgc f32 [C][LDF]; daqk, dakk f32 [C][LDC]
constexpr size_t SMEM_BWD_INTRA = 3 * C * LDB * 2 + 2 * C * LDF * 4 + 2 * C * LDC * 4;

__global__ void __launch_bounds__(NTH, 1) gdn_bwd_intra_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const float* __restrict__ g,
    const bf16* __restrict__ bg, const float* __restrict__ daqk, const float* __restrict__ dakk,
    const float* __restrict__ dq_p, const float* __restrict__ dk_p, const float* __restrict__ dgc_p,
    const float* __restrict__ dbk_wy, const float* __restrict__ dgc_wy, const float* __restrict__ dgcl,
    float scale, int L, int H, bf16* __restrict__ dq_o, bf16* __restrict__ dk_o, bf16* __restrict__ db_o,
    float* __restrict__ dg_o) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* q_s = reinterpret_cast<bf16*>(smem);
  bf16* k_s = q_s + C * LDB;
  bf16* b_s = k_s + C * LDB;
  float* gc_s = reinterpret_cast<float*>(b_s + C * LDB);
  float* dgc_s = gc_s + C * LDF;
  float* daqk_s = dgc_s + C * LDF;
  float* dakk_s = daqk_s + C * LDC;

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const Idx ix{L, H, NC};
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t cb = ix.chunk(b, h, n);
  load_seq_tile(q_s, q, ix, b, n, h, NTH);
  load_seq_tile(k_s, k, ix, b, n, h, NTH);
  load_seq_tile(b_s, bg, ix, b, n, h, NTH);
  load_chunk_tile_f32(daqk_s, LDC, daqk + cb * C * C, C, C, NTH);
  load_chunk_tile_f32(dakk_s, LDC, dakk + cb * C * C, C, C, NTH);
  load_gc(gc_s, g, ix, b, n, h, NTH);

  // warp tile: rows of block I (16 rows), 32 channel columns (quarter nq)
  const int I = warp & 3, nq = warp >> 2;
  const int m0 = 16 * I, n0 = 32 * nq;
  const int r0 = m0;  // reference row of block I
  // diagonal blocks are factorised like the others unless their decay span could overflow
  __shared__ int exact_blk[4];
  if (warp < 4) {
    const int lane = tid & 31;
    float span = 0.f;
    for (int d = lane; d < D; d += 32) span = fmaxf(span, gc_s[16 * warp * LDF + d] - gc_s[(16 * warp + 15) * LDF + d]);
    span = warp_max(span);
    if (lane == 0) exact_blk[warp] = !(span <= 60.f);
  }
  __syncthreads();
  const bool exact = exact_blk[I];
  float dq[4][4], dbk[4][4], dk[4][4];
  zero_acc<4>(dq);
  zero_acc<4>(dbk);
  zero_acc<4>(dk);
  // (a) row side, columns j < 16I (and j <= i inside block I unless it is exact): dq_I, dbk_I
  //     (B = k_j e^{gc_r - gc_j}, A masked to the causal pairs)
  const int a_hi = exact ? r0 : r0 + 16;
  if (a_hi > 0) {
    const float* gr = gc_s + r0 * LDF;
    auto fb = [&](int kj, int nd) -> uint32_t {
      return pack2(bf(k_s[kj * LDB + nd]) * __expf(gr[nd] - gc_s[kj * LDF + nd]),
                   bf(k_s[(kj + 1) * LDB + nd]) * __expf(gr[nd] - gc_s[(kj + 1) * LDF + nd]));
    };
    auto fa_q = [&](int r, int kk) -> uint32_t {
      return pack2(kk <= r ? daqk_s[r * LDC + kk] : 0.f, kk + 1 <= r ? daqk_s[r * LDC + kk + 1] : 0.f);
    };
    auto fa_k = [&](int r, int kk) -> uint32_t {
      return pack2(kk < r ? dakk_s[r * LDC + kk] : 0.f, kk + 1 < r ? dakk_s[r * LDC + kk + 1] : 0.f);
    };
    warp_mma<4>(dq, fa_q, fb, m0, n0, 0, a_hi);
    warp_mma<4>(dbk, fa_k, fb, m0, n0, 0, a_hi);
    for_acc<4>(dq, m0, n0, [&](int r, int c, float& x) { x *= scale * __expf(gc_s[r * LDF + c] - gr[c]); });
    for_acc<4>(dbk, m0, n0, [&](int r, int c, float& x) { x *= __expf(gc_s[r * LDF + c] - gr[c]); });
  }
  // (b) column side from blocks I2 >= I (I2 = I only when factorised):
  //     dk_j += e^{gc_r2 - gc_j} sum_i dA[i,j] x_i e^{gc_i - gc_r2}, pairs with i >= j (i > j for Akk)
  for (int I2 = exact ? I + 1 : I; I2 < 4; ++I2) {
    const int r2 = 16 * I2;
    const float* gr = gc_s + r2 * LDF;
    auto fa_q = [&](int rj, int ci) -> uint32_t {  // A(j, i) = daqk[r2+i][m0+j]
      const int i0 = r2 + ci;
      return pack2(i0 >= rj ? daqk_s[i0 * LDC + rj] : 0.f, i0 + 1 >= rj ? daqk_s[(i0 + 1) * LDC + rj] : 0.f);
    };
    auto fa_k = [&](int rj, int ci) -> uint32_t {
      const int i0 = r2 + ci;
      return pack2(i0 > rj ? dakk_s[i0 * LDC + rj] : 0.f, i0 + 1 > rj ? dakk_s[(i0 + 1) * LDC + rj] : 0.f);
    };
    auto fb_q = [&](int ki, int nd) -> uint32_t {
      return pack2(bf(q_s[(r2 + ki) * LDB + nd]) * __expf(gc_s[(r2 + ki) * LDF + nd] - gr[nd]),
                   bf(q_s[(r2 + ki + 1) * LDB + nd]) * __expf(gc_s[(r2 + ki + 1) * LDF + nd] - gr[nd]));
    };
    auto fb_k = [&](int ki, int nd) -> uint32_t {
      const int i0 = r2 + ki, i1 = i0 + 1;
      return pack2(bf(b_s[i0 * LDB + nd]) * bf(k_s[i0 * LDB + nd]) * __expf(gc_s[i0 * LDF + nd] - gr[nd]),
                   bf(b_s[i1 * LDB + nd]) * bf(k_s[i1 * LDB + nd]) * __expf(gc_s[i1 * LDF + nd] - gr[nd]));
    };
    float t1[4][4], t2[4][4];
    zero_acc<4>(t1);
    zero_acc<4>(t2);
    // A operand rows are j within block I: pass m0 offset through the loader (rj includes m0)
    warp_mma<4>(t1, fa_q, fb_q, m0, n0, 0, 16);
    warp_mma<4>(t2, fa_k, fb_k, m0, n0, 0, 16);
    const int lane = tid & 31, gq = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int r = m0 + gq + (e >> 1) * 8, c = n0 + 8 * j + 2 * t + (e & 1);
        dk[j][e] += (scale * t1[j][e] + t2[j][e]) * __expf(gr[c] - gc_s[r * LDF + c]);
      }
  }
  // (c) exact diagonal sums (blocks with a wide decay span only) and assembly, per fragment element
  {
    const int lane = tid & 31, gq = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = m0 + gq + (e >> 1) * 8, c = n0 + 8 * j + 2 * t + (e & 1);
        const float gi = gc_s[r * LDF + c];
        const float qi = bf(q_s[r * LDB + c]);
        const float bki = bf(b_s[r * LDB + c]) * bf(k_s[r * LDB + c]);
        const float ki = bf(k_s[r * LDB + c]);
        float aq = 0.f, ab = 0.f, ak = 0.f;
        for (int s = m0; exact && s < m0 + 16; ++s) {
          const float gs = gc_s[s * LDF + c];
          if (s <= r) {  // row side: pairs (r, s), s <= r
            const float ex = __expf(fmaxf(gi - gs, -20.f));
            const float ks = bf(k_s[s * LDB + c]) * ex;
            aq += daqk_s[r * LDC + s] * ks;
            if (s < r) ab += dakk_s[r * LDC + s] * ks;
          }
          if (s >= r) {  // column side: pairs (s, r), s >= r
            const float ex = __expf(fmaxf(gs - gi, -20.f));
            const float qs = bf(q_s[s * LDB + c]);
            const float bks = bf(b_s[s * LDB + c]) * bf(k_s[s * LDB + c]);
            ak += (scale * daqk_s[s * LDC + r] * qs + (s > r ? dakk_s[s * LDC + r] * bks : 0.f)) * ex;
          }
        }
        dq[j][e] += scale * aq;
        dbk[j][e] += ab;
        dk[j][e] += ak;
        // assembly
        const int64_t ci = cb * C * D + (int64_t)r * D + c;
        const float dbk_t = dbk[j][e] + dbk_wy[ci];
        const float dq_t = dq[j][e] + dq_p[ci];
        const float dk_t = dk[j][e] + dk_p[ci] + dbk_t * bf(b_s[r * LDB + c]);
        const float db_t = dbk_t * ki;
        float dgc = dgc_p[ci] + dgc_wy[ci] + qi * dq[j][e] + bki * dbk[j][e] - ki * dk[j][e];
        if (r == C - 1) dgc += dgcl[cb * D + c];
        dgc_s[r * LDF + c] = dgc;
        const int64_t gi2 = ix.seq(b, (int64_t)n * C + r, h) + c;
        dq_o[gi2] = __float2bfloat16_rn(dq_t);
        dk_o[gi2] = __float2bfloat16_rn(dk_t);
        db_o[gi2] = __float2bfloat16_rn(db_t);
      }
  }
  __syncthreads();
  // dg = reverse cumsum over the chunk rows
  if (tid < D) {
    float s = 0.f;
    for (int r = C - 1; r >= 0; --r) {
      s += dgc_s[r * LDF + tid];
      dg_o[ix.seq(b, (int64_t)n * C + r, h) + tid] = s;
    }
  }
}

template <class K>
void set_smem(K kernel, size_t bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

// ===================================================================== launchers
int ahb_gdn_supported(int D_) { return D_ == D ? C : 0; }

void ahb_gdn_bwd_states(const void* q, const void* k, const float* g, const void* dout, const void* h_store,
                        const void* dh_store, const void* vn_store, const void* dvn_store, float scale, int B, int L,
                        int H, float* dq_p, float* dk_p, float* dgc_p, float* dwt, float* dgcl, float* daqk,
                        cudaStream_t st) {
  static bool init = false;
  if (!init) { set_smem(gdn_bwd_states_kernel, SMEM_BWD_STATES); init = true; }
  dim3 grid(L / C, H, B);
  gdn_bwd_states_kernel<<<grid, NTH, SMEM_BWD_STATES, st>>>(
      (const bf16*)q, (const bf16*)k, g, (const bf16*)dout, (const bf16*)h_store, (const bf16*)dh_store,
      (const bf16*)vn_store, (const bf16*)dvn_store, scale, L, H, dq_p, dk_p, dgc_p, dwt, dgcl, daqk);
}

void ahb_gdn_bwd_wy(const void* k, const void* v, const float* g, const void* bg, const void* wg,
                    const float* a_store, const void* dvn_store, const float* dwt, int B, int L, int H, void* dv,
                    void* dw, float* dbk_wy, float* dgc_wy, float* dakk, cudaStream_t st) {
  static bool init = false;
  if (!init) { set_smem(gdn_bwd_wy_kernel, SMEM_BWD_WY); init = true; }
  dim3 grid(L / C, H, B);
  gdn_bwd_wy_kernel<<<grid, NTH, SMEM_BWD_WY, st>>>((const bf16*)k, (const bf16*)v, g, (const bf16*)bg,
                                                    (const bf16*)wg, a_store, (const bf16*)dvn_store, dwt, L, H,
                                                    (bf16*)dv, (bf16*)dw, dbk_wy, dgc_wy, dakk);
}

void ahb_gdn_bwd_intra(const void* q, const void* k, const float* g, const void* bg, const float* daqk,
                       const float* dakk, const float* dq_p, const float* dk_p, const float* dgc_p,
                       const float* dbk_wy, const float* dgc_wy, const float* dgcl, float scale, int B, int L, int H,
                       void* dq, void* dk, void* db, float* dg, cudaStream_t st) {
  static bool init = false;
  if (!init) { set_smem(gdn_bwd_intra_kernel, SMEM_BWD_INTRA); init = true; }
  dim3 grid(L / C, H, B);
  gdn_bwd_intra_kernel<<<grid, NTH, SMEM_BWD_INTRA, st>>>(
      (const bf16*)q, (const bf16*)k, g, (const bf16*)bg, daqk, dakk, dq_p, dk_p, dgc_p, dbk_wy, dgc_wy, dgcl, scale,
      L, H, (bf16*)dq, (bf16*)dk, (bf16*)db, dg);
}
