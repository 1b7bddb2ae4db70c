// Grouped GEMM for the MoE experts on the 5th-generation tensor cores (tcgen05).
//
// One persistent, warp-specialised kernel covers every expert GEMM of the MoE
// forward and backward (reference `atomic_ops/moe_gmm.py:251-336`, megablox
// gmm/tgmm):
//   * M-grouped  (fwd, dgrad): rows of the expert-sorted token matrix are split in
//     groups (one per expert, each padded to a multiple of 128 rows, so no tile
//     straddles two experts); group e multiplies by expert e's weight.
//   * K-grouped  (wgrad): the contraction runs over group e's token rows and the
//     product is ADDED into expert e's fp32 gradient (the flat gradient store).
// Roles per CTA (192 threads): warp 0 issues TMA tile loads (no multicast) into a
// 4-stage 128B-swizzled ring; one thread of warp 1 issues tcgen05.mma into a
// double-buffered TMEM accumulator (2 x 256 fp32 columns); warps 2-5 read the
// accumulator with tcgen05.ld and run the fused epilogue (SwiGLU / GELU forward
// with saved pre-activations, their backward, bf16 store or fp32 accumulate)
// while the next tile's MMAs proceed.  Every mbarrier wait is bounded: on a
// timeout the kernel records an error code, stops all roles and frees its TMEM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstring>
#include "common.cuh"
#include "sm100.cuh"
#include "launchers.h"

using namespace ahb;
using namespace ahb::sm100;
using bf16 = __nv_bfloat16;

namespace {

constexpr int BM = 128, BK = 64, STAGES = 4, NTHREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = 256 * BK * 2;  // 32 KB (NB * BNacc = 256 columns)
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;

enum Epi { EPI_STORE = 0, EPI_SWIGLU_FWD = 1, EPI_GELU_FWD = 2, EPI_SWIGLU_BWD = 3, EPI_GELU_BWD = 4, EPI_ACC = 5,
           EPI_STORE_PEER = 6, EPI_CE_FWD = 7, EPI_CE_BWD = 8 };

constexpr int MAX_PEERS = 8;
// EPI_STORE_PEER stages each warp's 32 x 256 output rows in shared memory and writes every row
// as one 512-byte warp store (coalesced NVLink writes); it runs a 3-stage ring to make room.
constexpr int STG_LD = 256 + 8;
constexpr size_t STG_BYTES = 4 * 32 * STG_LD * 2;
template <int EPI>
constexpr int n_stages() { return EPI == EPI_STORE_PEER ? 3 : STAGES; }
template <int EPI>
constexpr size_t smem_bytes() {
  return (size_t)n_stages<EPI>() * STAGE_BYTES + 1024 + 1024 + (EPI == EPI_STORE_PEER ? STG_BYTES : 0);
}

struct Params {
  CUtensorMap ta0, ta1, tb0, tb1;
  const int* grp_off;  // E+1 offsets (multiples of 128) into A's rows (M-grouped) or token rows (K-grouped)
  int E, N, Mout, kb_split, kb_total, b_rows;
  void* out0;
  void* out1;
  void* out2;
  const bf16* aux0;
  const bf16* aux1;
  const float* alpha;  // optional device scalar multiplying the product (STORE / ACC epilogues)
  float clip;
  int* err;
  // EPI_STORE_PEER: group g's rows go to out_tab[g] (row - grp_off[g]) * N + col, which may
  // be another GPU's memory (plain 16-byte stores over NVLink); M tiles are visited from
  // tile m_rot on, so that the ranks start on different destinations
  void* out_tab[MAX_PEERS];
  int m_rot;
  // M-grouped raster: 0 = N tiles fastest (the A row tile stays hot), 1 = M tiles fastest (the B
  // column tile stays hot while the CTAs sweep the rows: the LM head, whose vocabulary matrix is
  // larger than L2 and would otherwise be read once per row tile)
  int m_fast;
  int m_limit;  // M-grouped: rows at or beyond it are not stored (0: every row of the padded groups)
  // LM-head cross entropy (EPI_CE_*): token labels (-100 = masked), row log-sum-exp (backward),
  // label smoothing weights sp = 1 - ls and sn = ls / (V - 1), vocabulary tiles per row
  const int64_t* labels;
  const float* row_lse;
  float ce_sp, ce_sn;
  int ce_tiles;
  // EPI_STORE extras (dense projections): bias per output column, and a bf16 matrix of the
  // output's shape added to the product (accumulation over several launches, beta = 1)
  const bf16* bias;
  const bf16* beta_src;
  int acc_bf16;  // EPI_ACC into bf16 accumulators (AHB_GEMM_ACC_BF16)
};

AHB_DEVICE float clampf(float x, float c) { return c > 0.f ? fminf(fmaxf(x, -c), c) : x; }
AHB_DEVICE float gelu_t(float x) {
  const float k = 0.7978845608028654f;
  return 0.5f * x * (1.f + tanhf(k * (x + 0.044715f * x * x * x)));
}
AHB_DEVICE float gelu_t_grad(float x) {
  const float k = 0.7978845608028654f;
  const float t = tanhf(k * (x + 0.044715f * x * x * x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k * (1.f + 3.f * 0.044715f * x * x);
}
AHB_DEVICE void store_bf16x32(bf16* dst, const float* v) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[i], v[i + 1]);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
    __nv_bfloat162 p3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
    uint4 w;
    w.x = *reinterpret_cast<uint32_t*>(&p0);
    w.y = *reinterpret_cast<uint32_t*>(&p1);
    w.z = *reinterpret_cast<uint32_t*>(&p2);
    w.w = *reinterpret_cast<uint32_t*>(&p3);
    *reinterpret_cast<uint4*>(dst + i) = w;
  }
}

// 32 consecutive bf16 accumulators += alpha * v (read, add in fp32, round once)
AHB_DEVICE void acc_add_bf16(bf16* d, const float* v, float alpha) {
  bf16 cur[32];
#pragma unroll
  for (int i = 0; i < 32; i += 8) *reinterpret_cast<uint4*>(cur + i) = *reinterpret_cast<const uint4*>(d + i);
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = __bfloat162float(cur[i]) + alpha * v[i];
  store_bf16x32(d, o);
}

struct Tile {
  int e, m0, n0, k0row, nkb;
};

template <bool KGROUP>
AHB_DEVICE bool decode(const Params& p, const int* off, int tile, int n_tiles, Tile& t) {
  if (!KGROUP) {
    const int m_total = off[p.E] / BM;
    const int mt = p.m_fast ? (tile % m_total + p.m_rot) % m_total : (tile / n_tiles + p.m_rot) % m_total;
    const int nt = p.m_fast ? tile / m_total : tile % n_tiles;
    t.m0 = mt * BM;
    int e = 0;
    while (e + 1 < p.E && off[e + 1] <= t.m0) ++e;
    t.e = e;
    t.n0 = nt;
    t.k0row = 0;
    t.nkb = p.kb_total;
  } else {
    const int m_tiles = p.Mout / BM;
    const int per_e = m_tiles * n_tiles;
    t.e = tile / per_e;
    const int r = tile % per_e;
    t.m0 = (r / n_tiles) * BM;
    t.n0 = r % n_tiles;
    t.k0row = off[t.e];
    t.nkb = (off[t.e + 1] - off[t.e]) / BK;
  }
  return true;
}

// Epilogue of one accumulator tile for the 32 rows of one epilogue warp: `tb` is the warp's TMEM
// lane quarter at the accumulator, `row_base` the tile row of its lane 0 (rows at or beyond
// `m_limit`, when set, are not written).
template <int EPI, int NB>
AHB_DEVICE void epilogue_tile(const Params& p, const int* off, const Tile& t, uint32_t tb, int row_base, int lane,
                              unsigned char* stg_base, int q) {
  constexpr int BNA = 256 / NB;
  const int row = row_base + lane;
  const int n0 = t.n0 * BNA;
  const bool live = p.m_limit <= 0 || row < p.m_limit;
  const float alpha = p.alpha ? *p.alpha : 1.f;
  if constexpr (EPI == EPI_CE_FWD || EPI == EPI_CE_BWD) {
    // logits of this row over the tile's vocabulary columns, rounded to bf16 and clipped as the
    // row kernel of the unfused head reads them (reference `optimizer.py:244-312`)
    const int64_t lab = live ? p.labels[row] : -100;
    const bool valid = lab != -100;
    const int y = valid ? (int)(lab < 0 ? 0 : (lab >= p.N ? p.N - 1 : lab)) : -1;
    if constexpr (EPI == EPI_CE_FWD) {
      // per-row partials of this tile: running max, sum of e^{z - max}, z at the label, sum of z
      float m = -INFINITY, s = 0.f, zs = 0.f, zy = 0.f;
#pragma unroll 1
      for (int c = 0; c < BNA / 32; ++c) {
        const int col = n0 + c * 32;
        if (col >= p.N) break;
        float v[32];
        tmem_ld32(tb + c * 32, v);
        float cm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = sanitize(__bfloat162float(__float2bfloat16_rn(v[i])), 1e4f);
          cm = fmaxf(cm, v[i]);
          zs += v[i];
          if (col + i == y) zy = v[i];
        }
        const float mn = fmaxf(m, cm);
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) a += __expf(v[i] - mn);
        s = s * __expf(m - mn) + a;
        m = mn;
      }
      if (live) reinterpret_cast<float4*>(p.out0)[static_cast<int64_t>(row) * p.ce_tiles + t.n0] = make_float4(m, s, zy, zs);
    } else {
      // d loss_row / d z = softmax - sn - (sp - sn) [v == y]; zero on masked and padding rows
      const float lse = valid ? p.row_lse[row] : 0.f;
#pragma unroll 1
      for (int c = 0; c < BNA / 32; ++c) {
        const int col = n0 + c * 32;
        if (col >= p.N) break;
        float v[32];
        tmem_ld32(tb + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float z = sanitize(__bfloat162float(__float2bfloat16_rn(v[i])), 1e4f);
          v[i] = valid ? __expf(z - lse) - p.ce_sn - (col + i == y ? p.ce_sp - p.ce_sn : 0.f) : 0.f;
        }
        store_bf16x32(static_cast<bf16*>(p.out0) + static_cast<int64_t>(row) * p.N + col, v);
      }
    }
    return;
  }
  if constexpr (EPI == EPI_STORE_PEER) {
    bf16* stg = reinterpret_cast<bf16*>(stg_base) + q * 32 * STG_LD;
#pragma unroll 1
    for (int c = 0; c < BNA / 32; ++c) {
      if (n0 + c * 32 >= p.N) break;
      float v0[32];
      tmem_ld32(tb + c * 32, v0);
      store_bf16x32(stg + lane * STG_LD + c * 32, v0);
    }
    __syncwarp();
    // row r of the warp's 32: lanes write its 256 columns as one 512-byte segment
    bf16* dst = static_cast<bf16*>(p.out_tab[t.e]) + static_cast<int64_t>(row_base - off[t.e]) * p.N;
    const int col = n0 + lane * 8;
    if (col < p.N) {
#pragma unroll 4
      for (int r = 0; r < 32; ++r)
        *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * p.N + col) =
            *reinterpret_cast<const uint4*>(stg + r * STG_LD + lane * 8);
    }
    __syncwarp();
  }
#pragma unroll 1
  for (int c = 0; c < (EPI == EPI_STORE_PEER ? 0 : BNA / 32); ++c) {
    const int col = n0 + c * 32;
    if (col >= p.N) break;  // partial last tile (N % 32 == 0)
    float v0[32];
    tmem_ld32(tb + c * 32, v0);
    const int64_t o = static_cast<int64_t>(row) * p.N + col;
    if constexpr (EPI == EPI_STORE) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v0[i] = v0[i] * alpha;
      if (p.bias) {
        bf16 bv[32];
#pragma unroll
        for (int i = 0; i < 32; i += 8) *reinterpret_cast<uint4*>(bv + i) = *reinterpret_cast<const uint4*>(p.bias + col + i);
#pragma unroll
        for (int i = 0; i < 32; ++i) v0[i] += __bfloat162float(bv[i]);
      }
      if (p.beta_src && live) {
        bf16 sv[32];
#pragma unroll
        for (int i = 0; i < 32; i += 8) *reinterpret_cast<uint4*>(sv + i) = *reinterpret_cast<const uint4*>(p.beta_src + o + i);
#pragma unroll
        for (int i = 0; i < 32; ++i) v0[i] += __bfloat162float(sv[i]);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v0[i] = clampf(v0[i], p.clip);
      if (live) store_bf16x32(static_cast<bf16*>(p.out0) + o, v0);
    } else if constexpr (EPI == EPI_SWIGLU_FWD) {
      float v1[32], h[32];
      tmem_ld32(tb + BNA + c * 32, v1);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v0[i] = clampf(v0[i], p.clip);
        v1[i] = clampf(v1[i], p.clip);
        h[i] = v0[i] * sigmoidf_(v0[i]) * v1[i];
      }
      store_bf16x32(static_cast<bf16*>(p.out0) + o, h);
      store_bf16x32(static_cast<bf16*>(p.out1) + o, v0);
      store_bf16x32(static_cast<bf16*>(p.out2) + o, v1);
    } else if constexpr (EPI == EPI_GELU_FWD) {
      float h[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v0[i] = clampf(v0[i], p.clip);
        h[i] = gelu_t(v0[i]);
      }
      store_bf16x32(static_cast<bf16*>(p.out0) + o, h);
      store_bf16x32(static_cast<bf16*>(p.out1) + o, v0);
    } else if constexpr (EPI == EPI_SWIGLU_BWD) {
      float d1[32], d3[32];
      bf16 a1v[32], a3v[32];
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        *reinterpret_cast<uint4*>(a1v + i) = *reinterpret_cast<const uint4*>(p.aux0 + o + i);
        *reinterpret_cast<uint4*>(a3v + i) = *reinterpret_cast<const uint4*>(p.aux1 + o + i);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a1 = __bfloat162float(a1v[i]), a3 = __bfloat162float(a3v[i]);
        const float s = sigmoidf_(a1);
        d1[i] = v0[i] * a3 * s * (1.f + a1 * (1.f - s));
        d3[i] = v0[i] * a1 * s;
      }
      store_bf16x32(static_cast<bf16*>(p.out0) + o, d1);
      store_bf16x32(static_cast<bf16*>(p.out1) + o, d3);
    } else if constexpr (EPI == EPI_GELU_BWD) {
      bf16 a1v[32];
#pragma unroll
      for (int i = 0; i < 32; i += 8) *reinterpret_cast<uint4*>(a1v + i) = *reinterpret_cast<const uint4*>(p.aux0 + o + i);
#pragma unroll
      for (int i = 0; i < 32; ++i) v0[i] *= gelu_t_grad(__bfloat162float(a1v[i]));
      store_bf16x32(static_cast<bf16*>(p.out0) + o, v0);
    } else {  // EPI_ACC: out_e[row, col] += acc  ((E, Mout, N), fp32 or, with acc_bf16, bf16)
      const int64_t oo = (static_cast<int64_t>(t.e) * p.Mout + row) * p.N + col;
      if (p.acc_bf16) {  // the product summed in fp32, rounded once as it is added
        acc_add_bf16(static_cast<bf16*>(p.out0) + oo, v0, alpha);
      } else {
        float* d0p = static_cast<float*>(p.out0) + oo;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 x = *reinterpret_cast<float4*>(d0p + i);
          x.x += alpha * v0[i]; x.y += alpha * v0[i + 1]; x.z += alpha * v0[i + 2]; x.w += alpha * v0[i + 3];
          *reinterpret_cast<float4*>(d0p + i) = x;
        }
      }
      if constexpr (NB == 2) {
        float v1[32];
        tmem_ld32(tb + BNA + c * 32, v1);
        if (p.acc_bf16) {
          acc_add_bf16(static_cast<bf16*>(p.out1) + oo, v1, alpha);
        } else {
          float* d1p = static_cast<float*>(p.out1) + oo;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 x = *reinterpret_cast<float4*>(d1p + i);
            x.x += alpha * v1[i]; x.y += alpha * v1[i + 1]; x.z += alpha * v1[i + 2]; x.w += alpha * v1[i + 3];
            *reinterpret_cast<float4*>(d1p + i) = x;
          }
        }
      }
    }
  }
}

template <bool KGROUP, bool A_MN, bool B_MN, int NB, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) moe_gemm_kernel(const __grid_constant__ Params p) {
  constexpr int BNA = 256 / NB;  // columns per accumulator
  constexpr int NST = n_stages<EPI>();
  constexpr uint32_t IDESC = idesc_bf16(BM, BNA, A_MN, B_MN);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * STAGE_BYTES);
  uint64_t* empty = full + NST;
  uint64_t* tfull = empty + NST;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* off = const_cast<int*>(reinterpret_cast<const int*>(tmem_slot + 2));  // E+1 ints (E <= 192)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i <= p.E; i += NTHREADS) off[i] = p.grp_off[i];
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = (p.N + BNA - 1) / BNA;
  const int total = KGROUP ? p.E * (p.Mout / BM) * n_tiles : (off[p.E] / BM) * n_tiles;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    prefetch_tmap(&p.ta0);
    prefetch_tmap(&p.tb0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      Tile t;
      decode<KGROUP>(p, off, tile, n_tiles, t);
      const int n0 = t.n0 * BNA;
      for (int kb = 0; kb < t.nkb; ++kb) {
        if (!mbar_wait(empty + stage, phase ^ 1, abort_flag, p.err, 1)) { ok = false; break; }
        unsigned char* sa = smem + stage * STAGE_BYTES;
        unsigned char* sb = sa + A_BYTES;
        mbar_expect_tx(full + stage, STAGE_BYTES);
        const int part = (!KGROUP && kb >= p.kb_split) ? 1 : 0;
        const int kk = (part ? kb - p.kb_split : kb) * BK;
        const CUtensorMap* ma = part ? &p.ta1 : &p.ta0;
        if (!KGROUP) {
          if (A_MN) {
            tma_load_2d(sa, ma, full + stage, t.m0, kk);
            tma_load_2d(sa + 8192, ma, full + stage, t.m0 + 64, kk);
          } else {
            tma_load_2d(sa, ma, full + stage, kk, t.m0);
          }
        } else {
          const int r = t.k0row + kb * BK;
          tma_load_2d(sa, ma, full + stage, t.m0, r);
          tma_load_2d(sa + 8192, ma, full + stage, t.m0 + 64, r);
        }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const CUtensorMap* mb = (NB == 2) ? (nb ? &p.tb1 : &p.tb0) : (part ? &p.tb1 : &p.tb0);
          unsigned char* sbn = sb + nb * BNA * BK * 2;
          if (!KGROUP) {
            if (B_MN) {
#pragma unroll
              for (int i = 0; i < BNA / 64; ++i) tma_load_2d(sbn + i * 8192, mb, full + stage, n0 + 64 * i, t.e * p.b_rows + kk);
            } else {
              tma_load_2d(sbn, mb, full + stage, kk, t.e * p.b_rows + n0);
            }
          } else {
            const int r = t.k0row + kb * BK;
#pragma unroll
            for (int i = 0; i < BNA / 64; ++i) tma_load_2d(sbn + i * 8192, mb, full + stage, n0 + 64 * i, r);
          }
        }
        if (++stage == NST) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) {  // let copies already in flight land before the CTA exits
      const uint64_t t0 = globaltimer();
      while (globaltimer() - t0 < 2000000ull) {}
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    bool issued = false;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      Tile t;
      decode<KGROUP>(p, off, tile, n_tiles, t);
      if (t.nkb == 0) continue;
      if (!mbar_wait(tempty + acc, acc_phase ^ 1, abort_flag, p.err, 2)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d0 = tmem_base + acc * 256;
      for (int kb = 0; kb < t.nkb; ++kb) {
        if (!mbar_wait(full + stage, phase, abort_flag, p.err, 3)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
        const uint32_t sb = sa + A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = A_MN ? smem_desc(sa + k * 2048, 8192, 1024) : smem_desc(sa + k * 32, 16, 1024);
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint32_t sbn = sb + nb * BNA * BK * 2;
            const uint64_t bd = B_MN ? smem_desc(sbn + k * 2048, 8192, 1024) : smem_desc(sbn + k * 32, 16, 1024);
            umma_bf16(d0 + nb * BNA, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
        }
        issued = true;
        umma_commit(empty + stage);
        if (++stage == NST) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      umma_commit(tfull + acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (!ok && issued) {  // wait (bounded) for the MMAs already issued before freeing TMEM
      umma_commit(drain);
      volatile int dummy = 0;
      mbar_wait(drain, 0, &dummy, nullptr, 0, 100000000ull);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      Tile t;
      decode<KGROUP>(p, off, tile, n_tiles, t);
      if (t.nkb == 0) continue;
      if (!mbar_wait(tfull + acc, acc_phase, abort_flag, p.err, 4)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 256;
      epilogue_tile<EPI, NB>(p, off, t, tb, t.m0 + q * 32, lane, smem + NST * STAGE_BYTES + 1024, q);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // peer stores must be visible system-wide before the barrier that follows the kernel
    if constexpr (EPI == EPI_STORE_PEER) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ---------------------------------------------------------------- CTA-pair kernel
// The same GEMMs with one tcgen05.mma spanning the two CTAs of a cluster (cta_group::2): a pair
// computes a 256 x 256 tile (NB = 2: two 256 x 128 accumulators), each CTA loading its 128 rows
// of A and its half of the B columns, so a CTA streams 32 KB of operands per 64-deep k-block
// instead of 48 KB for a 128 x 256 tile.  Six 32 KB stages.  Only the leader CTA (rank 0) runs
// the MMA role; both CTAs' TMA loads complete on the leader's `full` barrier; its commits
// arrive on `empty` / `tfull` of both CTAs; both CTAs' epilogue warps release an accumulator on
// the leader's `tempty`.  M-grouped groups (and K-grouped Mout) must be multiples of 256 rows.
// Seven 32 KB stages (224 KB of the 227 KB a CTA may take).  A weight gradient of 2048 x 2048 has
// 64 tiles for 74 pairs (any power-of-two tile count leaves the last wave short of 74 or 148); the
// pairs walk the token dimension in lockstep, so the rows they read stay in L2 (an even split of
// the (tile, k-block) iterations over the pairs spreads them over all of x and dy and re-read
// them from DRAM five times: measured, no faster).
constexpr int PAIR_BM = 256, PAIR_STAGES = 7;
constexpr int PAIR_A_BYTES = 128 * BK * 2;  // 16 KB: this CTA's 128 rows
constexpr int PAIR_B_BYTES = 128 * BK * 2;  // 16 KB: this CTA's half of the 256 columns
constexpr int PAIR_STAGE_BYTES = PAIR_A_BYTES + PAIR_B_BYTES;
constexpr size_t PAIR_SMEM = (size_t)PAIR_STAGES * PAIR_STAGE_BYTES + 1024 + 1024;

template <bool KGROUP>
AHB_DEVICE void decode_pair(const Params& p, const int* off, int tile, int n_tiles, Tile& t) {
  if (!KGROUP) {
    const int m_total = off[p.E] / PAIR_BM;
    const int mt = p.m_fast ? tile % m_total : tile / n_tiles, nt = p.m_fast ? tile / m_total : tile % n_tiles;
    t.m0 = mt * PAIR_BM;
    int e = 0;
    while (e + 1 < p.E && off[e + 1] <= t.m0) ++e;
    t.e = e;
    t.n0 = nt;
    t.k0row = 0;
    t.nkb = p.kb_total;
  } else {
    const int m_tiles = p.Mout / PAIR_BM;
    const int per_e = m_tiles * n_tiles;
    t.e = tile / per_e;
    const int r = tile % per_e;
    t.m0 = (r / n_tiles) * PAIR_BM;
    t.n0 = r % n_tiles;
    t.k0row = off[t.e];
    t.nkb = (off[t.e + 1] - off[t.e]) / BK;
  }
}

// One unit of work of a pair: a tile and its k-blocks [kb0, kb1).  Every role of both CTAs walks
// the same sequence: tiles cid, cid + ncl, ...
struct PairWork {
  Tile t;
  int kb0, kb1;
};

template <bool KGROUP>
struct PairSched {
  const Params& p;
  const int* off;
  int n_tiles, total, ncl;
  int tile;
  AHB_DEVICE PairSched(const Params& p_, const int* off_, int n_tiles_, int total_, int cid, int ncl_)
      : p(p_), off(off_), n_tiles(n_tiles_), total(total_), ncl(ncl_), tile(cid) {}
  AHB_DEVICE bool next(PairWork& w) {
    if (tile >= total) return false;
    decode_pair<KGROUP>(p, off, tile, n_tiles, w.t);
    w.kb0 = 0;
    w.kb1 = w.t.nkb;
    tile += ncl;
    return true;
  }
};

template <bool KGROUP, bool A_MN, bool B_MN, int NB, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1) moe_gemm_pair_kernel(const __grid_constant__ Params p) {
  constexpr int BNA = 256 / NB;       // columns per accumulator (the pair's N of one MMA)
  constexpr int HALF = BNA / 2;       // B columns of one MMA held by this CTA
  constexpr uint32_t IDESC = idesc_bf16(PAIR_BM, BNA, A_MN, B_MN);
  static_assert(EPI != EPI_STORE_PEER, "peer-store epilogue runs on the single-CTA kernel");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PAIR_STAGES * PAIR_STAGE_BYTES);
  uint64_t* empty = full + PAIR_STAGES;
  uint64_t* tfull = empty + PAIR_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* off = const_cast<int*>(reinterpret_cast<const int*>(tmem_slot + 2));  // E+1 ints (E <= 192)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 8);  // 4 epilogue warps in each CTA of the pair
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i <= p.E; i += NTHREADS) off[i] = p.grp_off[i];
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive or load completes
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = (p.N + BNA - 1) / BNA;
  const int total = KGROUP ? p.E * (p.Mout / PAIR_BM) * n_tiles : (off[p.E] / PAIR_BM) * n_tiles;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    prefetch_tmap(&p.ta0);
    prefetch_tmap(&p.tb0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    PairSched<KGROUP> sched(p, off, n_tiles, total, cid, ncl);
    PairWork wk;
    while (ok && sched.next(wk)) {
      const Tile& t = wk.t;
      const int n0 = t.n0 * BNA;
      const int mrow = t.m0 + 128 * (int)rank;
      for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
        if (!mbar_wait(empty + stage, phase ^ 1, abort_flag, p.err, 11)) { ok = false; break; }
        unsigned char* sa = smem + stage * PAIR_STAGE_BYTES;
        unsigned char* sb = sa + PAIR_A_BYTES;
        const uint32_t fb = mapa_shared(full + stage, 0);
        if (rank == 0) mbar_expect_tx(full + stage, 2 * PAIR_STAGE_BYTES);
        const int part = (!KGROUP && kb >= p.kb_split) ? 1 : 0;
        const int kk = (part ? kb - p.kb_split : kb) * BK;
        const CUtensorMap* ma = part ? &p.ta1 : &p.ta0;
        if (!KGROUP) {
          if (A_MN) {
            tma_load_2d_pair(sa, ma, fb, mrow, kk);
            tma_load_2d_pair(sa + 8192, ma, fb, mrow + 64, kk);
          } else {
            tma_load_2d_pair(sa, ma, fb, kk, mrow);
          }
        } else {
          const int r = t.k0row + kb * BK;
          tma_load_2d_pair(sa, ma, fb, mrow, r);
          tma_load_2d_pair(sa + 8192, ma, fb, mrow + 64, r);
        }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const CUtensorMap* mb = (NB == 2) ? (nb ? &p.tb1 : &p.tb0) : (part ? &p.tb1 : &p.tb0);
          unsigned char* sbn = sb + nb * HALF * BK * 2;
          const int c0 = n0 + HALF * (int)rank;
          if (!KGROUP) {
            if (B_MN) {
#pragma unroll
              for (int i = 0; i < HALF / 64; ++i) tma_load_2d_pair(sbn + i * 8192, mb, fb, c0 + 64 * i, t.e * p.b_rows + kk);
            } else {
              tma_load_2d_pair(sbn, mb, fb, kk, t.e * p.b_rows + c0);
            }
          } else {
            const int r = t.k0row + kb * BK;
#pragma unroll
            for (int i = 0; i < HALF / 64; ++i) tma_load_2d_pair(sbn + i * 8192, mb, fb, c0 + 64 * i, r);
          }
        }
        if (++stage == PAIR_STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) {  // let copies already in flight land before the CTA exits
      const uint64_t t0 = globaltimer();
      while (globaltimer() - t0 < 2000000ull) {}
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    bool issued = false;
    PairSched<KGROUP> sched(p, off, n_tiles, total, cid, ncl);
    PairWork wk;
    while (ok && sched.next(wk)) {
      if (wk.kb1 <= wk.kb0) continue;
      if (!mbar_wait(tempty + acc, acc_phase ^ 1, abort_flag, p.err, 12)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d0 = tmem_base + acc * 256;
      for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
        if (!mbar_wait(full + stage, phase, abort_flag, p.err, 13)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * PAIR_STAGE_BYTES);
        const uint32_t sb = sa + PAIR_A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = A_MN ? smem_desc(sa + k * 2048, 8192, 1024) : smem_desc(sa + k * 32, 16, 1024);
#pragma unroll
          for (int nb = 0; nb < NB; ++nb) {
            const uint32_t sbn = sb + nb * HALF * BK * 2;
            const uint64_t bd = B_MN ? smem_desc(sbn + k * 2048, 8192, 1024) : smem_desc(sbn + k * 32, 16, 1024);
            umma_bf16_pair(d0 + nb * BNA, ad, bd, IDESC, (kb > wk.kb0 || k != 0) ? 1u : 0u);
          }
        }
        issued = true;
        umma_commit_pair(empty + stage, 0x3);
        if (++stage == PAIR_STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      umma_commit_pair(tfull + acc, 0x3);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (!ok && issued) {  // wait (bounded) for the MMAs already issued before freeing TMEM
      umma_commit_pair(drain, 0x1);
      volatile int dummy = 0;
      mbar_wait(drain, 0, &dummy, nullptr, 0, 100000000ull);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const uint32_t tempty0 = mapa_shared(tempty, 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    PairSched<KGROUP> sched(p, off, n_tiles, total, cid, ncl);
    PairWork wk;
    while (sched.next(wk)) {
      if (wk.kb1 <= wk.kb0) continue;
      if (!mbar_wait(tfull + acc, acc_phase, abort_flag, p.err, 14)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 256;
      epilogue_tile<EPI, NB>(p, off, wk.t, tb, wk.t.m0 + 128 * (int)rank + q * 32, lane, nullptr, q);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into this CTA's TMEM and shared memory are done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map: `rows` x `cols` row-major with row stride `ld` elements; box = {64, box_rows}.
int make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !ptr) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <bool KG, bool AMN, bool BMN, int NB, int EPI>
int launch(const Params& p, int grid, cudaStream_t st) {
  auto k = moe_gemm_kernel<KG, AMN, BMN, NB, EPI>;
  constexpr size_t SMEM = smem_bytes<EPI>();
  static bool init = false;
  if (!init) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM) != cudaSuccess) return -3;
    init = true;
  }
  k<<<grid, NTHREADS, SMEM, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <bool KG, bool AMN, bool BMN, int NB, int EPI>
int launch_pair(const Params& p, int grid, cudaStream_t st) {
  auto k = moe_gemm_pair_kernel<KG, AMN, BMN, NB, EPI>;
  static bool init = false;
  if (!init) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PAIR_SMEM) != cudaSuccess) return -3;
    init = true;
  }
  k<<<grid, NTHREADS, PAIR_SMEM, st>>>(p);  // cluster dims (2, 1, 1) are part of the kernel
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace

// kind: see launchers.h (AHB_GEMM_*)
int ahb_moe_gemm(int kind, const void* a0, const void* a1, int64_t a_rows, int64_t a_cols, const void* b0,
                 const void* b1, int64_t b_rows_total, int64_t b_cols, int b_rows_per_group, const int* grp_off,
                 int E, int N, int Mout, int K, int kb_split, void* out0, void* out1, void* out2, const void* aux0,
                 const void* aux1, float clip, int* err, int num_sms, cudaStream_t st, const float* alpha,
                 int m_limit) {
  const bool pair = (kind & AHB_GEMM_PAIR) != 0;
  const bool acc16 = (kind & AHB_GEMM_ACC_BF16) != 0;
  kind &= ~(AHB_GEMM_PAIR | AHB_GEMM_ACC_BF16);
  if (E < 1 || E > 192 || N % 32 != 0 || K % 64 != 0) return -10;  // offsets live in the kernel's smem tail
  Params p;
  memset(&p, 0, sizeof(p));
  p.grp_off = grp_off;
  p.E = E;
  p.N = N;
  p.Mout = Mout;
  p.kb_split = kb_split;
  p.kb_total = K / BK;
  p.b_rows = b_rows_per_group;
  p.out0 = out0;
  p.out1 = out1;
  p.out2 = out2;
  p.aux0 = static_cast<const bf16*>(aux0);
  p.aux1 = static_cast<const bf16*>(aux1);
  p.clip = clip;
  p.alpha = alpha;
  p.err = err;
  p.m_limit = m_limit;
  p.acc_bf16 = acc16 ? 1 : 0;
  const bool kg = kind == AHB_GEMM_WGRAD || kind == AHB_GEMM_WGRAD_DUAL;
  const bool a_mn = kg;
  const bool b_mn = kg || kind == AHB_GEMM_FWD_SWIGLU || kind == AHB_GEMM_FWD_GELU || kind == AHB_GEMM_FWD_DOWN;
  const int nb = (kind == AHB_GEMM_FWD_SWIGLU || kind == AHB_GEMM_WGRAD_DUAL) ? 2 : 1;
  const int bna = 256 / nb;
  // a partial last column tile is fine where the epilogue stops at N (store, fp32 accumulate)
  if (N % bna != 0 && kind != AHB_GEMM_DENSE && kind != AHB_GEMM_FWD_DOWN && kind != AHB_GEMM_DX &&
      kind != AHB_GEMM_WGRAD)
    return -11;
  if (kg && Mout % (pair ? PAIR_BM : BM) != 0) return -12;
  // a CTA of a pair loads half of each accumulator's columns of B
  const int b_box = b_mn ? 64 : (pair ? bna / 2 : bna);
  int rc = 0;
  rc |= make_map(&p.ta0, a0, a_rows, a_cols, a_cols, a_mn ? 64 : BM);
  if (a1) rc |= make_map(&p.ta1, a1, a_rows, a_cols, a_cols, a_mn ? 64 : BM);
  rc |= make_map(&p.tb0, b0, b_rows_total, b_cols, b_cols, b_box);
  if (b1) rc |= make_map(&p.tb1, b1, b_rows_total, b_cols, b_cols, b_box);
  if (!a1) p.ta1 = p.ta0;
  if (!b1) p.tb1 = p.tb0;
  if (rc) return -20;
  if (pair) {
    const int grid = (num_sms / 2) * 2;
    switch (kind) {
      case AHB_GEMM_DENSE: return launch_pair<false, false, false, 1, EPI_STORE>(p, grid, st);
      case AHB_GEMM_FWD_SWIGLU: return launch_pair<false, false, true, 2, EPI_SWIGLU_FWD>(p, grid, st);
      case AHB_GEMM_FWD_GELU: return launch_pair<false, false, true, 1, EPI_GELU_FWD>(p, grid, st);
      case AHB_GEMM_FWD_DOWN: return launch_pair<false, false, true, 1, EPI_STORE>(p, grid, st);
      case AHB_GEMM_DH_SWIGLU: return launch_pair<false, false, false, 1, EPI_SWIGLU_BWD>(p, grid, st);
      case AHB_GEMM_DH_GELU: return launch_pair<false, false, false, 1, EPI_GELU_BWD>(p, grid, st);
      case AHB_GEMM_DX: return launch_pair<false, false, false, 1, EPI_STORE>(p, grid, st);
      case AHB_GEMM_WGRAD: return launch_pair<true, true, true, 1, EPI_ACC>(p, grid, st);
      case AHB_GEMM_WGRAD_DUAL: return launch_pair<true, true, true, 2, EPI_ACC>(p, grid, st);
      default: return -30;
    }
  }
  const int grid = num_sms;
  switch (kind) {
    case AHB_GEMM_DENSE: return launch<false, false, false, 1, EPI_STORE>(p, grid, st);
    case AHB_GEMM_FWD_SWIGLU: return launch<false, false, true, 2, EPI_SWIGLU_FWD>(p, grid, st);
    case AHB_GEMM_FWD_GELU: return launch<false, false, true, 1, EPI_GELU_FWD>(p, grid, st);
    case AHB_GEMM_FWD_DOWN: return launch<false, false, true, 1, EPI_STORE>(p, grid, st);
    case AHB_GEMM_DH_SWIGLU: return launch<false, false, false, 1, EPI_SWIGLU_BWD>(p, grid, st);
    case AHB_GEMM_DH_GELU: return launch<false, false, false, 1, EPI_GELU_BWD>(p, grid, st);
    case AHB_GEMM_DX: return launch<false, false, false, 1, EPI_STORE>(p, grid, st);
    case AHB_GEMM_WGRAD: return launch<true, true, true, 1, EPI_ACC>(p, grid, st);
    case AHB_GEMM_WGRAD_DUAL: return launch<true, true, true, 2, EPI_ACC>(p, grid, st);
    default: return -30;
  }
}

// Dense projection pieces on the grouped GEMM (one group; rows padded to the tile height, rows
// at or beyond M read as zeros and not stored):
// (lda / ldb: row strides in elements, multiples of 8: A and B may be column slices of wider rows)
//   mode 0  y = x W (+ bias) (+ beta_src)    x (M,K) K-major, W (K,N) MN-major
//   mode 1  y = dy W^T (+ beta_src)          dy (M,K) K-major, W (N,K) K-major (W^T of an (N,K) kernel)
//   mode 2  acc (K,N) fp32 += x^T dy          x (M,K), dy (M,N), contraction over the M rows
int ahb_dense_gemm(int mode, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int K, int N,
                   const void* bias, const void* beta_src, void* out, const int* grp_off, int* err, int num_sms,
                   cudaStream_t st, bool pair) {
  if (K % BK != 0 || N % 32 != 0 || M <= 0 || lda % 8 != 0 || ldb % 8 != 0) return -10;
  Params p;
  memset(&p, 0, sizeof(p));
  p.grp_off = grp_off;
  p.E = 1;
  p.N = N;
  p.err = err;
  p.out0 = out;
  p.bias = static_cast<const bf16*>(bias);
  p.beta_src = static_cast<const bf16*>(beta_src);
  int rc = 0;
  if (mode == 2) {  // K-grouped: Mout = K rows of the weight, contraction over the M token rows
    if (K % (pair ? PAIR_BM : BM) != 0) return -12;
    p.Mout = K;
    rc |= make_map(&p.ta0, a, M, K, lda, 64);
    rc |= make_map(&p.tb0, b, M, N, ldb, 64);
  } else {
    p.kb_split = K / BK;
    p.kb_total = K / BK;
    p.m_limit = (int)M;
    rc |= make_map(&p.ta0, a, M, K, lda, BM);
    if (mode == 0) rc |= make_map(&p.tb0, b, K, N, ldb, 64);      // W (K rows, N cols), MN-major
    else rc |= make_map(&p.tb0, b, N, K, ldb, pair ? 128 : 256);   // W (N rows, K cols), K-major
    p.b_rows = mode == 0 ? K : N;
  }
  if (rc) return -20;
  p.ta1 = p.ta0;
  p.tb1 = p.tb0;
  const int g2 = (num_sms / 2) * 2;
  if (pair) {
    switch (mode) {
      case 0: return launch_pair<false, false, true, 1, EPI_STORE>(p, g2, st);
      case 1: return launch_pair<false, false, false, 1, EPI_STORE>(p, g2, st);
      default: return launch_pair<true, true, true, 1, EPI_ACC>(p, g2, st);
    }
  }
  switch (mode) {
    case 0: return launch<false, false, true, 1, EPI_STORE>(p, num_sms, st);
    case 1: return launch<false, false, false, 1, EPI_STORE>(p, num_sms, st);
    default: return launch<true, true, true, 1, EPI_ACC>(p, num_sms, st);
  }
}

// LM-head GEMM logits = h W^T (h: rows x d, W: V x d, both K-major) with a cross-entropy epilogue that
// never stores the logits: `bwd` false writes per-(row, 256-column tile) partials (max, sum-exp,
// label logit, logit sum) as float4 [rows][ce_tiles]; `bwd` true writes bf16 dlogits [rows_pad][V]
// (zeros on masked rows and rows at or beyond `rows`).  Rows are padded to the tile height (256
// with `pair`): h rows beyond `rows` read as zeros.
int ahb_ce_gemm(bool bwd, const void* h, int64_t rows, int d, const void* W, int V, const int* grp_off,
                const int64_t* labels, const float* lse, float ls, void* out, int* err, int num_sms, cudaStream_t st,
                bool pair) {
  if (d % BK != 0 || V % 32 != 0 || rows <= 0) return -10;
  Params p;
  memset(&p, 0, sizeof(p));
  p.grp_off = grp_off;
  p.E = 1;
  p.N = V;
  p.kb_split = d / BK;
  p.kb_total = d / BK;
  p.b_rows = 0;
  p.out0 = out;
  p.err = err;
  p.m_limit = (int)rows;
  p.labels = labels;
  p.row_lse = lse;
  p.ce_sp = 1.f - ls;
  p.ce_sn = ls > 0.f ? ls / (float)(V - 1) : 0.f;
  p.ce_tiles = (V + 255) / 256;
  p.m_fast = 1;
  int rc = make_map(&p.ta0, h, rows, d, d, BM);
  rc |= make_map(&p.tb0, W, V, d, d, pair ? 128 : 256);
  if (rc) return -20;
  p.ta1 = p.ta0;
  p.tb1 = p.tb0;
  if (pair) {
    const int grid = (num_sms / 2) * 2;
    return bwd ? launch_pair<false, false, false, 1, EPI_CE_BWD>(p, grid, st)
               : launch_pair<false, false, false, 1, EPI_CE_FWD>(p, grid, st);
  }
  return bwd ? launch<false, false, false, 1, EPI_CE_BWD>(p, num_sms, st)
             : launch<false, false, false, 1, EPI_CE_FWD>(p, num_sms, st);
}

// GEMM -> reduce-scatter over peer memory: out rows of group g (rows [grp_off[g], grp_off[g+1]) of A)
// are the partial sums owed to rank g and are stored at out_tab[g] (its receive slot for this rank).
int ahb_gemm_rs_peer(const void* a, int64_t a_rows, int64_t K, const void* b, int64_t N, const int* grp_off, int W,
                     void* const* out_tab, int m_rot, int* err, int num_sms, cudaStream_t st) {
  if (W < 1 || W > MAX_PEERS || a_rows % BM != 0 || K % BK != 0 || N % 32 != 0) return -10;
  Params p;
  memset(&p, 0, sizeof(p));
  p.grp_off = grp_off;
  p.E = W;
  p.N = (int)N;
  p.Mout = 0;
  p.kb_split = (int)(K / BK);
  p.kb_total = (int)(K / BK);
  p.b_rows = 0;  // every group multiplies by the same weight
  p.err = err;
  for (int g = 0; g < W; ++g) p.out_tab[g] = out_tab[g];
  p.m_rot = m_rot;
  int rc = make_map(&p.ta0, a, a_rows, K, K, BM);
  rc |= make_map(&p.tb0, b, K, N, N, 64);
  p.ta1 = p.ta0;
  p.tb1 = p.tb0;
  if (rc) return -20;
  return launch<false, false, true, 1, EPI_STORE_PEER>(p, num_sms, st);
}
