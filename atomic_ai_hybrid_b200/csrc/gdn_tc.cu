// GDN-2 chunk kernels on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// Math (per (batch, head), chunks of C = 64 tokens, head dim D = 128, per-channel decay;
// reference `atomic_ops/gdn2_wy_reference.py:33-152`, kernels A-D `atomic_ops/kernel_{a,b,c,d}_*.py`):
//   gc = cumsum_t g ; gcl = gc[C-1]
//   Aqk[i,j] = scale sum_d q_id k_jd e^{gc_id - gc_jd} (i >= j) ; Akk[i,j] = sum_d (bk)_id k_jd e^{...} (i > j)
//   A = (I + Akk)^-1 ; w~ = A (bk e^gc) ; u = A (w v)
//   v_new = u - w~ h ; o = scale (q e^gc) h + Aqk v_new ; h' = e^{gcl} h + (k e^{gcl-gc})^T v_new
//
// gdn_chunk_fwd_tc (one CTA per chunk, 128 threads, two CTAs per SM):
//   * scores: the pairwise decay e^{gc_i - gc_j} is split at a reference row r = 16 I, the
//     first row of query block I (every row i of block I has i >= r): rows carry
//     e^{gc_i - gc_r} <= 1, keys j <= 16 I + 15 carry e^{gc_r - gc_j} (<= 1 below the block,
//     <= e^{span} inside it).  One M = 128 MMA per reference block I multiplies the stacked
//     [q-rows ; bk-rows] operand by that block's key operand into its own TMEM region; row i
//     reads the region of its own block.  A diagonal block whose 16-row decay span exceeds 60
//     is summed exactly per channel instead (the reference's -20 floor on the exponent).
//   * (I + Akk)^-1 in fp32 on the CUDA cores: 16 x 16 diagonal inverses by substitution,
//     then the off-diagonal blocks by distance (reference kernel B's blocked solve).
//   * w~ and u: two M = 64 MMAs, A as the K-major operand, (bk e^gc) and (w v) as MN-major.
// Intermediates for the state kernels are written as 128-byte-swizzled tile images (the exact
// shared-memory layout the tensor core reads), so the consumers fetch them with one bulk copy.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstring>
#include "common.cuh"
#include "sm100.cuh"
#include "umma.cuh"
#include "launchers.h"
#include "tmap.h"

using namespace ahb;
using namespace ahb::umma;
using bf16 = __nv_bfloat16;

namespace {

constexpr int C = 64, D = 128;
constexpr int TILE_CD = C * D * 2;  // bytes of a swizzled 64 x 128 bf16 tile image
constexpr int TILE_CC = C * C * 2;  // 64 x 64

AHB_DEVICE float guard(float x) {  // nan_to_num(nan=0, +-inf -> +-1e4), clip 1e4
  if (x != x) return 0.f;
  return fminf(fmaxf(x, -1e4f), 1e4f);
}

struct SeqIdx {
  int64_t L, H;
  AHB_DEVICE int64_t row(int b, int64_t t, int h) const { return ((b * L + t) * H + h) * D; }
};

// ============================================================ chunk-parallel forward
// shared memory: R1 (32 KB) stacked score rows, later A fp32, later (bk e^gc | w v) tiles;
//                R2 (32 KB) key operands (two buffers), later Akk fp32 and the A tile; GC (32 KB)
constexpr int F1_THREADS = 128;
constexpr int F1_LDA = C + 1;  // fp32 row stride of the 64 x 64 work matrices
constexpr size_t F1_SMEM = 1024 + 3 * 32768 + 256;

__global__ void __launch_bounds__(F1_THREADS, 2) gdn_chunk_fwd_tc(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
    const float* __restrict__ g, const bf16* __restrict__ bg, const bf16* __restrict__ wg, float scale, int L,
    int H, unsigned char* __restrict__ wt_t, unsigned char* __restrict__ u_t, unsigned char* __restrict__ qg_t,
    unsigned char* __restrict__ kg_t, unsigned char* __restrict__ aqk_t, float* __restrict__ gcl_o,
    float* __restrict__ a_o, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* R1 = smem;
  unsigned char* R2 = smem + 32768;
  float* GC = reinterpret_cast<float*>(smem + 65536);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 98304);  // [0..3] score blocks, [4] w~/u
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0..3] exact diagonal block, [4] abort
  float* span_w = reinterpret_cast<float*>(flags + 8);  // [4 warps][4 blocks]

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SeqIdx ix{L, H};
  const int64_t t0 = (int64_t)n * C;
  const int64_t cb = ((int64_t)b * H + h) * NC + n;
  const uint32_t sR1 = smem_u32(R1), sR2 = smem_u32(R2);

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) sm100::mbar_init(bars + i, 1);
    flags[4] = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 256);

  // 1. g -> GC, cumulative sum per channel (thread d owns channel d)
  for (int e = tid; e < C * (D / 4); e += F1_THREADS) {
    const int r = e >> 5, c4 = (e & 31) << 2;
    *reinterpret_cast<float4*>(GC + r * D + c4) = *reinterpret_cast<const float4*>(g + ix.row(b, t0 + r, h) + c4);
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  {
    const int d = tid;
    float s = 0.f;
    for (int r = 0; r < C; ++r) {
      s += GC[r * D + d];
      GC[r * D + d] = s;
    }
    gcl_o[cb * D + d] = s;
    float sp[4];
#pragma unroll
    for (int I = 0; I < 4; ++I) sp[I] = warp_max(GC[16 * I * D + d] - GC[(16 * I + 15) * D + d]);
    if (lane == 0)
#pragma unroll
      for (int I = 0; I < 4; ++I) span_w[warp * 4 + I] = sp[I];
  }
  __syncthreads();
  if (tid < 4) {
    float m = fmaxf(fmaxf(span_w[tid], span_w[4 + tid]), fmaxf(span_w[8 + tid], span_w[12 + tid]));
    flags[tid] = !(m <= 60.f);  // NaN spans take the exact path too
  }
  __syncthreads();

  // 2. stacked score rows: R1 rows 0-63 = q e^{gc - gc_r}, rows 64-127 = (b k) e^{gc - gc_r};
  //    qg = q e^gc and kg = k e^{gcl - gc} go straight out as tile images
  unsigned char* qg_c = qg_t + cb * TILE_CD;
  unsigned char* kg_c = kg_t + cb * TILE_CD;
  for (int it = 0; it < (C * D / 8) / F1_THREADS; ++it) {
    const int u_ = it * F1_THREADS + tid;
    const int i = u_ >> 4, c = (u_ & 15) << 3;
    const int64_t gi = ix.row(b, t0 + i, h) + c;
    float qv[8], kv[8], bv[8];
    unpack8(*reinterpret_cast<const uint4*>(q + gi), qv);
    unpack8(*reinterpret_cast<const uint4*>(k + gi), kv);
    unpack8(*reinterpret_cast<const uint4*>(bg + gi), bv);
    const float* gci = GC + i * D + c;
    const float* gcr = GC + (i & ~15) * D + c;
    const float* gcl = GC + (C - 1) * D + c;
    float a[8], bk[8], qg[8], kg[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float er = __expf(gci[e] - gcr[e]);
      a[e] = qv[e] * er;
      bk[e] = bv[e] * kv[e] * er;
      qg[e] = qv[e] * __expf(gci[e]);
      kg[e] = kv[e] * __expf(gcl[e] - gci[e]);
    }
    st_chunk8(sR1 + sw_off16(128, i, c), a);
    st_chunk8(sR1 + sw_off16(128, C + i, c), bk);
    *reinterpret_cast<uint4*>(qg_c + sw_off16(C, i, c)) = pack8(qg);
    *reinterpret_cast<uint4*>(kg_c + sw_off16(C, i, c)) = pack8(kg);
  }

  // 3. key operands per reference block and the score MMAs (region I = TMEM columns [64 I, 64 I + 64))
  constexpr uint32_t IDESC_S[4] = {sm100::idesc_bf16(128, 16, false, false), sm100::idesc_bf16(128, 32, false, false),
                                   sm100::idesc_bf16(128, 48, false, false), sm100::idesc_bf16(128, 64, false, false)};
  for (int I = 0; I < 4; ++I) {
    unsigned char* buf = R2 + (I & 1) * TILE_CD;
    if (I >= 2 && !wait_bar(bars + I - 2, 0, err, 0x4701)) flags[4] = 1;
    const int rows = 16 * (I + 1);
    const bool exact = flags[I];
    const float* gcr = GC + 16 * I * D;
    for (int u_ = tid; u_ < rows * 16; u_ += F1_THREADS) {
      const int j = u_ >> 4, c = (u_ & 15) << 3;
      float kv[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(k + ix.row(b, t0 + j, h) + c), kv);
      const float* gcj = GC + j * D + c;
      const bool zero = exact && j >= 16 * I;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = zero ? 0.f : kv[e] * __expf(gcr[c + e] - gcj[e]);
      st_chunk8(smem_u32(buf) + sw_off16(C, j, c), o);
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      sm100::tc_fence_after();
      const uint32_t sb = smem_u32(buf);
      mma_steps(tmem + 64 * I, [&](int s) { return kdesc(sR1, 128, s); }, [&](int s) { return kdesc(sb, C, s); },
                D / 16, IDESC_S[I], false);
      sm100::umma_commit(bars + I);
    }
  }
  if (!wait_bar(bars + 2, 0, err, 0x4702) || !wait_bar(bars + 3, 0, err, 0x4703)) flags[4] = 1;
  sm100::tc_fence_after();

  // 4. scores out of TMEM: lane m of quarter q is row m = 32 q + lane of the stack
  float* AKK = reinterpret_cast<float*>(R2);  // fp32 [64][65]
  {
    const int m = 32 * warp + lane;
    const bool is_q = m < C;
    const int i = is_q ? m : m - C;
    const int I = i >> 4;
    const int Ilo = 2 * (warp & 1), Ihi = Ilo + 1;
    float row[64];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float t[16];
      if (p <= Ilo) {
        tmem_ld16(tmem_at(tmem, warp, 64 * Ilo + 16 * p), t);
        if (I == Ilo)
#pragma unroll
          for (int e = 0; e < 16; ++e) row[16 * p + e] = t[e];
      }
      if (p <= Ihi) {
        tmem_ld16(tmem_at(tmem, warp, 64 * Ihi + 16 * p), t);
        if (I == Ihi)
#pragma unroll
          for (int e = 0; e < 16; ++e) row[16 * p + e] = t[e];
      }
    }
    // exact per-channel sums on a diagonal block with a wide decay span
    if (flags[I]) {
      const bf16* xi = (is_q ? q : bg) + ix.row(b, t0 + i, h);
      const bf16* ki = k + ix.row(b, t0 + i, h);
      for (int j = 16 * I; j <= i; ++j) {
        const bf16* kj = k + ix.row(b, t0 + j, h);
        float s = 0.f;
        for (int d = 0; d < D; ++d) {
          float x = __bfloat162float(xi[d]);
          if (!is_q) x *= __bfloat162float(ki[d]);
          s += x * __bfloat162float(kj[d]) * __expf(fmaxf(GC[i * D + d] - GC[j * D + d], -20.f));
        }
#pragma unroll
        for (int jj = 0; jj < 64; ++jj)
          if (jj == j) row[jj] = s;
      }
    }
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const bool keep = is_q ? (j <= i) : (j < i);
      row[j] = keep ? guard(is_q ? row[j] * scale : row[j]) : 0.f;
    }
    if (is_q) {
      unsigned char* aqk_c = aqk_t + cb * TILE_CC;
#pragma unroll
      for (int c = 0; c < 64; c += 8) *reinterpret_cast<uint4*>(aqk_c + sw_off16(C, i, c)) = pack8(row + c);
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j) AKK[i * F1_LDA + j] = row[j];
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (flags[4]) goto teardown;
  {
    // 5. A = (I + Akk)^-1 in fp32: diagonal 16 x 16 blocks by substitution (warp w: block w),
    //    then X_IJ = -X_II sum_{K=J}^{I-1} Akk_IK X_KJ by block distance
    float* AF = reinterpret_cast<float*>(R1);
    float* TS = AF + C * F1_LDA;
    for (int e = tid; e < C * C; e += F1_THREADS) {
      const int r = e >> 6, c = e & 63;
      if ((c >> 4) != (r >> 4)) AF[r * F1_LDA + c] = 0.f;
    }
    {
      const int base = 16 * warp;
      for (int i = 0; i < 16; ++i) {
        float x = 0.f;
        if (lane < 16) {
          x = lane == i ? 1.f : 0.f;
          for (int j = lane; j < i; ++j) x -= AKK[(base + i) * F1_LDA + base + j] * AF[(base + j) * F1_LDA + base + lane];
        }
        __syncwarp();
        if (lane < 16) AF[(base + i) * F1_LDA + base + lane] = lane <= i ? x : 0.f;
        __syncwarp();
      }
    }
    __syncthreads();
    for (int dist = 1; dist < 4; ++dist) {
      const int np = 4 - dist;
      for (int e = tid; e < np * 256; e += F1_THREADS) {
        const int p = e >> 8, ii = (e >> 4) & 15, cc = e & 15;
        const int J = p, I = p + dist;
        float s = 0.f;
        for (int K = J; K < I; ++K)
#pragma unroll 4
          for (int kk = 0; kk < 16; ++kk)
            s += AKK[(16 * I + ii) * F1_LDA + 16 * K + kk] * AF[(16 * K + kk) * F1_LDA + 16 * J + cc];
        TS[e] = s;
      }
      __syncthreads();
      for (int e = tid; e < np * 256; e += F1_THREADS) {
        const int p = e >> 8, ii = (e >> 4) & 15, cc = e & 15;
        const int J = p, I = p + dist;
        float s = 0.f;
        for (int m = 0; m <= ii; ++m) s += AF[(16 * I + ii) * F1_LDA + 16 * I + m] * TS[(p << 8) + (m << 4) + cc];
        AF[(16 * I + ii) * F1_LDA + 16 * J + cc] = guard(-s);
      }
      __syncthreads();
    }
    // A out: fp32 rows for the chunk-parallel backward, bf16 operand tile (rows i, columns j)
    unsigned char* AT = R2 + 24576;
    for (int e = tid; e < C * 8; e += F1_THREADS) {
      const int i = e >> 3, c = (e & 7) << 3;
      float x[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) x[t] = AF[i * F1_LDA + c + t];
      st_chunk8(smem_u32(AT) + sw_off16(C, i, c), x);
      if (a_o) {
        float* dst = a_o + cb * C * C + i * C + c;
        *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
      }
    }
    __syncthreads();

    // 6. (b k) e^gc and (w v) tiles (rows j, columns d) in R1
    for (int it = 0; it < (C * D / 8) / F1_THREADS; ++it) {
      const int u_ = it * F1_THREADS + tid;
      const int i = u_ >> 4, c = (u_ & 15) << 3;
      const int64_t gi = ix.row(b, t0 + i, h) + c;
      float kv[8], bv[8], wv[8], vv[8], x[8], y[8];
      unpack8(*reinterpret_cast<const uint4*>(k + gi), kv);
      unpack8(*reinterpret_cast<const uint4*>(bg + gi), bv);
      unpack8(*reinterpret_cast<const uint4*>(wg + gi), wv);
      unpack8(*reinterpret_cast<const uint4*>(v + gi), vv);
      const float* gci = GC + i * D + c;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        x[e] = bv[e] * kv[e] * __expf(gci[e]);
        y[e] = wv[e] * vv[e];
      }
      st_chunk8(sR1 + sw_off16(C, i, c), x);
      st_chunk8(sR1 + TILE_CD + sw_off16(C, i, c), y);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    // 7. w~ = A (bk e^gc) -> TMEM columns [0, 128); u = A (w v) -> [128, 256)   (M = 64)
    if (tid == 0) {
      sm100::tc_fence_after();
      constexpr uint32_t IDESC_W = sm100::idesc_bf16(64, 128, false, true);
      const uint32_t sa = smem_u32(AT);
      auto fa = [&](int s) { return kdesc(sa, C, s); };
      mma_steps(tmem, fa, [&](int s) { return mndesc(sR1, C, s); }, C / 16, IDESC_W, false);
      mma_steps(tmem + 128, fa, [&](int s) { return mndesc(sR1 + TILE_CD, C, s); }, C / 16, IDESC_W, false);
      sm100::umma_commit(bars + 4);
    }
    if (!wait_bar(bars + 4, 0, err, 0x4704)) goto teardown;
    sm100::tc_fence_after();
    // 8. rows i = 16 warp + lane (lanes 0-15) of w~ and u out as tile images
    {
      const int i = 16 * warp + lane;
      unsigned char* wt_c = wt_t + cb * TILE_CD;
      unsigned char* u_c = u_t + cb * TILE_CD;
#pragma unroll 1
      for (int p = 0; p < 4; ++p) {
        float x[32];
        tmem_ld32(tmem_at(tmem, warp, 32 * p), x);
        if (lane < 16)
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = guard(x[c + e]);
            *reinterpret_cast<uint4*>(wt_c + sw_off16(C, i, 32 * p + c)) = pack8(y);
          }
        tmem_ld32(tmem_at(tmem, warp, 128 + 32 * p), x);
        if (lane < 16)
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = guard(x[c + e]);
            *reinterpret_cast<uint4*>(u_c + sw_off16(C, i, 32 * p + c)) = pack8(y);
          }
      }
    }
  }
teardown:
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 256);
}

// ============================================================ state recurrence, forward
// One CTA per (batch, head) walks the chunks in order with the whole 128 x 128 state: thread
// dk (= TMEM lane dk) keeps state row dk in registers.  Per chunk (tile images prefetched by
// bulk copies two chunks ahead):
//   V  = w~ h, O1 = qg h            (M = 64 rows of the chunk, K = 128)
//   v_new = u - V  -> bf16 tile     (CUDA cores)
//   O2 = Aqk v_new (K = 64), HH = kg^T v_new (M = 128 state rows, K = 64)
//   o = scale O1 + O2 ; h <- e^{gcl} h + HH (clip 1e4)
// (reference `atomic_ops/kernel_d_pipeline.py:94-158`, the inter-chunk combine with state)
constexpr int F2_THREADS = 128;
constexpr int F2_STAGE = 3 * TILE_CD + TILE_CC;  // w~, qg, kg, Aqk tile images
constexpr int F2_H = 2 * F2_STAGE;                // state tile (rows dk, columns dv), 32 KB
constexpr int F2_VN = F2_H + 2 * TILE_CD;         // v_new tile (rows i, columns dv), 16 KB
constexpr int F2_BARS = F2_VN + TILE_CD;
constexpr size_t F2_SMEM = 1024 + F2_BARS + 256;

__global__ void __launch_bounds__(F2_THREADS, 1) gdn_state_fwd_tc(
    const unsigned char* __restrict__ wt_t, const unsigned char* __restrict__ u_t,
    const unsigned char* __restrict__ qg_t, const unsigned char* __restrict__ kg_t,
    const unsigned char* __restrict__ aqk_t, const float* __restrict__ gcl, float scale, int L, int H, int NC,
    const float* __restrict__ h0, bf16* __restrict__ o, float* __restrict__ h_final, bf16* __restrict__ h_store,
    bf16* __restrict__ vn_store, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F2_BARS);  // full[2], mma1, mma2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const uint32_t sH = smem_u32(smem + F2_H), sVN = smem_u32(smem + F2_VN);

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = (int64_t)b * H + h;
  const SeqIdx ix{L, H};
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) sm100::mbar_init(bars + i, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto issue = [&](int n) {
    unsigned char* st = smem + (n & 1) * F2_STAGE;
    const int64_t c = bh * NC + n;
    sm100::mbar_expect_tx(bars + (n & 1), F2_STAGE);
    bulk_g2s(st, wt_t + c * TILE_CD, TILE_CD, bars + (n & 1));
    bulk_g2s(st + TILE_CD, qg_t + c * TILE_CD, TILE_CD, bars + (n & 1));
    bulk_g2s(st + 2 * TILE_CD, kg_t + c * TILE_CD, TILE_CD, bars + (n & 1));
    bulk_g2s(st + 3 * TILE_CD, aqk_t + c * TILE_CC, TILE_CC, bars + (n & 1));
  };
  if (tid == 0) {
    issue(0);
    if (NC > 1) issue(1);
  }
  const int dk = tid;
  float hr[D];
#pragma unroll
  for (int c = 0; c < D; ++c) hr[c] = h0 ? h0[(bh * D + dk) * D + c] : 0.f;

  constexpr uint32_t ID_ROWS = sm100::idesc_bf16(64, 128, false, true);  // chunk rows x dv
  constexpr uint32_t ID_STATE = sm100::idesc_bf16(128, 128, true, true);  // dk x dv
  int n = 0;
  for (; n < NC; ++n) {
    const int64_t cbn = bh * NC + n;
    const uint32_t st = smem_u32(smem + (n & 1) * F2_STAGE);
    // state row dk -> operand tile (MN-major B: rows dk, columns dv) and the per-chunk store
#pragma unroll
    for (int c = 0; c < D; c += 8) {
      st_chunk8(sH + sw_off16(D, dk, c), hr + c);
      if (h_store) *reinterpret_cast<uint4*>(h_store + cbn * D * D + dk * D + c) = pack8(hr + c);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      if (!wait_bar(bars + (n & 1), (n >> 1) & 1, err, 0x4711)) *abort_flag = 1;
      sm100::tc_fence_after();
      if (!*abort_flag) {
        auto fh = [&](int s) { return mndesc(sH, D, s); };
        mma_steps(tmem, [&](int s) { return kdesc(st, C, s); }, fh, D / 16, ID_ROWS, false);
        mma_steps(tmem + 128, [&](int s) { return kdesc(st + TILE_CD, C, s); }, fh, D / 16, ID_ROWS, false);
      }
      sm100::umma_commit(bars + 2);
    }
    if (!wait_bar(bars + 2, n & 1, err, 0x4712)) *abort_flag = 1;
    sm100::tc_fence_after();
    // v_new rows i = 16 warp + lane (lanes 0-15)
    {
      const int i = 16 * warp + lane;
      const unsigned char* u_c = u_t + cbn * TILE_CD;
#pragma unroll 1
      for (int p = 0; p < 4; ++p) {
        float x[32];
        tmem_ld32(tmem_at(tmem, warp, 32 * p), x);
        if (lane < 16)
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float uu[8], y[8];
            unpack8(*reinterpret_cast<const uint4*>(u_c + sw_off16(C, i, 32 * p + c)), uu);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = uu[e] - x[c + e];
            st_chunk8(sVN + sw_off16(C, i, 32 * p + c), y);
            if (vn_store) *reinterpret_cast<uint4*>(vn_store + cbn * C * D + i * D + 32 * p + c) = pack8(y);
          }
      }
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0) {
      sm100::tc_fence_after();
      auto fvn = [&](int s) { return mndesc(sVN, C, s); };
      mma_steps(tmem + 256, [&](int s) { return kdesc(st + 3 * TILE_CD, C, s); }, fvn, C / 16, ID_ROWS, false);
      mma_steps(tmem + 384, [&](int s) { return mndesc(st + 2 * TILE_CD, C, s); }, fvn, C / 16, ID_STATE, false);
      sm100::umma_commit(bars + 3);
    }
    if (!wait_bar(bars + 3, n & 1, err, 0x4713)) *abort_flag = 1;
    sm100::tc_fence_after();
    if (o) {
      const int i = 16 * warp + lane;
      bf16* orow = o + ix.row(b, (int64_t)n * C + i, h);
#pragma unroll 1
      for (int p = 0; p < 4; ++p) {
        float x1[32], x2[32];
        tmem_ld32(tmem_at(tmem, warp, 128 + 32 * p), x1);
        tmem_ld32(tmem_at(tmem, warp, 256 + 32 * p), x2);
        if (lane < 16)
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = guard(scale * x1[c + e] + x2[c + e]);
            *reinterpret_cast<uint4*>(orow + 32 * p + c) = pack8(y);
          }
      }
    }
    {
      const float eg = __expf(gcl[cbn * D + dk]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float x[32];
        tmem_ld32(tmem_at(tmem, warp, 384 + 32 * p), x);
#pragma unroll
        for (int e = 0; e < 32; ++e) hr[32 * p + e] = sanitize(eg * hr[32 * p + e] + x[e], 1e4f);
      }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0 && n + 2 < NC) issue(n + 2);
  }
  if (h_final && n == NC)
#pragma unroll
    for (int c = 0; c < D; ++c) h_final[(bh * D + dk) * D + c] = hr[c];
  if (*abort_flag && tid == 0) {  // let copies in flight land before the CTA exits
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 512);
}

// ============================================================ state recurrence, backward
// Reverse walk over the chunks with the state gradient dh (rows dk in registers), reference
// `atomic_ops/kernel_bwd_b1_dhu.py:14-44`:
//   DVN = Aqk^T do + kg dh              (M = 64, K = 64 + 128)   -> dv_new
//   D1  = qg^T do , D2 = w~^T dv_new    (M = 128 state rows, K = 64)
//   dh  <- e^{gcl} dh + scale D1 - D2
// do arrives by TMA (3-D map over (B, L, H, D), two 64-column boxes per chunk).
constexpr int B1_THREADS = 128;
constexpr int B1_STAGE = 4 * TILE_CD + TILE_CC;  // w~, qg, kg, Aqk, do
constexpr int B1_DO = 3 * TILE_CD + TILE_CC;      // offset of do inside a stage
constexpr int B1_DH = 2 * B1_STAGE;
constexpr int B1_DVN = B1_DH + 2 * TILE_CD;
constexpr int B1_BARS = B1_DVN + TILE_CD;
constexpr size_t B1_SMEM = 1024 + B1_BARS + 256;

__global__ void __launch_bounds__(B1_THREADS, 1) gdn_state_bwd_tc(
    const __grid_constant__ CUtensorMap tm_do, const unsigned char* __restrict__ wt_t,
    const unsigned char* __restrict__ qg_t, const unsigned char* __restrict__ kg_t,
    const unsigned char* __restrict__ aqk_t, const float* __restrict__ gcl, float scale, int L, int H, int NC,
    const float* __restrict__ dh_final, bf16* __restrict__ dh_store, bf16* __restrict__ dvn_store,
    float* __restrict__ dh0, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + B1_BARS);  // full[2], mma1, mma2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const uint32_t sDH = smem_u32(smem + B1_DH), sDVN = smem_u32(smem + B1_DVN);

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = (int64_t)b * H + h;
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) sm100::mbar_init(bars + i, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tm_do);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto issue = [&](int n, int s) {
    unsigned char* st = smem + s * B1_STAGE;
    const int64_t c = bh * NC + n;
    sm100::mbar_expect_tx(bars + s, B1_STAGE);
    bulk_g2s(st, wt_t + c * TILE_CD, TILE_CD, bars + s);
    bulk_g2s(st + TILE_CD, qg_t + c * TILE_CD, TILE_CD, bars + s);
    bulk_g2s(st + 2 * TILE_CD, kg_t + c * TILE_CD, TILE_CD, bars + s);
    bulk_g2s(st + 3 * TILE_CD, aqk_t + c * TILE_CC, TILE_CC, bars + s);
    const int row = b * L + n * C;
    tma_load_3d(st + B1_DO, &tm_do, bars + s, 0, h, row);
    tma_load_3d(st + B1_DO + TILE_CD / 2, &tm_do, bars + s, 64, h, row);
  };
  if (tid == 0) {
    issue(NC - 1, 0);
    if (NC > 1) issue(NC - 2, 1);
  }
  const int dk = tid;
  float dr[D];
#pragma unroll
  for (int c = 0; c < D; ++c) dr[c] = dh_final ? dh_final[(bh * D + dk) * D + c] : 0.f;

  constexpr uint32_t ID_RR = sm100::idesc_bf16(64, 128, true, true);    // rows i x dv, A = Aqk^T (MN)
  constexpr uint32_t ID_RK = sm100::idesc_bf16(64, 128, false, true);   // rows i x dv, A = kg (K-major)
  constexpr uint32_t ID_ST = sm100::idesc_bf16(128, 128, true, true);   // dk x dv
  int it = 0;
  for (; it < NC; ++it) {
    const int n = NC - 1 - it, s = it & 1;
    const int64_t cbn = bh * NC + n;
    const uint32_t st = smem_u32(smem + s * B1_STAGE);
#pragma unroll
    for (int c = 0; c < D; c += 8) {
      st_chunk8(sDH + sw_off16(D, dk, c), dr + c);
      *reinterpret_cast<uint4*>(dh_store + cbn * D * D + dk * D + c) = pack8(dr + c);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      if (!wait_bar(bars + s, (it >> 1) & 1, err, 0x4721)) *abort_flag = 1;
      sm100::tc_fence_after();
      if (!*abort_flag) {
        const uint32_t sdo = st + B1_DO;
        auto fdo = [&](int k) { return mndesc(sdo, C, k); };
        mma_steps(tmem, [&](int k) { return mndesc(st + 3 * TILE_CD, C, k); }, fdo, C / 16, ID_RR, false);
        mma_steps(tmem, [&](int k) { return kdesc(st + 2 * TILE_CD, C, k); }, [&](int k) { return mndesc(sDH, D, k); },
                  D / 16, ID_RK, true);
        mma_steps(tmem + 128, [&](int k) { return mndesc(st + TILE_CD, C, k); }, fdo, C / 16, ID_ST, false);
      }
      sm100::umma_commit(bars + 2);
    }
    if (!wait_bar(bars + 2, it & 1, err, 0x4722)) *abort_flag = 1;
    sm100::tc_fence_after();
    {
      const int i = 16 * warp + lane;
#pragma unroll 1
      for (int p = 0; p < 4; ++p) {
        float x[32];
        tmem_ld32(tmem_at(tmem, warp, 32 * p), x);
        if (lane < 16)
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            st_chunk8(sDVN + sw_off16(C, i, 32 * p + c), x + c);
            *reinterpret_cast<uint4*>(dvn_store + cbn * C * D + i * D + 32 * p + c) = pack8(x + c);
          }
      }
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0) {
      sm100::tc_fence_after();
      mma_steps(tmem + 256, [&](int k) { return mndesc(st, C, k); }, [&](int k) { return mndesc(sDVN, C, k); }, C / 16,
                ID_ST, false);
      sm100::umma_commit(bars + 3);
    }
    if (!wait_bar(bars + 3, it & 1, err, 0x4723)) *abort_flag = 1;
    sm100::tc_fence_after();
    {
      const float eg = __expf(gcl[cbn * D + dk]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float x1[32], x2[32];
        tmem_ld32(tmem_at(tmem, warp, 128 + 32 * p), x1);
        tmem_ld32(tmem_at(tmem, warp, 256 + 32 * p), x2);
#pragma unroll
        for (int e = 0; e < 32; ++e) dr[32 * p + e] = eg * dr[32 * p + e] + scale * x1[e] - x2[e];
      }
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0 && it + 2 < NC) issue(n - 2, s);
  }
  if (dh0 && it == NC)
#pragma unroll
    for (int c = 0; c < D; ++c) dh0[(bh * D + dk) * D + c] = dr[c];
  if (*abort_flag && tid == 0) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 512);
}

template <class K>
int set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess ? 0 : -3;
}

}  // namespace

// ===================================================================== launchers
int ahb_gdn_chunk_fwd_tc(const void* q, const void* k, const void* v, const float* g, const void* bg, const void* wg,
                         float scale, int B, int L, int H, void* wt_t, void* u_t, void* qg_t, void* kg_t, void* aqk_t,
                         float* gcl, float* a_out, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_chunk_fwd_tc, F1_SMEM);
  if (init) return init;
  gdn_chunk_fwd_tc<<<dim3(L / C, H, B), F1_THREADS, F1_SMEM, st>>>(
      (const bf16*)q, (const bf16*)k, (const bf16*)v, g, (const bf16*)bg, (const bf16*)wg, scale, L, H,
      (unsigned char*)wt_t, (unsigned char*)u_t, (unsigned char*)qg_t, (unsigned char*)kg_t, (unsigned char*)aqk_t,
      gcl, a_out, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int ahb_gdn_state_fwd_tc(const void* wt_t, const void* u_t, const void* qg_t, const void* kg_t, const void* aqk_t,
                         const float* gcl, float scale, int B, int L, int H, const float* h0, void* o, float* h_final,
                         void* h_store, void* vn_store, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_state_fwd_tc, F2_SMEM);
  if (init) return init;
  gdn_state_fwd_tc<<<dim3(H, B), F2_THREADS, F2_SMEM, st>>>(
      (const unsigned char*)wt_t, (const unsigned char*)u_t, (const unsigned char*)qg_t, (const unsigned char*)kg_t,
      (const unsigned char*)aqk_t, gcl, scale, L, H, L / C, h0, (bf16*)o, h_final, (bf16*)h_store, (bf16*)vn_store,
      err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int ahb_gdn_state_bwd_tc(const void* wt_t, const void* qg_t, const void* kg_t, const void* aqk_t, const float* gcl,
                         const void* dout, float scale, int B, int L, int H, const float* dh_final, void* dh_store,
                         void* dvn_store, float* dh0, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_state_bwd_tc, B1_SMEM);
  if (init) return init;
  CUtensorMap tm;
  if (tmap_seq_bf16(&tm, dout, (int64_t)B * L, H, D, C)) return -20;
  gdn_state_bwd_tc<<<dim3(H, B), B1_THREADS, B1_SMEM, st>>>(
      tm, (const unsigned char*)wt_t, (const unsigned char*)qg_t, (const unsigned char*)kg_t,
      (const unsigned char*)aqk_t, gcl, scale, L, H, L / C, dh_final, (bf16*)dh_store, (bf16*)dvn_store, dh0, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
