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
#include "phase_prof.cuh"
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
// fp32 Akk [64][64] with its 16-byte column groups XOR-swizzled by the row: the writers (one row per
// lane, same group) spread over the banks, the readers (whole warp, one row) get a broadcast
AHB_DEVICE int akk_at(int i, int j4) { return i * C + ((j4 ^ (i & 15)) << 2); }

// rows [R0, R0 + 8) of x = DI acc for one diagonal block (DI unit lower triangular, [r][k] fp32 rows
// of 16, read as broadcast 16-byte vectors); entries of blocks off the column's diagonal are guarded
template <int R0>
AHB_DEVICE void inv_rows(const float* Dw, const float (&a)[16], float (&xo)[8], bool off) {
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int rr = R0 + r;
    float s0 = a[rr], s1 = 0.f;
#pragma unroll
    for (int k = 0; k + 3 < rr; k += 4) {
      const float4 d4 = *reinterpret_cast<const float4*>(Dw + 16 * rr + k);
      s0 += d4.x * a[k] + d4.z * a[k + 2];
      s1 += d4.y * a[k + 1] + d4.w * a[k + 3];
    }
#pragma unroll
    for (int k = rr & ~3; k < rr; ++k) s0 += Dw[16 * rr + k] * a[k];
    xo[r] = off ? guard(s0 + s1) : s0 + s1;
  }
}
constexpr size_t F1_SMEM = 1024 + 3 * 32768 + 256;

__global__ void __launch_bounds__(F1_THREADS, 2) gdn_chunk_fwd_tc(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
    const float* __restrict__ g, const bf16* __restrict__ bg, const bf16* __restrict__ wg, float scale, int L,
    int H, unsigned char* __restrict__ wt_t, unsigned char* __restrict__ u_t, unsigned char* __restrict__ qg_t,
    unsigned char* __restrict__ kg_t, unsigned char* __restrict__ aqk_t, float* __restrict__ gcl_o,
    unsigned char* __restrict__ at_t, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* R1 = smem;
  unsigned char* R2 = smem + 32768;
  float* GC = reinterpret_cast<float*>(smem + 65536);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 98304);  // [0..3] score blocks, [4] w~/u
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0..3] exact diagonal block, [4] abort
  float* span_w = reinterpret_cast<float*>(flags + 8);  // [4 warps][4 blocks]
  PhaseClock pc(0);

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

  // 1. g -> GC, cumulative sum per channel (thread d owns channel d); the q / k / b rows of
  //    step 2 are requested first so their latency overlaps the scan
  constexpr int UNITS = (C * D / 8) / F1_THREADS;  // 16-byte units per thread and tile
  uint4 qa[UNITS], ka[UNITS], ba[UNITS];
#pragma unroll
  for (int it = 0; it < UNITS; ++it) {
    const int u_ = it * F1_THREADS + tid;
    const int64_t gi = ix.row(b, t0 + (u_ >> 4), h) + ((u_ & 15) << 3);
    qa[it] = *reinterpret_cast<const uint4*>(q + gi);
    ka[it] = *reinterpret_cast<const uint4*>(k + gi);
    ba[it] = *reinterpret_cast<const uint4*>(bg + gi);
  }
#pragma unroll
  for (int e = tid; e < C * (D / 4); e += F1_THREADS) {
    const int r = e >> 5, c4 = (e & 31) << 2;
    cp_async16(GC + r * D + c4, g + ix.row(b, t0 + r, h) + c4);  // no registers held for the gate rows
  }
  cp_async_wait_all();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pc.mark(0);
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
  pc.mark(1);

  // 2. stacked score rows: R1 rows 0-63 = q e^{gc - gc_r}, rows 64-127 = (b k) e^{gc - gc_r};
  //    qg = q e^gc and kg = k e^{gcl - gc} go straight out as tile images
  unsigned char* qg_c = qg_t + cb * TILE_CD;
  unsigned char* kg_c = kg_t + cb * TILE_CD;
#pragma unroll
  for (int it = 0; it < UNITS; ++it) {
    const int u_ = it * F1_THREADS + tid;
    const int i = u_ >> 4, c = (u_ & 15) << 3;
    float qv[8], kv[8], bv[8];
    unpack8(qa[it], qv);
    unpack8(ka[it], kv);
    unpack8(ba[it], bv);
    float gci[8], gcr[8], gcl[8];
    ld8f_x(GC + i * D + c, gci);
    ld8f_x(GC + (i & ~15) * D + c, gcr);
    ld8f_x(GC + (C - 1) * D + c, gcl);
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
#pragma unroll
  for (int I = 0; I < 4; ++I) {
    unsigned char* buf = R2 + (I & 1) * TILE_CD;
    if (I >= 2 && !wait_bar(bars + I - 2, 0, err, 0x4701)) flags[4] = 1;
    const bool exact = flags[I];
    const float* gcr = GC + 16 * I * D;
    // rows j < 16 (I + 1): the k rows held from step 2 are units 0 .. 2 (I + 1) - 1 of this thread
#pragma unroll
    for (int it = 0; it < 2 * (I + 1); ++it) {
      const int u_ = it * F1_THREADS + tid;
      const int j = u_ >> 4, c = (u_ & 15) << 3;
      float kv[8], o[8];
      unpack8(ka[it], kv);
      float gcj[8], gr8[8];
      ld8f_x(GC + j * D + c, gcj);
      ld8f_x(gcr + c, gr8);
      const bool zero = exact && j >= 16 * I;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = zero ? 0.f : kv[e] * __expf(gr8[e] - gcj[e]);
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
  pc.mark(2);
  if (!wait_bar(bars + 2, 0, err, 0x4702) || !wait_bar(bars + 3, 0, err, 0x4703)) flags[4] = 1;
  sm100::tc_fence_after();
  pc.mark(3);

  // 4. scores out of TMEM: lane m of quarter q is row m = 32 q + lane of the stack
  float* AKK = reinterpret_cast<float*>(R2);  // fp32 [64][64], akk_at
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
    if (is_q) {  // the Aqk tile image, staged for one bulk store (per-lane row stores stall the warps)
#pragma unroll
      for (int c = 0; c < 64; c += 8) *reinterpret_cast<uint4*>(R2 + 16384 + sw_off16(C, i, c)) = pack8(row + c);
      fence_async_smem();
    } else {
#pragma unroll
      for (int j = 0; j < 64; j += 4)
        *reinterpret_cast<float4*>(AKK + akk_at(i, j >> 2)) = make_float4(row[j], row[j + 1], row[j + 2], row[j + 3]);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    bulk_s2g(aqk_t + cb * TILE_CC, R2 + 16384, TILE_CC);
    bulk_commit();
  }
  pc.mark(4);
  const long long t_after4 = clock64();
  if (flags[4]) goto teardown;
  {
    // 5. A = (I + Akk)^-1 in fp32 by blocked forward substitution.
    //    (a) warp w inverts the diagonal 16 x 16 block w of (I + Akk) by substitution (lane j =
    //        column j) into DI, rows 0-15 of the accumulator region (never read as accumulators);
    //    (b) column c by two threads, block by block: the block's x = DI_B acc_B (independent dot
    //        products, no chain over the rows), then acc_i -= sum_{j in block} Akk_ij x_j for the
    //        rows below (fp32 [i][c] in the first half of R1, acc_i = [i == c] before any update).
    //        Entries outside the diagonal blocks are guarded.
    unsigned char* AT = R2 + 24576;
    float* ACC = reinterpret_cast<float*>(R1);           // [i][c]
    float* DI = ACC;                                     // [w][r][j], 4 x 16 x 16
    float* XS = reinterpret_cast<float*>(R2 + 16384);    // [r][c]: x of the current block
    {
      // 6b. (w v) tile (rows j, columns d) in the second half of R1, 8 units per thread in two
      //     batches; the first batch's loads are in flight during the DI solve
      uint4 wa[4], va[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int u_ = q * F1_THREADS + tid;
        const int64_t gi = ix.row(b, t0 + (u_ >> 4), h) + ((u_ & 15) << 3);
        wa[q] = *reinterpret_cast<const uint4*>(wg + gi);
        va[q] = *reinterpret_cast<const uint4*>(v + gi);
      }
      if (lane < 16) {
        const int j = lane, w = warp;
        float y[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const int i = 16 * w + r;
          float s = r == j ? 1.f : 0.f;
#pragma unroll
          for (int k = 0; k < r; ++k) s -= AKK[akk_at(i, 4 * w + (k >> 2)) + (k & 3)] * y[k];
          y[r] = r < j ? 0.f : s;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) DI[(16 * w + r) * 16 + j] = y[r];
      }
#pragma unroll 1
      for (int b2 = 0; b2 < 2; ++b2) {
        if (b2 == 1)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int u_ = (4 + q) * F1_THREADS + tid;
            const int64_t gi = ix.row(b, t0 + (u_ >> 4), h) + ((u_ & 15) << 3);
            wa[q] = *reinterpret_cast<const uint4*>(wg + gi);
            va[q] = *reinterpret_cast<const uint4*>(v + gi);
          }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int u_ = (4 * b2 + q) * F1_THREADS + tid;
          float wv[8], vv[8];
          unpack8(wa[q], wv);
          unpack8(va[q], vv);
#pragma unroll
          for (int e = 0; e < 8; ++e) wv[e] *= vv[e];
          st_chunk8(sR1 + TILE_CD + sw_off16(C, u_ >> 4, (u_ & 15) << 3), wv);
        }
      }
    }
    if (tid == 0) bulk_wait_read();  // the Aqk staging tile has been read: XS reuses it
    __syncthreads();
    {
      // (b) two threads per column c: thread half hh computes rows [8 hh, 8 hh + 8) of each block's
      //     x = DI_B acc_B, the halves meet in XS, and each thread updates every other group of 8
      //     rows below the block
      const int c = tid & (C - 1), hh = tid >> 6;
#pragma unroll 1
      for (int B = 0; B < 4; ++B) {
        float a[16], xh[8], x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) a[r] = B == 0 ? (r == c ? 1.f : 0.f) : ACC[(16 * B + r) * C + c];
        const float* Dw = DI + 256 * B;
        const bool off = B != (c >> 4);
        if (hh == 0)
          inv_rows<0>(Dw, a, xh, off);
        else
          inv_rows<8>(Dw, a, xh, off);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          XS[(8 * hh + r) * C + c] = xh[r];
          *reinterpret_cast<bf16*>(AT + sw_off(C, 16 * B + 8 * hh + r, c)) = __float2bfloat16_rn(xh[r]);
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 16; ++r) x[r] = XS[r * C + c];
        // rows below, eight at a time, alternate groups per half: the group's loads come before its stores
#pragma unroll 1
        for (int i0 = 16 * B + 16 + 8 * hh; i0 < C; i0 += 16) {
          float prev[8], upd[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) prev[t] = B == 0 ? (i0 + t == c ? 1.f : 0.f) : ACC[(i0 + t) * C + c];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 l4 = *reinterpret_cast<const float4*>(AKK + akk_at(i0 + t, 4 * B + q));
              s0 += l4.x * x[4 * q] + l4.z * x[4 * q + 2];
              s1 += l4.y * x[4 * q + 1] + l4.w * x[4 * q + 3];
            }
            upd[t] = prev[t] - (s0 + s1);
          }
#pragma unroll
          for (int t = 0; t < 8; ++t) ACC[(i0 + t) * C + c] = upd[t];
        }
        __syncthreads();  // the rows below are complete before the next block reads them; XS is free
      }
    }
    pc.warp_mark(10, t_after4);
    __syncthreads();
    pc.mark(5);
    // 6a. (b k) e^gc tile (rows j, columns d) over the accumulators in the first half of R1 (all
    //     the gate loads before the stores)
    {
      float xb[UNITS][8];
#pragma unroll
      for (int it = 0; it < UNITS; ++it) {
        const int u_ = it * F1_THREADS + tid;
        const int i = u_ >> 4, c = (u_ & 15) << 3;
        float kv[8], bv[8], gci[8];
        unpack8(ka[it], kv);
        unpack8(ba[it], bv);
        ld8f_x(GC + i * D + c, gci);
#pragma unroll
        for (int e = 0; e < 8; ++e) xb[it][e] = bv[e] * kv[e] * __expf(gci[e]);
      }
#pragma unroll
      for (int it = 0; it < UNITS; ++it) {
        const int u_ = it * F1_THREADS + tid;
        st_chunk8(sR1 + sw_off16(C, u_ >> 4, (u_ & 15) << 3), xb[it]);
      }
    }
    pc.mark(9);
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    // A as a tile image for the backward
    if (at_t)
#pragma unroll
      for (int e = tid; e < C * 8; e += F1_THREADS)
        *reinterpret_cast<uint4*>(at_t + cb * TILE_CC + 16 * e) = *reinterpret_cast<const uint4*>(AT + 16 * e);
    pc.mark(6);
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
    pc.mark(7);
    // 8. rows i = 16 warp + (lane & 15) of w~ and u as tile images: lanes 0-15 hold the rows
    //    (M = 64), lanes 16-31 take the upper 16 columns of each 32-column load by shuffle; staged
    //    over the dead operands in R1, then two bulk stores
    {
      const int i = 16 * warp + (lane & 15), hf = lane >> 4;
#pragma unroll 1
      for (int p = 0; p < 8; ++p) {
        unsigned char* dst = R1 + (p < 4 ? 0 : TILE_CD);
        const int col = 32 * (p & 3) + 16 * hf;
        float x[32], y[16];
        tmem_ld32(tmem_at(tmem, warp, 32 * p), x);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, x[16 + e], lane & 15);
          y[e] = guard(hf ? sh : x[e]);
        }
        *reinterpret_cast<uint4*>(dst + sw_off16(C, i, col)) = pack8(y);
        *reinterpret_cast<uint4*>(dst + sw_off16(C, i, col + 8)) = pack8(y + 8);
      }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      bulk_s2g(wt_t + cb * TILE_CD, R1, TILE_CD);
      bulk_s2g(u_t + cb * TILE_CD, R1 + TILE_CD, TILE_CD);
      bulk_commit();
    }
  }
teardown:
  if (tid == 0) bulk_wait_all();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  pc.mark(8);
  if (warp == 0) sm100::tmem_dealloc(tmem, 256);
  pc.done();
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
constexpr int F2_STAGE = 4 * TILE_CD + TILE_CC;  // w~, qg, kg, Aqk tile images, this CTA's u columns
constexpr int F2_U = 3 * TILE_CD + TILE_CC;       // offset of u inside a stage
constexpr int F2_H = 2 * F2_STAGE;                // state tile (rows dk, columns dv), 32 KB
constexpr int F2_VN = F2_H + 2 * TILE_CD;         // v_new tile (rows i, columns dv), 16 KB
constexpr int F2_O = F2_VN + TILE_CD;            // o rows (two 64-column swizzled boxes), 16 KB
constexpr int F2_BARS = F2_O + TILE_CD;
constexpr size_t F2_SMEM = 1024 + F2_BARS + 256;

// NH = 2: the value columns split over two CTAs per (batch, head) (blockIdx.z = half; the columns of
// the state and of v_new evolve independently), for batches with fewer (batch, head) pairs than half
// the SMs; each CTA keeps 64 columns and writes its slab of the per-chunk images.
template <int NH>
__global__ void __launch_bounds__(F2_THREADS, 1) gdn_state_fwd_tc(
    const __grid_constant__ CUtensorMap tm_o, const unsigned char* __restrict__ wt_t, const unsigned char* __restrict__ u_t,
    const unsigned char* __restrict__ qg_t, const unsigned char* __restrict__ kg_t,
    const unsigned char* __restrict__ aqk_t, const float* __restrict__ gcl, float scale, int L, int H, int NC,
    const float* __restrict__ h0, bf16* __restrict__ o, float* __restrict__ h_final, unsigned char* __restrict__ h_store,
    unsigned char* __restrict__ vn_store, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F2_BARS);  // full[2], mma1, mma2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const uint32_t sH = smem_u32(smem + F2_H), sVN = smem_u32(smem + F2_VN);
  PhaseClock pc(32);

  constexpr int DV = D / NH;  // value columns of this CTA
  constexpr uint32_t TCOLS = NH == 1 ? 512 : 256;
  // TMEM: V [0, DV), O1 [DV, 2 DV), O2 [2 DV, 3 DV), HH [3 DV, 4 DV)
  const int h = blockIdx.x, b = blockIdx.y, v0 = DV * (int)blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = (int64_t)b * H + h;
  const SeqIdx ix{L, H};
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) sm100::mbar_init(bars + i, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, TCOLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto issue = [&](int n) {
    unsigned char* st = smem + (n & 1) * F2_STAGE;
    const int64_t c = bh * NC + n;
    sm100::mbar_expect_tx(bars + (n & 1), F2_U + DV * C * 2);
    bulk_g2s(st, wt_t + c * TILE_CD, TILE_CD, bars + (n & 1));
    bulk_g2s(st + TILE_CD, qg_t + c * TILE_CD, TILE_CD, bars + (n & 1));
    bulk_g2s(st + 2 * TILE_CD, kg_t + c * TILE_CD, TILE_CD, bars + (n & 1));
    bulk_g2s(st + 3 * TILE_CD, aqk_t + c * TILE_CC, TILE_CC, bars + (n & 1));
    bulk_g2s(st + F2_U, u_t + c * TILE_CD + (v0 >> 6) * (C * 128), DV * C * 2, bars + (n & 1));
  };
  if (tid == 0) {
    issue(0);
    if (NC > 1) issue(1);
  }
  const int dk = tid;
  float hr[DV];
#pragma unroll
  for (int c = 0; c < DV; ++c) hr[c] = h0 ? h0[(bh * D + dk) * D + v0 + c] : 0.f;

  constexpr uint32_t ID_ROWS = sm100::idesc_bf16(64, DV, false, true);  // chunk rows x dv
  constexpr uint32_t ID_STATE = sm100::idesc_bf16(128, DV, true, true);  // dk x dv
  int n = 0;
  for (; n < NC; ++n) {
    const int64_t cbn = bh * NC + n;
    const uint32_t st = smem_u32(smem + (n & 1) * F2_STAGE);
    // state row dk -> operand tile (MN-major B: rows dk, columns dv) and the per-chunk store
#pragma unroll
    for (int c = 0; c < DV; c += 8) {
      st_chunk8(sH + sw_off16(D, dk, c), hr + c);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(0);
    if (tid == 0) {
      if (h_store) {  // the state tile image: this CTA's column half (or both) as one bulk store
        bulk_s2g(h_store + cbn * (2 * TILE_CD) + (v0 >> 6) * (D * 128), smem + F2_H, DV * D * 2);
        bulk_commit();
      }
      if (!wait_bar(bars + (n & 1), (n >> 1) & 1, err, 0x4711)) *abort_flag = 1;
      pc.mark(6);
      sm100::tc_fence_after();
      if (!*abort_flag) {
        auto fh = [&](int s) { return mndesc(sH, D, s); };
        mma_steps(tmem, [&](int s) { return kdesc(st, C, s); }, fh, D / 16, ID_ROWS, false);
        mma_steps(tmem + DV, [&](int s) { return kdesc(st + TILE_CD, C, s); }, fh, D / 16, ID_ROWS, false);
      }
      sm100::umma_commit(bars + 2);
    }
    if (!wait_bar(bars + 2, n & 1, err, 0x4712)) *abort_flag = 1;
    sm100::tc_fence_after();
    pc.mark(1);
    // v_new rows i = 16 warp + (lane & 15) (M = 64: lanes 0-15 hold them); lanes 16-31 take the
    // upper 16 columns of each 32-column load by shuffle
    {
      const int i = 16 * warp + (lane & 15), hf = lane >> 4;
      const unsigned char* u_c = smem + (n & 1) * F2_STAGE + F2_U;  // this CTA's columns
      if (!wait_bar(bars + (n & 1), (n >> 1) & 1, err, 0x4714)) *abort_flag = 1;  // every thread reads u
#pragma unroll 1
      for (int p = 0; p < DV / 32; ++p) {
        float x[32], xs[16];
        tmem_ld32(tmem_at(tmem, warp, 32 * p), x);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, x[16 + e], lane & 15);
          xs[e] = hf ? sh : x[e];
        }
#pragma unroll
        for (int c = 0; c < 16; c += 8) {
          const int col = 32 * p + 16 * hf + c;
          float uu[8], y[8];
          unpack8(*reinterpret_cast<const uint4*>(u_c + sw_off16(C, i, col)), uu);
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = uu[e] - xs[c + e];
          st_chunk8(sVN + sw_off16(C, i, col), y);
        }
      }
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(2);
    if (*abort_flag) break;
    if (tid == 0) {
      if (o) bulk_wait_read();  // the previous chunk's o box is read before the epilogue below rewrites it
      if (vn_store) {
        bulk_s2g(vn_store + cbn * TILE_CD + (v0 >> 6) * (C * 128), smem + F2_VN, DV * C * 2);
        bulk_commit();
      }
      sm100::tc_fence_after();
      auto fvn = [&](int s) { return mndesc(sVN, C, s); };
      mma_steps(tmem + 2 * DV, [&](int s) { return kdesc(st + 3 * TILE_CD, C, s); }, fvn, C / 16, ID_ROWS, false);
      mma_steps(tmem + 3 * DV, [&](int s) { return mndesc(st + 2 * TILE_CD, C, s); }, fvn, C / 16, ID_STATE, false);
      sm100::umma_commit(bars + 3);
    }
    if (!wait_bar(bars + 3, n & 1, err, 0x4713)) *abort_flag = 1;
    sm100::tc_fence_after();
    pc.mark(3);
    if (o) {  // o rows into the swizzled boxes (all lanes, as v_new); stored by TMA after the chunk's last barrier
      const int i = 16 * warp + (lane & 15), hf = lane >> 4;
#pragma unroll 1
      for (int p = 0; p < DV / 32; ++p) {
        float x1[32], x2[32], ys[16];
        tmem_ld32(tmem_at(tmem, warp, DV + 32 * p), x1);
        tmem_ld32(tmem_at(tmem, warp, 2 * DV + 32 * p), x2);
#pragma unroll
        for (int e = 0; e < 32; ++e) x1[e] = scale * x1[e] + x2[e];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, x1[16 + e], lane & 15);
          ys[e] = guard(hf ? sh : x1[e]);
        }
#pragma unroll
        for (int c = 0; c < 16; c += 8)
          *reinterpret_cast<uint4*>(smem + F2_O + sw_off16(C, i, 32 * p + 16 * hf + c)) = pack8(ys + c);
      }
      fence_async_smem();
    }
    pc.mark(4);
    {
      const float eg = __expf(gcl[cbn * D + dk]);
#pragma unroll
      for (int p = 0; p < DV / 32; ++p) {
        float x[32];
        tmem_ld32(tmem_at(tmem, warp, 3 * DV + 32 * p), x);
#pragma unroll
        for (int e = 0; e < 32; ++e) hr[32 * p + e] = sanitize(eg * hr[32 * p + e] + x[e], 1e4f);
      }
    }
    if (tid == 0) bulk_wait_read();  // the h / v_new tiles are rewritten in the next step
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(5);
    if (tid == 0 && o) {
#pragma unroll
      for (int hb = 0; hb < DV / 64; ++hb)
        tma_store_3d(&tm_o, smem + F2_O + hb * (C * 128), v0 + 64 * hb, h, b * L + n * C);
      bulk_commit();
    }
    if (*abort_flag) break;
    if (tid == 0 && n + 2 < NC) issue(n + 2);
  }
  if (h_final && n == NC)
#pragma unroll
    for (int c = 0; c < DV; ++c) h_final[(bh * D + dk) * D + v0 + c] = hr[c];
  if (tid == 0) bulk_wait_all();
  if (*abort_flag && tid == 0) {  // let copies in flight land before the CTA exits
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, TCOLS);
  pc.done();
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

// NH = 2: the value columns split over two CTAs per (batch, head), as in the forward.
template <int NH>
__global__ void __launch_bounds__(B1_THREADS, 1) gdn_state_bwd_tc(
    const __grid_constant__ CUtensorMap tm_do, const unsigned char* __restrict__ wt_t,
    const unsigned char* __restrict__ qg_t, const unsigned char* __restrict__ kg_t,
    const unsigned char* __restrict__ aqk_t, const float* __restrict__ gcl, float scale, int L, int H, int NC,
    const float* __restrict__ dh_final, unsigned char* __restrict__ dh_store, unsigned char* __restrict__ dvn_store,
    float* __restrict__ dh0, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + B1_BARS);  // full[2], mma1, mma2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const uint32_t sDH = smem_u32(smem + B1_DH), sDVN = smem_u32(smem + B1_DVN);
  PhaseClock pc(48);

  constexpr int DV = D / NH;  // value columns of this CTA
  constexpr uint32_t TCOLS = NH == 1 ? 512 : 256;
  // TMEM: DVN [0, DV), D1 [DV, 2 DV), D2 [2 DV, 3 DV)
  const int h = blockIdx.x, b = blockIdx.y, v0 = DV * (int)blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = (int64_t)b * H + h;
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) sm100::mbar_init(bars + i, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tm_do);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, TCOLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto issue = [&](int n, int s) {
    unsigned char* st = smem + s * B1_STAGE;
    const int64_t c = bh * NC + n;
    sm100::mbar_expect_tx(bars + s, B1_STAGE - (NH == 2 ? TILE_CD / 2 : 0));
    bulk_g2s(st, wt_t + c * TILE_CD, TILE_CD, bars + s);
    bulk_g2s(st + TILE_CD, qg_t + c * TILE_CD, TILE_CD, bars + s);
    bulk_g2s(st + 2 * TILE_CD, kg_t + c * TILE_CD, TILE_CD, bars + s);
    bulk_g2s(st + 3 * TILE_CD, aqk_t + c * TILE_CC, TILE_CC, bars + s);
    const int row = b * L + n * C;
    tma_load_3d(st + B1_DO, &tm_do, bars + s, v0, h, row);  // this CTA's 64-column box(es) of do
    if (NH == 1) tma_load_3d(st + B1_DO + TILE_CD / 2, &tm_do, bars + s, 64, h, row);
  };
  if (tid == 0) {
    issue(NC - 1, 0);
    if (NC > 1) issue(NC - 2, 1);
  }
  const int dk = tid;
  float dr[DV];
#pragma unroll
  for (int c = 0; c < DV; ++c) dr[c] = dh_final ? dh_final[(bh * D + dk) * D + v0 + c] : 0.f;

  constexpr uint32_t ID_RR = sm100::idesc_bf16(64, DV, true, true);    // rows i x dv, A = Aqk^T (MN)
  constexpr uint32_t ID_RK = sm100::idesc_bf16(64, DV, false, true);   // rows i x dv, A = kg (K-major)
  constexpr uint32_t ID_ST = sm100::idesc_bf16(128, DV, true, true);   // dk x dv
  int it = 0;
  for (; it < NC; ++it) {
    const int n = NC - 1 - it, s = it & 1;
    const int64_t cbn = bh * NC + n;
    const uint32_t st = smem_u32(smem + s * B1_STAGE);
#pragma unroll
    for (int c = 0; c < DV; c += 8) {
      st_chunk8(sDH + sw_off16(D, dk, c), dr + c);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(0);
    if (tid == 0) {  // the dh tile image: this CTA's column half (or both) as one bulk store
      bulk_s2g(dh_store + cbn * (2 * TILE_CD) + (v0 >> 6) * (D * 128), smem + B1_DH, DV * D * 2);
      bulk_commit();
      if (!wait_bar(bars + s, (it >> 1) & 1, err, 0x4721)) *abort_flag = 1;
      pc.mark(6);
      sm100::tc_fence_after();
      if (!*abort_flag) {
        const uint32_t sdo = st + B1_DO;
        auto fdo = [&](int k) { return mndesc(sdo, C, k); };
        mma_steps(tmem, [&](int k) { return mndesc(st + 3 * TILE_CD, C, k); }, fdo, C / 16, ID_RR, false);
        mma_steps(tmem, [&](int k) { return kdesc(st + 2 * TILE_CD, C, k); }, [&](int k) { return mndesc(sDH, D, k); },
                  D / 16, ID_RK, true);
        mma_steps(tmem + DV, [&](int k) { return mndesc(st + TILE_CD, C, k); }, fdo, C / 16, ID_ST, false);
      }
      sm100::umma_commit(bars + 2);
    }
    if (!wait_bar(bars + 2, it & 1, err, 0x4722)) *abort_flag = 1;
    sm100::tc_fence_after();
    pc.mark(1);
    {  // dv_new rows i = 16 warp + (lane & 15); lanes 16-31 take the upper 16 columns by shuffle
      const int i = 16 * warp + (lane & 15), hf = lane >> 4;
#pragma unroll 1
      for (int p = 0; p < DV / 32; ++p) {
        float x[32], xs[16];
        tmem_ld32(tmem_at(tmem, warp, 32 * p), x);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, x[16 + e], lane & 15);
          xs[e] = hf ? sh : x[e];
        }
#pragma unroll
        for (int c = 0; c < 16; c += 8) st_chunk8(sDVN + sw_off16(C, i, 32 * p + 16 * hf + c), xs + c);
      }
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(2);
    if (*abort_flag) break;
    if (tid == 0) {
      bulk_s2g(dvn_store + cbn * TILE_CD + (v0 >> 6) * (C * 128), smem + B1_DVN, DV * C * 2);
      bulk_commit();
      sm100::tc_fence_after();
      mma_steps(tmem + 2 * DV, [&](int k) { return mndesc(st, C, k); }, [&](int k) { return mndesc(sDVN, C, k); },
                C / 16, ID_ST, false);
      sm100::umma_commit(bars + 3);
    }
    if (!wait_bar(bars + 3, it & 1, err, 0x4723)) *abort_flag = 1;
    sm100::tc_fence_after();
    pc.mark(3);
    {
      const float eg = __expf(gcl[cbn * D + dk]);
#pragma unroll
      for (int p = 0; p < DV / 32; ++p) {
        float x1[32], x2[32];
        tmem_ld32(tmem_at(tmem, warp, DV + 32 * p), x1);
        tmem_ld32(tmem_at(tmem, warp, 2 * DV + 32 * p), x2);
#pragma unroll
        for (int e = 0; e < 32; ++e) dr[32 * p + e] = eg * dr[32 * p + e] + scale * x1[e] - x2[e];
      }
    }
    if (tid == 0) bulk_wait_read();  // the dh / dv_new tiles are rewritten in the next step
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(5);
    if (*abort_flag) break;
    if (tid == 0 && it + 2 < NC) issue(n - 2, s);
  }
  if (dh0 && it == NC)
#pragma unroll
    for (int c = 0; c < DV; ++c) dh0[(bh * D + dk) * D + v0 + c] = dr[c];
  if (tid == 0) bulk_wait_all();
  if (*abort_flag && tid == 0) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, TCOLS);
  pc.done();
}

// Row i of an M = 64 accumulator (TMEM columns [col0, col0 + 64)) -> bf16 row i + row_off of a
// 128B-swizzled tile of R rows, on all 256 threads: row i = 16 quarter + (lane & 15) sits in lane
// i & 15 of its lane quarter, so four threads share a row (warpgroup wg takes columns
// [32 wg, 32 wg + 32), lanes 16-31 the upper 16 of them by shuffle).  MODE gives the stored value:
// 0 causal (j <= i), 1 strictly lower (j < i), 2 all, 3 negated strictly lower; with `gt` the row is
// also stored transposed, as column i of rows t_row + j of a tile of Rt rows.  Not inlined: its
// registers stay out of the caller's.
template <int MODE>
__device__ __noinline__ void rows64_out(uint32_t tmem, int col0, int quarter, int wg, int lane, uint32_t dst, int R,
                                        int row_off, unsigned char* gt, int Rt, int t_row) {
  const int hf = lane >> 4, i = 16 * quarter + (lane & 15), j0 = 32 * wg + 16 * hf;
  float x[32], y[16];
  tmem_ld32(tmem_at(tmem, quarter, col0 + 32 * wg), x);
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float sh = __shfl_sync(0xffffffffu, x[16 + e], lane & 15);
    const float v = hf ? sh : x[e];
    const int j = j0 + e;
    y[e] = MODE == 0 ? (j <= i ? v : 0.f) : MODE == 1 ? (j < i ? v : 0.f) : MODE == 2 ? v : (j < i ? -v : 0.f);
  }
  st_chunk8(dst + sw_off16(R, row_off + i, j0), y);
  st_chunk8(dst + sw_off16(R, row_off + i, j0 + 8), y + 8);
  if (gt)
#pragma unroll
    for (int e = 0; e < 16; ++e)
      *reinterpret_cast<bf16*>(gt + sw_off(Rt, t_row + j0 + e, i)) = __float2bfloat16_rn(y[e]);
}

// ============================================================ chunk-parallel backward
// One CTA per chunk, 256 threads.  Everything per (row i, channel d) is held transposed: the
// M = 128 accumulators have the channel as TMEM lane, so thread d assembles channel d of the
// chunk and runs the reverse cumulative sum of dg down its own column.
// Reference B2-B5 (`atomic_ops/kernel_bwd_b2_dav.py:17-51`, `kernel_bwd_b3_wy_dqkg.py:33-148`,
// `kernel_bwd_b4_intra.py:57-165`, `kernel_bwd_b5_reverse_cumsum.py:17-24`).
//   states:  P1 = h do^T, P2 = dh' vn^T, P3 = h dvn^T   ([dk][i], M = 128)
//            Gqk = do vn^T (causal)                     ([i][j], M = 64)
//   WY:      dA = dvn (w v)^T + dw~ (bk e^gc)^T, dw~ = -P3^T (strictly lower)
//            d(wv)^T = dvn^T A, dbke^T = dw~^T A        ([d][j], M = 128) -> dv, dw
//            T = dA A^T, Gkk = -(A^T T) (strictly lower)
//   intra:   row side per reference block I (r = 16 I): dq_b, dbk_b for the rows of block I
//              [d][i] += (k e^{gc_r - gc})[j][d] G[i][j]      then x e^{gc_i - gc_r}
//            column side per key block J (s = 16 J + 15): dk_b for the columns of block J
//              [d][j] += (x e^{gc - gc_s})[i][d] G^T[j][i]    then x e^{gc_s - gc_j}
//            (diagonal blocks with a 16-row decay span > 60: exact per-channel sums instead)
//   assembly: dq, dk, db, dgc; dg = reverse cumsum of dgc (+ dgcl at the last row)
// Exact per-channel sums of a diagonal 16 x 16 block of the intra backward (channel d, row /
// column i of block [i0, i0 + 16)), exponent floored at -20 as in the reference; used only for
// blocks whose decay span is too wide for the factorised products.
__device__ __noinline__ void bc_exact_diag(const unsigned char* G, const float* GC, const bf16* q, const bf16* k,
                                           const bf16* bg, SeqIdx ix, int b, int64_t t0, int h, int d, int i0,
                                           int i, float scale, float& dq_b, float& dbk_b, float& dk_b) {
  const float gci = GC[i * D + d];
  for (int j = i0; j <= i; ++j) {
    const int64_t gj = ix.row(b, t0 + j, h) + d;
    const float e = __expf(fmaxf(gci - GC[j * D + d], -20.f));
    const float kj = __bfloat162float(k[gj]);
    dq_b += scale * __bfloat162float(*reinterpret_cast<const bf16*>(G + sw_off(128, i, j))) * kj * e;
    if (j < i) dbk_b += __bfloat162float(*reinterpret_cast<const bf16*>(G + sw_off(128, C + i, j))) * kj * e;
  }
  for (int i2 = i; i2 < i0 + 16; ++i2) {
    const int64_t g2 = ix.row(b, t0 + i2, h) + d;
    const float e = __expf(fmaxf(GC[i2 * D + d] - gci, -20.f));
    float t = scale * __bfloat162float(*reinterpret_cast<const bf16*>(G + sw_off(128, i2, i))) *
              __bfloat162float(q[g2]);
    if (i2 > i)
      t += __bfloat162float(*reinterpret_cast<const bf16*>(G + sw_off(128, C + i2, i))) *
           __bfloat162float(bg[g2]) * __bfloat162float(k[g2]);
    dk_b += t * e;
  }
}

constexpr int BC_THREADS = 256;
constexpr int BC_H = 0, BC_DH = 32768, BC_DO = 65536, BC_VN = 81920, BC_DVN = 98304, BC_AT = 114688;
constexpr int BC_GC = 122880;  // fp32 [64][128]
constexpr int BC_BAR = BC_GC + 32768;
// reuse after the state products: WV @0, BKE @16K, DWT (rows dk, columns i) @32K, DA @48K, T @56K,
// G (rows: Gqk i, then Gkk i; columns j) @64K, GT (rows: Gqk^T j, then Gkk^T j) @80K;
// row-side key operands @0 / @16K; column-side operands (q part, bk part) @0+16K / @32K+48K
constexpr int BC_WV = 0, BC_BKE = 16384, BC_DWT = 32768, BC_DA = 49152, BC_T = 57344, BC_G = 65536, BC_GT = 81920;
// assembly: plain q, k, b rows over the dead column-side buffer 1 and the dv_new tile
constexpr int BC_QP = 32768, BC_KP = 49152, BC_BP = 98304;
// intra-chunk operand regions: row block I (16 (I + 1) rows) at bc_row_off(I) in [0, 40K); column
// block J (64 - 16 J rows; part 0 = q, 1 = b k) at bc_col_off(J, part): blocks 0 and 3 in the free
// [40K, 64K) and [96K, 120K), blocks 1 and 2 over the row blocks once their MMAs are done
AHB_DEVICE int bc_row_off(int I) { return I == 0 ? 0 : (I == 1 ? 4096 : (I == 2 ? 12288 : 24576)); }
AHB_DEVICE int bc_col_off(int J, int part) {
  if (J == 0) return part ? 98304 : 40960;
  if (J == 3) return part ? 114688 : 57344;
  if (J == 1) return part ? 12288 : 0;
  return part ? 32768 : 24576;
}
constexpr size_t BC_SMEM = 1024 + BC_BAR + 512;

__global__ void __launch_bounds__(BC_THREADS, 1) gdn_chunk_bwd_tc(
    const __grid_constant__ CUtensorMap tm_do, const bf16* __restrict__ q, const bf16* __restrict__ k,
    const bf16* __restrict__ v, const float* __restrict__ g, const bf16* __restrict__ bg,
    const bf16* __restrict__ wgate, const unsigned char* __restrict__ hs_t, const unsigned char* __restrict__ dhs_t,
    const unsigned char* __restrict__ vn_t, const unsigned char* __restrict__ dvn_t,
    const unsigned char* __restrict__ at_t, float scale, int L, int H, bf16* __restrict__ dq_o,
    bf16* __restrict__ dk_o, bf16* __restrict__ dv_o, bf16* __restrict__ db_o, bf16* __restrict__ dw_o,
    float* __restrict__ dg_o, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t S = smem_u32(smem);
  float* GC = reinterpret_cast<float*>(smem + BC_GC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BC_BAR);  // 0 load, 1 states, 2 WY, 3 T, 4 Gkk, 5 rows, 6-7 columns
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);          // [0..3] exact diagonal block, [4] abort
  float* span_w = reinterpret_cast<float*>(flags + 8);         // [4][4]
  float* dgcl_s = span_w + 16;                                 // [128]
  float* tail_s = dgcl_s + 128;                                // [128] reverse-sum hand-over between warpgroups
  PhaseClock pc(16);

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quarter = warp & 3, wg = warp >> 2;
  const SeqIdx ix{L, H};
  const int64_t t0 = (int64_t)n * C;
  const int64_t cb = ((int64_t)b * H + h) * NC + n;

  if (tid == 0) {
    for (int i = 0; i < 13; ++i) sm100::mbar_init(bars + i, 1);
    flags[4] = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tm_do);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    sm100::mbar_expect_tx(bars, 2 * (2 * TILE_CD) + 3 * TILE_CD + TILE_CC);
    bulk_g2s(smem + BC_H, hs_t + cb * (2 * TILE_CD), 2 * TILE_CD, bars);
    bulk_g2s(smem + BC_DH, dhs_t + cb * (2 * TILE_CD), 2 * TILE_CD, bars);
    bulk_g2s(smem + BC_VN, vn_t + cb * TILE_CD, TILE_CD, bars);
    bulk_g2s(smem + BC_DVN, dvn_t + cb * TILE_CD, TILE_CD, bars);
    bulk_g2s(smem + BC_AT, at_t + cb * TILE_CC, TILE_CC, bars);
    tma_load_3d(smem + BC_DO, &tm_do, bars, 0, h, (int)(b * L + t0));
    tma_load_3d(smem + BC_DO + TILE_CD / 2, &tm_do, bars, 64, h, (int)(b * L + t0));
  }
  // this thread's 16-byte units of the chunk's q, k, b, w, v rows (unit it: row 16 it + tid / 16,
  // columns 8 (tid % 16) ..), requested up front and kept in registers for every later use
  constexpr int BU = (C * D / 8) / BC_THREADS;
  uint4 qa[BU], ka[BU], ba[BU], wa[BU], va[BU];
#pragma unroll
  for (int it = 0; it < BU; ++it) {
    const int64_t gi = ix.row(b, t0 + 16 * it + (tid >> 4), h) + ((tid & 15) << 3);
    qa[it] = *reinterpret_cast<const uint4*>(q + gi);
    ka[it] = *reinterpret_cast<const uint4*>(k + gi);
    ba[it] = *reinterpret_cast<const uint4*>(bg + gi);
    wa[it] = *reinterpret_cast<const uint4*>(wgate + gi);
    va[it] = *reinterpret_cast<const uint4*>(v + gi);
  }
#pragma unroll
  for (int e = tid; e < C * (D / 4); e += BC_THREADS) {
    const int r = e >> 5, c4 = (e & 31) << 2;
    cp_async16(GC + r * D + c4, g + ix.row(b, t0 + r, h) + c4);  // no registers held for the gate rows
  }
  cp_async_wait_all();
  __syncthreads();
  if (!wait_bar(bars, 0, err, 0x4731)) flags[4] = 1;
  pc.mark(0);
  // state products (one thread issues; the others scan g meanwhile)
  if (tid == 0 && !flags[4]) {
    sm100::tc_fence_after();
    constexpr uint32_t ID_P = sm100::idesc_bf16(128, 64, false, false);
    constexpr uint32_t ID_G = sm100::idesc_bf16(64, 64, false, false);
    auto fh = [&](int s) { return kdesc(S + BC_H, D, s); };
    mma_steps(tmem + 0, fh, [&](int s) { return kdesc(S + BC_DO, C, s); }, D / 16, ID_P, false);
    mma_steps(tmem + 64, [&](int s) { return kdesc(S + BC_DH, D, s); }, [&](int s) { return kdesc(S + BC_VN, C, s); },
              D / 16, ID_P, false);
    mma_steps(tmem + 128, fh, [&](int s) { return kdesc(S + BC_DVN, C, s); }, D / 16, ID_P, false);
    mma_steps(tmem + 192, [&](int s) { return kdesc(S + BC_DO, C, s); }, [&](int s) { return kdesc(S + BC_VN, C, s); },
              D / 16, ID_G, false);
    sm100::umma_commit(bars + 1);
  }
  if (tid < D) {
    const int d = tid;
    float s = 0.f;
    for (int r = 0; r < C; ++r) {
      s += GC[r * D + d];
      GC[r * D + d] = s;
    }
    float sp[4];
#pragma unroll
    for (int I = 0; I < 4; ++I) sp[I] = warp_max(GC[16 * I * D + d] - GC[(16 * I + 15) * D + d]);
    if (lane == 0)
#pragma unroll
      for (int I = 0; I < 4; ++I) span_w[warp * 4 + I] = sp[I];
    // e^{gcl} sum_dv dh'[d][dv] h[d][dv] (state rows d of the two tile images)
    float acc = 0.f;
#pragma unroll 4
    for (int c = 0; c < D; c += 8) {
      float a8[8], b8[8];
      unpack8(*reinterpret_cast<const uint4*>(smem + BC_H + sw_off16(D, d, c)), a8);
      unpack8(*reinterpret_cast<const uint4*>(smem + BC_DH + sw_off16(D, d, c)), b8);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += a8[e] * b8[e];
    }
    dgcl_s[d] = __expf(s) * acc;
  }
  __syncthreads();
  if (tid < 4) {
    const float m = fmaxf(fmaxf(span_w[tid], span_w[4 + tid]), fmaxf(span_w[8 + tid], span_w[12 + tid]));
    flags[tid] = !(m <= 60.f);
  }
  if (!wait_bar(bars + 1, 0, err, 0x4732)) flags[4] = 1;
  pc.mark(1);
  sm100::tc_fence_after();
  // WV = w v and BKE = (b k) e^gc over the dead state tiles; the H region is free once the
  // state products completed
#pragma unroll
  for (int it = 0; it < BU; ++it) {
    const int i = 16 * it + (tid >> 4), c = (tid & 15) << 3;
    float kv[8], bv[8], wv[8], vv[8], x[8], y[8];
    unpack8(ka[it], kv);
    unpack8(ba[it], bv);
    unpack8(wa[it], wv);
    unpack8(va[it], vv);
    float gci[8];
    ld8f_x(GC + i * D + c, gci);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x[e] = wv[e] * vv[e];
      y[e] = bv[e] * kv[e] * __expf(gci[e]);
    }
    st_chunk8(S + BC_WV + sw_off16(C, i, c), x);
    st_chunk8(S + BC_BKE + sw_off16(C, i, c), y);
  }
  // dw~^T = -P3 -> DWT tile (rows dk, columns i); warpgroup wg takes columns [32 wg, 32 wg + 32)
  {
    const int dk = 32 * quarter + lane;
    float x[32];
    tmem_ld32(tmem_at(tmem, quarter, 128 + 32 * wg), x);
#pragma unroll
    for (int c = 0; c < 32; ++c) x[c] = -x[c];
#pragma unroll
    for (int c = 0; c < 32; c += 8) st_chunk8(S + BC_DWT + sw_off16(D, dk, 32 * wg + c), x + c);
  }
  // Gqk = do vn^T (causal) -> rows 0-63 of G and G^T
  rows64_out<0>(tmem, 192, quarter, wg, lane, S + BC_G, 128, 0, smem + BC_GT, 128, 0);
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  pc.mark(2);
  if (flags[4]) goto bc_teardown;
  // WY products: dA (M = 64) -> [256, 320); d(wv)^T -> [320, 384); dbke^T -> [384, 448)
  if (tid == 0) {
    sm100::tc_fence_after();
    mma_steps(tmem + 256, [&](int s) { return kdesc(S + BC_DVN, C, s); }, [&](int s) { return kdesc(S + BC_WV, C, s); },
              D / 16, sm100::idesc_bf16(64, 64, false, false), false);
    mma_steps(tmem + 256, [&](int s) { return mndesc(S + BC_DWT, D, s); }, [&](int s) { return kdesc(S + BC_BKE, C, s); },
              D / 16, sm100::idesc_bf16(64, 64, true, false), true);
    auto fat = [&](int s) { return mndesc(S + BC_AT, C, s); };
    mma_steps(tmem + 320, [&](int s) { return mndesc(S + BC_DVN, C, s); }, fat, C / 16,
              sm100::idesc_bf16(128, 64, true, true), false);
    mma_steps(tmem + 384, [&](int s) { return kdesc(S + BC_DWT, D, s); }, fat, C / 16,
              sm100::idesc_bf16(128, 64, false, true), false);
    sm100::umma_commit(bars + 2);
  }
  if (!wait_bar(bars + 2, 0, err, 0x4733)) flags[4] = 1;
  pc.mark(3);
  sm100::tc_fence_after();
  // dA strictly lower -> DA tile (rows i, columns l)
  rows64_out<1>(tmem, 256, quarter, wg, lane, S + BC_DA, C, 0, nullptr, 0, 0);
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  pc.mark(4);
  if (tid == 0 && !flags[4]) {
    sm100::tc_fence_after();
    mma_steps(tmem + 448, [&](int s) { return kdesc(S + BC_DA, C, s); }, [&](int s) { return kdesc(S + BC_AT, C, s); },
              C / 16, sm100::idesc_bf16(64, 64, false, false), false);
    sm100::umma_commit(bars + 3);
  }
  // dv, dw from d(wv)^T (lane = channel d, column j): transposed through shared memory (fp32 rows
  // j over the dead (w v | bke) tiles), then row units times the held v / w rows
  {
    const int d = 32 * quarter + lane;
    float* DWV = reinterpret_cast<float*>(smem + BC_WV);
    float x[32];
    tmem_ld32(tmem_at(tmem, quarter, 320 + 32 * wg), x);
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) DWV[(32 * wg + jj) * D + d] = x[jj];
    __syncthreads();
#pragma unroll
    for (int it = 0; it < BU; ++it) {
      const int j = 16 * it + (tid >> 4), c = (tid & 15) << 3;
      float vv[8], ww[8], y[8], z[8];
      unpack8(va[it], vv);
      unpack8(wa[it], ww);
      const float4 a0 = *reinterpret_cast<const float4*>(DWV + j * D + c);
      const float4 a1 = *reinterpret_cast<const float4*>(DWV + j * D + c + 4);
      const float xx[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        y[e] = xx[e] * vv[e];
        z[e] = xx[e] * ww[e];
      }
      const int64_t gi = ix.row(b, t0 + j, h) + c;
      *reinterpret_cast<uint4*>(dw_o + gi) = pack8(y);
      *reinterpret_cast<uint4*>(dv_o + gi) = pack8(z);
    }
  }
  pc.mark(5);
  if (!wait_bar(bars + 3, 0, err, 0x4734)) flags[4] = 1;
  sm100::tc_fence_after();
  // T = dA A^T -> T tile (rows l, columns j)
  rows64_out<2>(tmem, 448, quarter, wg, lane, S + BC_T, C, 0, nullptr, 0, 0);
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0 && !flags[4]) {
    sm100::tc_fence_after();
    mma_steps(tmem + 256, [&](int s) { return mndesc(S + BC_AT, C, s); }, [&](int s) { return mndesc(S + BC_T, C, s); },
              C / 16, sm100::idesc_bf16(64, 64, true, true), false);
    sm100::umma_commit(bars + 4);
  }
  if (!wait_bar(bars + 4, 0, err, 0x4735)) flags[4] = 1;
  pc.mark(6);
  sm100::tc_fence_after();
  // Gkk = -(A^T T) strictly lower -> rows 64-127 of G and G^T
  rows64_out<3>(tmem, 256, quarter, wg, lane, S + BC_G, 128, C, smem + BC_GT, 128, C);
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  pc.mark(7);
  if (flags[4]) goto bc_teardown;
  // intra, row side: per reference block I, key operand (k e^{gc_r - gc})[j][d] for j <= 16 I + 15
  // (16 (I + 1) rows at [0, 40K): offsets 0, 4K, 12K, 24K); dq_b -> TMEM [128 + 32 I, +16),
  // dbk_b -> [144 + 32 I, +16) (lane d, column i - 16 I).  All four blocks in one pass.
  {
    float ob[10][8];  // the ten units' operands, stored after all their gate loads
#pragma unroll
    for (int I = 0; I < 4; ++I) {
      const bool exact = flags[I];
      const float* gcr = GC + 16 * I * D;
#pragma unroll
      for (int it = 0; it <= I; ++it) {
        const int j = 16 * it + (tid >> 4), c = (tid & 15) << 3;
        float kv[8];
        unpack8(ka[it], kv);
        const bool zero = exact && j >= 16 * I;
        float gcj[8], gr8[8];
        ld8f_x(GC + j * D + c, gcj);
        ld8f_x(gcr + c, gr8);
#pragma unroll
        for (int e = 0; e < 8; ++e) ob[I * (I + 1) / 2 + it][e] = zero ? 0.f : kv[e] * __expf(gr8[e] - gcj[e]);
      }
    }
#pragma unroll
    for (int I = 0; I < 4; ++I)
#pragma unroll
      for (int it = 0; it <= I; ++it)
        st_chunk8(S + bc_row_off(I) + sw_off16(16 * (I + 1), 16 * it + (tid >> 4), (tid & 15) << 3),
                  ob[I * (I + 1) / 2 + it]);
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    sm100::tc_fence_after();
    constexpr uint32_t ID_R = sm100::idesc_bf16(128, 16, true, false);
#pragma unroll
    for (int I = 0; I < 4; ++I) {
      const uint32_t buf = S + bc_row_off(I);
      auto fa = [&](int s) { return mndesc(buf, 16 * (I + 1), s); };
      mma_steps(tmem + 128 + 32 * I, fa, [&](int s) { return kdesc(S + BC_G + 2048 * I, 128, s); }, I + 1, ID_R, false);
      mma_steps(tmem + 144 + 32 * I, fa, [&](int s) { return kdesc(S + BC_G + 8192 + 2048 * I, 128, s); }, I + 1, ID_R,
                false);
    }
    sm100::umma_commit(bars + 5);
  }
  // intra, column side: per key block J with reference s = 16 J + 15 (its last row), operands
  // (scale q e^{gc - gc_s}) and ((b k) e^{gc - gc_s}) for rows i >= 16 J (<= 1 below the block),
  // packed to those 64 - 16 J rows; dk_b -> TMEM [448 + 16 J, +16) (lane d, column j - 16 J), later
  // times e^{gc_s - gc_j} <= 1.  Blocks 0 and 3 go to the free [40K, 64K) and [96K, 120K) while the
  // row-side MMAs run, blocks 1 and 2 to the row-side buffers once those MMAs are done.
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && !wait_bar(bars + 5, 0, err, 0x4737)) flags[4] = 1;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int J = pass == 0 ? 3 * jj : 1 + jj;
      const int R = 64 - 16 * J;
      const uint32_t bq = S + bc_col_off(J, 0), bk2 = S + bc_col_off(J, 1);
      const bool exact = flags[J];
      const float* gcr = GC + (16 * J + 15) * D;
#pragma unroll
      for (int it = J; it < BU; ++it) {
        const int i = 16 * it + (tid >> 4), c = (tid & 15) << 3;
        float qv[8], kv[8], bv[8], xq[8], xk[8];
        unpack8(qa[it], qv);
        unpack8(ka[it], kv);
        unpack8(ba[it], bv);
        const bool zero = exact && i < 16 * J + 16;
        float gci[8], gr8[8];
        ld8f_x(GC + i * D + c, gci);
        ld8f_x(gcr + c, gr8);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float er = zero ? 0.f : __expf(gci[e] - gr8[e]);
          xq[e] = scale * qv[e] * er;
          xk[e] = bv[e] * kv[e] * er;
        }
        st_chunk8(bq + sw_off16(R, i - 16 * J, c), xq);
        st_chunk8(bk2 + sw_off16(R, i - 16 * J, c), xk);
      }
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0 && !flags[4]) {
      sm100::tc_fence_after();
      constexpr uint32_t ID_C = sm100::idesc_bf16(128, 16, true, false);
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int J = pass == 0 ? 3 * jj : 1 + jj;
        const int R = 64 - 16 * J;
        // descriptor bases shifted down by J K-steps: K step s (rows 16 s ..) sits at 2048 (s - J)
        const uint32_t bq = S + bc_col_off(J, 0) - 2048 * J, bk2 = S + bc_col_off(J, 1) - 2048 * J;
        const uint32_t dcol = tmem + 448 + 16 * J;
        for (int s = J; s < 4; ++s)
          sm100::umma_bf16(dcol, mndesc(bq, R, s), kdesc(S + BC_GT + 2048 * J, 128, s), ID_C, s > J ? 1u : 0u);
        for (int s = J; s < 4; ++s)
          sm100::umma_bf16(dcol, mndesc(bk2, R, s), kdesc(S + BC_GT + 8192 + 2048 * J, 128, s), ID_C, 1u);
      }
      sm100::umma_commit(bars + 6 + pass);
    }
  }
  pc.mark(8);
  if (!wait_bar(bars + 6, 0, err, 0x4739) || !wait_bar(bars + 7, 0, err, 0x4739)) flags[4] = 1;
  pc.mark(9);
  sm100::tc_fence_after();
  // plain row-major q, k, b tiles (256-byte rows) for the per-channel assembly reads
#pragma unroll
  for (int it = 0; it < BU; ++it) {
    const int off = (16 * it + (tid >> 4)) * 256 + ((tid & 15) << 4);
    *reinterpret_cast<uint4*>(smem + BC_QP + off) = qa[it];
    *reinterpret_cast<uint4*>(smem + BC_KP + off) = ka[it];
    *reinterpret_cast<uint4*>(smem + BC_BP + off) = ba[it];
  }
  __syncthreads();
  pc.mark(10);
  if (flags[4]) goto bc_teardown;
  {
    // assembly: thread d = channel, warpgroup wg = rows [32 wg, 32 wg + 32), one 16-row block at a time
    const int d = 32 * quarter + lane;
    float* DGC = reinterpret_cast<float*>(smem);  // dgc rows (the operand buffers are dead)
    const unsigned char* G = smem + BC_G;
    const float gcl = GC[(C - 1) * D + d];
    float dgcl_part = 0.f;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      const int I = 2 * wg + half, i0 = 16 * I;
      float p1[16], p2[16], w3[16], rq[16], rk[16], ck[16];
      tmem_ld16(tmem_at(tmem, quarter, i0), p1);
      tmem_ld16(tmem_at(tmem, quarter, 64 + i0), p2);
      tmem_ld16(tmem_at(tmem, quarter, 384 + i0), w3);
      tmem_ld16(tmem_at(tmem, quarter, 128 + 32 * I), rq);
      tmem_ld16(tmem_at(tmem, quarter, 144 + 32 * I), rk);
      tmem_ld16(tmem_at(tmem, quarter, 448 + i0), ck);
      const float gr = GC[i0 * D + d], gs = GC[(i0 + 15) * D + d];
      const bool exact = flags[I];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int i = i0 + r;
        const int64_t gi = ix.row(b, t0 + i, h) + d;
        const int po = i * 256 + 2 * d;
        const float qi = __bfloat162float(*reinterpret_cast<const bf16*>(smem + BC_QP + po));
        const float ki = __bfloat162float(*reinterpret_cast<const bf16*>(smem + BC_KP + po));
        const float bi = __bfloat162float(*reinterpret_cast<const bf16*>(smem + BC_BP + po));
        const float gci = GC[i * D + d];
        float dq_b = scale * __expf(gci - gr) * rq[r];
        float dbk_b = __expf(gci - gr) * rk[r];
        float dk_b = __expf(gs - gci) * ck[r];
        if (exact) bc_exact_diag(G, GC, q, k, bg, ix, b, t0, h, d, i0, i, scale, dq_b, dbk_b, dk_b);
        const float eg = __expf(gci), el = __expf(gcl - gci);
        const float dq_a = scale * p1[r] * eg, dk_a = p2[r] * el, dbk_wy = w3[r] * eg;
        const float bki = bi * ki;
        const float dbk = dbk_wy + dbk_b;
        dq_o[gi] = __float2bfloat16_rn(dq_a + dq_b);
        dk_o[gi] = __float2bfloat16_rn(dk_a + dk_b + dbk * bi);
        db_o[gi] = __float2bfloat16_rn(dbk * ki);
        DGC[i * D + d] = dq_a * qi - dk_a * ki + dbk_wy * bki + qi * dq_b + bki * dbk_b - ki * dk_b;
        dgcl_part += dk_a * ki;
      }
    }
    // dg = dgcl + reverse cumulative sum of dgc; rows 32-63 (warpgroup 1) hand their total to rows 0-31
    float dv32[32], tot = 0.f;  // this thread's 32 rows, loaded before the stores below
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      dv32[r] = DGC[(32 * wg + r) * D + d];
      tot += dv32[r];
    }
    if (wg == 1) {
      tail_s[d] = tot;
      dgcl_s[d] += dgcl_part;  // after the first barrier below warpgroup 0 adds its own part
    }
    __syncthreads();
    if (wg == 0) dgcl_s[d] += dgcl_part;
    __syncthreads();
    float run = dgcl_s[d] + (wg == 0 ? tail_s[d] : 0.f);
#pragma unroll
    for (int r = 31; r >= 0; --r) {
      const int i = 32 * wg + r;
      run += dv32[r];
      dg_o[ix.row(b, t0 + i, h) + d] = run;
    }
  }
bc_teardown:
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  pc.mark(11);
  if (warp == 0) sm100::tmem_dealloc(tmem, 512);
  pc.done();
}

template <class K>
int set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess ? 0 : -3;
}

}  // namespace

// ===================================================================== launchers
AHB_PHASE_PROF_SETTER(ahb_gdn_phase_prof)

int ahb_gdn_chunk_fwd_tc(const void* q, const void* k, const void* v, const float* g, const void* bg, const void* wg,
                         float scale, int B, int L, int H, void* wt_t, void* u_t, void* qg_t, void* kg_t, void* aqk_t,
                         float* gcl, void* at_t, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_chunk_fwd_tc, F1_SMEM);
  if (init) return init;
  gdn_chunk_fwd_tc<<<dim3(L / C, H, B), F1_THREADS, F1_SMEM, st>>>(
      (const bf16*)q, (const bf16*)k, (const bf16*)v, g, (const bf16*)bg, (const bf16*)wg, scale, L, H,
      (unsigned char*)wt_t, (unsigned char*)u_t, (unsigned char*)qg_t, (unsigned char*)kg_t, (unsigned char*)aqk_t,
      gcl, (unsigned char*)at_t, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// the value columns split over two CTAs when the (batch, head) pairs fill at most half the SMs
static bool gdn_state_split(int B, int H) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return 2 * B * H <= sms;
}

int ahb_gdn_state_fwd_tc(const void* wt_t, const void* u_t, const void* qg_t, const void* kg_t, const void* aqk_t,
                         const float* gcl, float scale, int B, int L, int H, const float* h0, void* o, float* h_final,
                         void* h_store, void* vn_store, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_state_fwd_tc<1>, F2_SMEM) | set_smem(gdn_state_fwd_tc<2>, F2_SMEM);
  if (init) return init;
  const bool split = gdn_state_split(B, H);
  CUtensorMap tmo;
  memset(&tmo, 0, sizeof(tmo));
  if (o && tmap_seq_bf16(&tmo, o, (int64_t)B * L, H, D, C)) return -20;
  auto k = split ? gdn_state_fwd_tc<2> : gdn_state_fwd_tc<1>;
  k<<<dim3(H, B, split ? 2 : 1), F2_THREADS, F2_SMEM, st>>>(
      tmo, (const unsigned char*)wt_t, (const unsigned char*)u_t, (const unsigned char*)qg_t, (const unsigned char*)kg_t,
      (const unsigned char*)aqk_t, gcl, scale, L, H, L / C, h0, (bf16*)o, h_final, (unsigned char*)h_store,
      (unsigned char*)vn_store, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
int ahb_gdn_state_bwd_tc(const void* wt_t, const void* qg_t, const void* kg_t, const void* aqk_t, const float* gcl,
                         const void* dout, float scale, int B, int L, int H, const float* dh_final, void* dh_store,
                         void* dvn_store, float* dh0, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_state_bwd_tc<1>, B1_SMEM) | set_smem(gdn_state_bwd_tc<2>, B1_SMEM);
  if (init) return init;
  CUtensorMap tm;
  if (tmap_seq_bf16(&tm, dout, (int64_t)B * L, H, D, C)) return -20;
  const bool split = gdn_state_split(B, H);
  auto k = split ? gdn_state_bwd_tc<2> : gdn_state_bwd_tc<1>;
  k<<<dim3(H, B, split ? 2 : 1), B1_THREADS, B1_SMEM, st>>>(
      tm, (const unsigned char*)wt_t, (const unsigned char*)qg_t, (const unsigned char*)kg_t,
      (const unsigned char*)aqk_t, gcl, scale, L, H, L / C, dh_final, (unsigned char*)dh_store,
      (unsigned char*)dvn_store, dh0, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int ahb_gdn_chunk_bwd_tc(const void* q, const void* k, const void* v, const float* g, const void* bg, const void* wg,
                         const void* dout, const void* hs_t, const void* dhs_t, const void* vn_t, const void* dvn_t,
                         const void* at_t, float scale, int B, int L, int H, void* dq, void* dk, void* dv, void* db,
                         void* dw, float* dg, int* err, cudaStream_t st) {
  static int init = set_smem(gdn_chunk_bwd_tc, BC_SMEM);
  if (init) return init;
  CUtensorMap tm;
  if (tmap_seq_bf16(&tm, dout, (int64_t)B * L, H, D, C)) return -20;
  gdn_chunk_bwd_tc<<<dim3(L / C, H, B), BC_THREADS, BC_SMEM, st>>>(
      tm, (const bf16*)q, (const bf16*)k, (const bf16*)v, g, (const bf16*)bg, (const bf16*)wg,
      (const unsigned char*)hs_t, (const unsigned char*)dhs_t, (const unsigned char*)vn_t, (const unsigned char*)dvn_t,
      (const unsigned char*)at_t, scale, L, H, (bf16*)dq, (bf16*)dk, (bf16*)dv, (bf16*)db, (bf16*)dw, dg, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
