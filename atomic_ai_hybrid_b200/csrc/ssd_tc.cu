// Mamba2 SSD on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// Per (batch, head, chunk of C = 64 steps), head dim P = 64, state N = 128, per-channel dt
// (reference `atomic_ops/mamba2_ssd_reference.py:56-148`, kernels M2-M4 and MB1-MB4):
//   c = clip(cumsum_t clip(dt A, +-20), +-1e4) ; cl = c[C-1] ; dBx = clip(dt x, 1e4)
//   CB[i,j] = clip(C_i . B_j, 1e4)
//   y_diag[i,p] = clip(sum_{j<=i} CB[i,j] e^{c_ip - c_jp} dBx[j,p], 1e4)
//   S_end[p,s]  = clip(sum_j e^{max(cl_p - c_jp, -20)} dBx[j,p] B[j,s], 1e4)
//   y_off[i,p]  = clip(e^{max(c_ip, -20)} sum_s C[i,s] S_in[p,s], 1e4) ; y = clip(y_diag + y_off, 1e4)
//   S_in(next)  = clip(S_in e^{max(cl_p, -20)} + S_end, 1e4)
//
// Forward in two kernels:
//   ssd_chunk_fwd_tc (one CTA per chunk and head, chunk-parallel): C B^T, S_end^T = B^T V
//     (M = 128 state rows) and y_diag^T: the blocks below the diagonal per 16-row reference block
//     (the pairwise decay split at r = 16 I, rows e^{c_i - c_r} <= 1, keys e^{c_r - c_j} <= 1) on
//     the tensor cores, the diagonal 16 x 16 blocks exactly per channel in fp32 (exponent floored
//     at -20 as the reference); writes S_end^T and the decay e^{max(c,-20)} as swizzled
//     tile images, y_diag^T rows (fp32: the backward's decay gradient cancels heavily) and the
//     chunk's last cumsum.
//   ssd_state_fwd_tc (one CTA per batch and head, chunk-sequential): the fp32 state lives in
//     registers (thread s holds S^T row s); per chunk y_off^T = S C^T on the tensor cores, the
//     output y, and (for the backward) the incoming state as a tile image.
// The reverse state-gradient recurrence (ssd_state_bwd_tc) mirrors the second kernel.
#include <cuda.h>
#include <cuda_runtime.h>
#include "common.cuh"
#include "sm100.cuh"
#include "umma.cuh"
#include "tmap.h"
#include "launchers.h"
#include "phase_prof.cuh"

using namespace ahb;
using namespace ahb::umma;
using bf16 = __nv_bfloat16;

namespace {

constexpr int C = 64, P = 64, N = 128;
constexpr int T_CP = C * P * 2;   // 64 x 64 bf16 tile (8 KB)
constexpr int T_CN = C * N * 2;   // 64 x 128 bf16 tile (16 KB)
constexpr int T_NP = N * P * 2;   // 128 x 64 bf16 tile (16 KB)

AHB_DEVICE float clip4(float x) { return sanitize(x, 1e4f); }

// Decay cumsum of the chunk for 256 threads: CUM[i][p] = clamp(sum_{i' <= i} clamp(dt[i'][p] A, +-20),
// +-1e4), four threads per channel p (rows [16 k, 16 k + 16) for k = tid >> 6), the block totals of
// the rows before a block added through `part` (4 x 64 floats of shared memory).  The forward and
// backward chunk kernels both use it, so their cumsums agree bit for bit.  Ends with __syncthreads.
AHB_DEVICE void chunk_cumsum(const unsigned char* dt_tile, float Ah, float* CUM, float* part, int tid) {
  const int p = tid & 63, k = tid >> 6;
  float v[16], s = 0.f;
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const float dtv = __bfloat162float(*reinterpret_cast<const bf16*>(dt_tile + sw_off(C, 16 * k + t, p)));
    s += fminf(fmaxf(dtv * Ah, -20.f), 20.f);
    v[t] = s;
  }
  part[k * 64 + p] = s;
  __syncthreads();
  float off = 0.f;
  for (int k2 = 0; k2 < k; ++k2) off += part[k2 * 64 + p];
#pragma unroll
  for (int t = 0; t < 16; ++t) CUM[(16 * k + t) * P + p] = fminf(fmaxf(off + v[t], -1e4f), 1e4f);
  __syncthreads();
}

// ============================================================ chunk-parallel forward
constexpr int S1_THREADS = 256;
// byte offsets; W (16 KB) holds the y_diag key operands, then the fp32 y_diag rows
constexpr int S1_B = 0, S1_C = 16384, S1_X = 32768, S1_DT = 40960, S1_CB = 49152, S1_V = 57344, S1_W0 = 65536,
              S1_CUM = 81920, S1_BAR = 98304;
constexpr size_t S1_SMEM = 1024 + S1_BAR + 256;

__global__ void __launch_bounds__(S1_THREADS, 2) ssd_chunk_fwd_tc(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dt, const float* __restrict__ A,
    int L, int H, unsigned char* __restrict__ send_t, float* __restrict__ yd_t, unsigned char* __restrict__ dec_t,
    float* __restrict__ cl_o, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t S = smem_u32(smem);
  float* CUM = reinterpret_cast<float*>(smem + S1_CUM);  // [i][p]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S1_BAR);  // 0 load, 1 CB, 2 S_end, 3 y_diag blocks
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [4] abort
  PhaseClock pc(0);

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quarter = warp & 3, wg = warp >> 2;
  const int row0 = b * L + n * C;
  const int64_t ch = ((int64_t)b * H + h) * NC + n;
  if (tid == 0) {
    for (int i = 0; i < 7; ++i) sm100::mbar_init(bars + i, 1);
    flags[4] = 0;
    sm100::fence_barrier_init();
    sm100::mbar_expect_tx(bars, 2 * T_CN + 2 * T_CP);
    sm100::tma_load_2d(smem + S1_B, &tm_b, bars, 0, row0);
    sm100::tma_load_2d(smem + S1_B + T_CN / 2, &tm_b, bars, 64, row0);
    sm100::tma_load_2d(smem + S1_C, &tm_c, bars, 0, row0);
    sm100::tma_load_2d(smem + S1_C + T_CN / 2, &tm_c, bars, 64, row0);
    tma_load_3d(smem + S1_X, &tm_x, bars, 0, h, row0);
    tma_load_3d(smem + S1_DT, &tm_dt, bars, 0, h, row0);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 256);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pc.mark(0);
  if (!wait_bar(bars, 0, err, 0x5301)) flags[4] = 1;
  pc.mark(1);
  if (tid == 0 && !flags[4]) {  // CB = C B^T  (M = 64 rows i, N = 64 keys j)
    sm100::tc_fence_after();
    mma_steps(tmem, [&](int s) { return kdesc(S + S1_C, C, s); }, [&](int s) { return kdesc(S + S1_B, C, s); }, N / 16,
              sm100::idesc_bf16(64, 64, false, false), false);
    sm100::umma_commit(bars + 1);
  }
  const float Ah = A[h];
  // decay cumsum (block totals exchanged in the V buffer, written only after it)
  chunk_cumsum(smem + S1_DT, Ah, CUM, reinterpret_cast<float*>(smem + S1_V), tid);
  if (tid < P) cl_o[ch * P + tid] = CUM[(C - 1) * P + tid];
  // V = dBx e^{max(cl - c, -20)}  (rows j, columns p)
  float vb[(C * P / 8) / S1_THREADS][8];  // stored after the loop (the units' loads come first)
#pragma unroll
  for (int it = 0; it < (C * P / 8) / S1_THREADS; ++it) {
    const int u_ = it * S1_THREADS + tid;
    const int j = u_ >> 3, c = (u_ & 7) << 3;
    float xv[8], dv[8];
    unpack8(*reinterpret_cast<const uint4*>(smem + S1_X + sw_off16(C, j, c)), xv);
    unpack8(*reinterpret_cast<const uint4*>(smem + S1_DT + sw_off16(C, j, c)), dv);
    float cj[8], cl8[8];
    ld8f_x(CUM + j * P + c, cj);
    ld8f_x(CUM + (C - 1) * P + c, cl8);
#pragma unroll
    for (int e = 0; e < 8; ++e) vb[it][e] = clip4(dv[e] * xv[e]) * __expf(fmaxf(cl8[e] - cj[e], -20.f));
  }
#pragma unroll
  for (int it = 0; it < (C * P / 8) / S1_THREADS; ++it) {
    const int u_ = it * S1_THREADS + tid;
    st_chunk8(S + S1_V + sw_off16(C, u_ >> 3, (u_ & 7) << 3), vb[it]);
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0 && !flags[4]) {  // S_end^T = B^T V  (M = 128 state rows s, N = 64 channels p)
    sm100::tc_fence_after();
    mma_steps(tmem + 64, [&](int k) { return mndesc(S + S1_B, C, k); }, [&](int k) { return mndesc(S + S1_V, C, k); },
              C / 16, sm100::idesc_bf16(128, 64, true, true), false);
    sm100::umma_commit(bars + 2);
  }
  pc.mark(2);
  if (!wait_bar(bars + 1, 0, err, 0x5302)) flags[4] = 1;
  sm100::tc_fence_after();
  {  // causal CB -> bf16 K-major tile (rows i, columns j <= i): row i = 16 quarter + (lane & 15) sits
     // in lane i & 15 of the quarter (M = 64); four threads per row, 16 columns each (lanes 16-31
     // take theirs by shuffle)
    const int hf = lane >> 4, i = 16 * quarter + (lane & 15), j0 = 32 * wg + 16 * hf;
    float x[32], y[16];
    tmem_ld32(tmem_at(tmem, quarter, 32 * wg), x);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float sh = __shfl_sync(0xffffffffu, x[16 + e], lane & 15);
      y[e] = hf ? sh : x[e];
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) y[e] = j0 + e <= i ? clip4(y[e]) : 0.f;
    st_chunk8(S + S1_CB + sw_off16(C, i, j0), y);
    st_chunk8(S + S1_CB + sw_off16(C, i, j0 + 8), y + 8);
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  pc.mark(3);
  // y_diag^T per reference block I (r = 16 I): W[j][p] = dBx e^{c_r - c_j} for keys j < 16 I (the
  // diagonal block is summed exactly below, so block 0 has no tensor-core part),
  // D[p][i in block I] += W^T CB^T  -> TMEM columns [128 + 16 I, +16)
  // The key operand is split into bf16 hi + lo parts (two MMAs): the backward's decay gradient
  // cancels these sums against the matching column sums, which bf16 alone would not resolve.
  // Blocks 1-3 are built in one pass (768 units), packed: block I's K steps 0 .. I - 1 (2 KB each)
  // from 0, 2 KB, 6 KB of the hi (W) and lo (dead C tile) regions.
  float hb[768 / S1_THREADS][8], lb[768 / S1_THREADS][8];  // stored after the loop
#pragma unroll
  for (int it = 0; it < 768 / S1_THREADS; ++it) {
    const int u_ = it * S1_THREADS + tid;
    const int I = u_ < 128 ? 1 : (u_ < 384 ? 2 : 3);
    const int lu = u_ - (I == 1 ? 0 : (I == 2 ? 128 : 384));
    const int j = lu >> 3, c = (lu & 7) << 3;
    float xv[8], dv[8];
    float* o = hb[it];
    float* lo = lb[it];
    unpack8(*reinterpret_cast<const uint4*>(smem + S1_X + sw_off16(C, j, c)), xv);
    unpack8(*reinterpret_cast<const uint4*>(smem + S1_DT + sw_off16(C, j, c)), dv);
    float cj[8], cr8[8];
    ld8f_x(CUM + j * P + c, cj);
    ld8f_x(CUM + 16 * I * P + c, cr8);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o[e] = clip4(dv[e] * xv[e]) * __expf(cr8[e] - cj[e]);
      lo[e] = o[e] - __bfloat162float(__float2bfloat16_rn(o[e]));
    }
  }
#pragma unroll
  for (int it = 0; it < 768 / S1_THREADS; ++it) {
    const int u_ = it * S1_THREADS + tid;
    const int I = u_ < 128 ? 1 : (u_ < 384 ? 2 : 3);
    const int lu = u_ - (I == 1 ? 0 : (I == 2 ? 128 : 384));
    const int j = lu >> 3, c = (lu & 7) << 3;
    const int boff = I == 1 ? 0 : (I == 2 ? 2048 : 6144);
    st_chunk8(S + S1_W0 + boff + sw_off16(C, j, c), hb[it]);
    st_chunk8(S + S1_C + boff + sw_off16(C, j, c), lb[it]);  // the C tile is dead once CB is formed
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0 && !flags[4]) {
    sm100::tc_fence_after();
    constexpr uint32_t ID = sm100::idesc_bf16(64, 16, true, false);
#pragma unroll
    for (int I = 1; I < 4; ++I) {
      const int boff = I == 1 ? 0 : (I == 2 ? 2048 : 6144);
      auto fcb = [&](int k) { return kdesc(S + S1_CB + 2048 * I, C, k); };
      mma_steps(tmem + 128 + 16 * I, [&](int k) { return mndesc(S + S1_W0 + boff, C, k); }, fcb, I, ID, false);
      mma_steps(tmem + 128 + 16 * I, [&](int k) { return mndesc(S + S1_C + boff, C, k); }, fcb, I, ID, true);
    }
    sm100::umma_commit(bars + 3);
  }
  pc.mark(4);
  if (!wait_bar(bars + 2, 0, err, 0x5304) || !wait_bar(bars + 3, 0, err, 0x5304)) flags[4] = 1;
  sm100::tc_fence_after();
  __syncthreads();
  pc.mark(5);
  if (flags[4]) goto s1_teardown;
  {
    // S_end^T rows (lane = state row s) -> tile image (rows s, columns p); warpgroup wg takes
    // columns [32 wg, 32 wg + 32)
    const int s = 32 * quarter + lane;
    unsigned char* dst = smem + S1_C;  // staged over the dead C tile for one bulk store
    {
      const int half = wg;
      float x[32];
      tmem_ld32(tmem_at(tmem, quarter, 64 + 32 * half), x);
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float y[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = clip4(x[c + e]);
        *reinterpret_cast<uint4*>(dst + sw_off16(N, s, 32 * half + c)) = pack8(y);
      }
      fence_async_smem();
    }
    // y_diag^T row p (lanes 0-15 of each quarter): the off-diagonal blocks from TMEM as fp32 rows
    // into the dead W buffers; then the diagonal 16 x 16 blocks summed exactly per channel (fp32,
    // exponent floored at -20: these terms dominate and the backward's decay gradient cancels
    // them against the matching column sums); then fp32 rows out
    float* YD = reinterpret_cast<float*>(smem + S1_W0);  // [i][p]
    {  // channel p = 16 quarter + (lane & 15), rows [32 wg + 16 hf, +16): one reference block per thread
      const int hf = lane >> 4, p = 16 * quarter + (lane & 15), i0 = 32 * wg + 16 * hf;
      float x[32], y[16];
      tmem_ld32(tmem_at(tmem, quarter, 128 + 32 * wg), x);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float sh = __shfl_sync(0xffffffffu, x[16 + e], lane & 15);
        y[e] = hf ? sh : (i0 == 0 ? 0.f : x[e]);  // block 0 has no tensor-core part
      }
      const float cr = CUM[i0 * P + p];
#pragma unroll
      for (int e = 0; e < 16; ++e) YD[(i0 + e) * P + p] = y[e] * __expf(CUM[(i0 + e) * P + p] - cr);
    }
    __syncthreads();
    if (tid == 0) {
      bulk_s2g(send_t + ch * T_NP, smem + S1_C, T_NP);
      bulk_commit();
    }
    pc.mark(6);
    {
      // four threads per channel p, one block each: y[i] += e^{c_i - c_r} sum_{j<=i} CB[i][j] (dBx_j e^{c_r - c_j})
      // with r the block's first row (fp32 factors; per-pair exponents where the block's span could
      // overflow them)
      const int p = tid & 63;
      {
        const int I = tid >> 6;
        const int r = 16 * I;
        const float cr = CUM[r * P + p];
        float w[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float xv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_X + sw_off(C, r + t, p)));
          const float dv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_DT + sw_off(C, r + t, p)));
          w[t] = clip4(dv * xv);
        }
        const bool wide = !(cr - CUM[(r + 15) * P + p] <= 80.f);
        if (!wide) {
#pragma unroll
          for (int t = 0; t < 16; ++t) w[t] *= __expf(cr - CUM[(r + t) * P + p]);
          float yv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {  // row r + i of CB: two 16-byte chunks, read by the whole block
            float cb[16];
            unpack8(*reinterpret_cast<const uint4*>(smem + S1_CB + sw_off16(C, r + i, r)), cb);
            unpack8(*reinterpret_cast<const uint4*>(smem + S1_CB + sw_off16(C, r + i, r + 8)), cb + 8);
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j <= i; ++j) acc += cb[j] * w[j];
            yv[i] = YD[(r + i) * P + p] + __expf(CUM[(r + i) * P + p] - cr) * acc;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) YD[(r + i) * P + p] = yv[i];  // after all the loads above
        } else {
#pragma unroll 1
          for (int i = 0; i < 16; ++i) {
            const float ci = CUM[(r + i) * P + p];
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)  // register indices stay constant: j <= i as a predicate
              if (j <= i)
                acc += __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_CB + sw_off(C, r + i, r + j))) *
                       w[j] * __expf(fmaxf(ci - CUM[(r + j) * P + p], -20.f));
            YD[(r + i) * P + p] += acc;
          }
        }
      }
    }
    __syncthreads();
    pc.mark(7);
    {  // fp32 rows [i][p] out as 16-byte vectors
      float* dst2 = yd_t + ch * (C * P);
#pragma unroll
      for (int it = 0; it < (C * P / 4) / S1_THREADS; ++it) {
        const int e4 = 4 * (it * S1_THREADS + tid);
        const float4 v4 = *reinterpret_cast<const float4*>(YD + e4);
        *reinterpret_cast<float4*>(dst2 + e4) = make_float4(clip4(v4.x), clip4(v4.y), clip4(v4.z), clip4(v4.w));
      }
    }
    // decay e^{max(c, -20)} as a tile image (rows i, columns p)
#pragma unroll
    for (int it = 0; it < (C * P / 8) / S1_THREADS; ++it) {
      const int u_ = it * S1_THREADS + tid;
      const int i = u_ >> 3, c = (u_ & 7) << 3;
      float o[8], ci[8];
      ld8f_x(CUM + i * P + c, ci);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __expf(fmaxf(ci[e], -20.f));
      *reinterpret_cast<uint4*>(dec_t + ch * T_CP + sw_off16(C, i, c)) = pack8(o);
    }
  }
s1_teardown:
  if (tid == 0) bulk_wait_all();
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  pc.mark(8);
  if (warp == 0) sm100::tmem_dealloc(tmem, 256);
  pc.done();
}

// ============================================================ state recurrence, forward
// One CTA per (batch, head); thread s keeps state row s (S^T[s][p], 64 fp32) in registers.
// Per chunk: the state (bf16) is written as the MN-major operand, y_off^T = S C^T runs on the
// tensor cores (M = 64 channels, N = 64 rows, K = 128) while the state is carried to the next
// chunk; y rows are transposed through shared memory for 16-byte stores.
constexpr int S2_THREADS = 128;
constexpr int S2_STAGE = T_CN + T_NP + T_CP;  // C tile, S_end^T image, decay image
constexpr int S2_CL = 2 * S2_STAGE;           // 2 x 64 fp32
constexpr int S2_S = S2_CL + 1024;            // state operand (rows s, columns p)
constexpr int S2_Y = S2_S + T_NP;             // y rows (plain [i][p] bf16)
constexpr int S2_BAR = S2_Y + T_CP;
constexpr size_t S2_SMEM = 1024 + S2_BAR + 256;

__global__ void __launch_bounds__(S2_THREADS, 1) ssd_state_fwd_tc(
    const __grid_constant__ CUtensorMap tm_c, const unsigned char* __restrict__ send_t,
    const float* __restrict__ yd_t, const unsigned char* __restrict__ dec_t, const float* __restrict__ cl,
    int L, int H, int NC, const float* __restrict__ s0, bf16* __restrict__ y, unsigned char* __restrict__ sin_t,
    float* __restrict__ s_final, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t Sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S2_BAR);  // full[2], mma
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  PhaseClock pc(32);
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t bh = (int64_t)b * H + h;
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) sm100::mbar_init(bars + i, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tm_c);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 64);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto issue = [&](int n) {
    const int st = n & 1;
    unsigned char* sp = smem + st * S2_STAGE;
    const int64_t c = bh * NC + n;
    const int row0 = b * L + n * C;
    sm100::mbar_expect_tx(bars + st, S2_STAGE + 256);
    sm100::tma_load_2d(sp, &tm_c, bars + st, 0, row0);
    sm100::tma_load_2d(sp + T_CN / 2, &tm_c, bars + st, 64, row0);
    bulk_g2s(sp + T_CN, send_t + c * T_NP, T_NP, bars + st);
    bulk_g2s(sp + T_CN + T_NP, dec_t + c * T_CP, T_CP, bars + st);
    bulk_g2s(smem + S2_CL + st * 256, cl + c * P, 256, bars + st);
  };
  if (tid == 0) {
    issue(0);
    if (NC > 1) issue(1);
  }
  const int s = tid;
  float S[P];
#pragma unroll
  for (int p = 0; p < P; ++p) S[p] = s0 ? s0[(bh * P + p) * N + s] : 0.f;
  int n = 0;
  for (; n < NC; ++n) {
    const int st = n & 1;
    const int64_t c = bh * NC + n;
    const uint32_t sc = Sb + st * S2_STAGE;
#pragma unroll
    for (int p = 0; p < P; p += 8) {
      st_chunk8(Sb + S2_S + sw_off16(N, s, p), S + p);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(0);
    if (tid == 0) {
      if (sin_t) {  // the chunk's start state image, one bulk store of the operand tile
        bulk_s2g(sin_t + c * T_NP, smem + S2_S, T_NP);
        bulk_commit();
      }
      if (!wait_bar(bars + st, (n >> 1) & 1, err, 0x5311)) *abort_flag = 1;
      sm100::tc_fence_after();
      if (!*abort_flag)
        mma_steps(tmem, [&](int k) { return mndesc(Sb + S2_S, N, k); }, [&](int k) { return kdesc(sc, C, k); }, N / 16,
                  sm100::idesc_bf16(64, 64, true, false), false);
      sm100::umma_commit(bars + 2);
    }
    // carry the state: S <- clip(S e^{max(cl, -20)} + S_end)   (S_end^T row s from the image)
    // y epilogue: channel p0 = 16 warp + (lane & 15) (M = 64: lanes 0-15 hold it), rows [ih, ih + 32)
    // per lane, lanes 16-31 taking rows 32-63 by shuffle
    const int p0 = 16 * warp + (lane & 15), ih = 32 * (lane >> 4);
    float ydr[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) ydr[i] = yd_t[c * (C * P) + (ih + i) * P + p0];
    if (!wait_bar(bars + st, (n >> 1) & 1, err, 0x5312)) *abort_flag = 1;  // every thread reads the stage
    {
      const float* clp = reinterpret_cast<const float*>(smem + S2_CL + st * 256);
      const unsigned char* se = smem + st * S2_STAGE + T_CN;
#pragma unroll
      for (int p = 0; p < P; p += 8) {
        float e8[8];
        unpack8(*reinterpret_cast<const uint4*>(se + sw_off16(N, s, p)), e8);
#pragma unroll
        for (int e = 0; e < 8; ++e) S[p + e] = clip4(S[p + e] * __expf(fmaxf(clp[p + e], -20.f)) + e8[e]);
      }
    }
    pc.mark(1);
    if (!wait_bar(bars + 2, n & 1, err, 0x5313)) *abort_flag = 1;
    sm100::tc_fence_after();
    pc.mark(2);
    {
      float yo[64], z[32];
      tmem_ld32(tmem_at(tmem, warp, 0), yo);
      tmem_ld32(tmem_at(tmem, warp, 32), yo + 32);
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float sh = __shfl_sync(0xffffffffu, yo[32 + e], lane & 15);
        z[e] = ih ? sh : yo[e];
      }
      const unsigned char* dec = smem + st * S2_STAGE + T_CN + T_NP;
      bf16* Y = reinterpret_cast<bf16*>(smem + S2_Y);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = ih + i;
        const float dh = __bfloat162float(*reinterpret_cast<const bf16*>(dec + sw_off(C, r, p0)));
        Y[r * P + p0] = __float2bfloat16_rn(clip4(ydr[i] + clip4(z[i] * dh)));
      }
    }
    if (tid == 0) bulk_wait_read();  // the state tile is rewritten in the next step
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(3);
    if (*abort_flag) break;
    if (tid == 0 && n + 2 < NC) issue(n + 2);
#pragma unroll
    for (int it = 0; it < (C * P / 8) / S2_THREADS; ++it) {
      const int u_ = it * S2_THREADS + tid;
      const int i = u_ >> 3, q8 = (u_ & 7) << 3;
      *reinterpret_cast<uint4*>(y + (((int64_t)b * L + (int64_t)n * C + i) * H + h) * P + q8) =
          *reinterpret_cast<const uint4*>(smem + S2_Y + (i * P + q8) * 2);
    }
  }
  if (s_final && n == NC)
#pragma unroll
    for (int p = 0; p < P; ++p) s_final[(bh * P + p) * N + s] = S[p];
  if (tid == 0) bulk_wait_all();
  if (*abort_flag && tid == 0) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 64);
  pc.done();
}

// ============================================================ state recurrence, backward
// Reverse walk with the state gradient dS^T (thread s holds row s): per chunk the gradient that
// reaches the chunk's S_end is stored, then G^T = C^T (dy e^{max(c,-20)}) (M = 128 state rows,
// N = 64 channels, K = 64 rows) and dS <- G^T + e^{max(cl,-20)} dS.
// (reference `atomic_ops/kernel_mamba2_bwd_b1_state.py:132-249`, the reverse state-only scan)
constexpr int B1S_THREADS = 128;
constexpr int B1S_STAGE = T_CN + 2 * T_CP;  // C tile, dy tile, decay image
constexpr int B1S_CL = 2 * B1S_STAGE;
constexpr int B1S_DYD = B1S_CL + 1024;
constexpr int B1S_G = B1S_DYD + T_CP;  // state-gradient image (rows s, columns p) for the bulk store
constexpr int B1S_BAR = B1S_G + T_NP;
constexpr size_t B1S_SMEM = 1024 + B1S_BAR + 256;

__global__ void __launch_bounds__(B1S_THREADS, 1) ssd_state_bwd_tc(
    const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_dy,
    const unsigned char* __restrict__ dec_t, const float* __restrict__ cl, int L, int H, int NC,
    const float* __restrict__ ds_final, unsigned char* __restrict__ dse_t, float* __restrict__ ds0,
    int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t Sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + B1S_BAR);  // full[2], mma
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t bh = (int64_t)b * H + h;
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) sm100::mbar_init(bars + i, 1);
    *abort_flag = 0;
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tm_c);
    sm100::prefetch_tmap(&tm_dy);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 64);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto issue = [&](int it) {
    const int n = NC - 1 - it, st = it & 1;
    unsigned char* sp = smem + st * B1S_STAGE;
    const int64_t c = bh * NC + n;
    const int row0 = b * L + n * C;
    sm100::mbar_expect_tx(bars + st, B1S_STAGE + 256);
    sm100::tma_load_2d(sp, &tm_c, bars + st, 0, row0);
    sm100::tma_load_2d(sp + T_CN / 2, &tm_c, bars + st, 64, row0);
    tma_load_3d(sp + T_CN, &tm_dy, bars + st, 0, h, row0);
    bulk_g2s(sp + T_CN + T_CP, dec_t + c * T_CP, T_CP, bars + st);
    bulk_g2s(smem + B1S_CL + st * 256, cl + c * P, 256, bars + st);
  };
  if (tid == 0) {
    issue(0);
    if (NC > 1) issue(1);
  }
  const int s = tid;
  float G[P];
#pragma unroll
  for (int p = 0; p < P; ++p) G[p] = ds_final ? ds_final[(bh * P + p) * N + s] : 0.f;
  int it = 0;
  for (; it < NC; ++it) {
    const int n = NC - 1 - it, st = it & 1;
    const int64_t c = bh * NC + n;
    const uint32_t sp = Sb + st * B1S_STAGE;
#pragma unroll
    for (int p = 0; p < P; p += 8)
      st_chunk8(Sb + B1S_G + sw_off16(N, s, p), G + p);
    if (!wait_bar(bars + st, (it >> 1) & 1, err, 0x5321)) *abort_flag = 1;
#pragma unroll
    for (int k8 = 0; k8 < (C * P / 8) / B1S_THREADS; ++k8) {
      const int u_ = k8 * B1S_THREADS + tid;
      const int i = u_ >> 3, q8 = (u_ & 7) << 3;
      float dy[8], dc[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(smem + st * B1S_STAGE + T_CN + sw_off16(C, i, q8)), dy);
      unpack8(*reinterpret_cast<const uint4*>(smem + st * B1S_STAGE + T_CN + T_CP + sw_off16(C, i, q8)), dc);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = dy[e] * dc[e];
      st_chunk8(Sb + B1S_DYD + sw_off16(C, i, q8), o);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0) {
      bulk_s2g(dse_t + c * T_NP, smem + B1S_G, T_NP);
      bulk_commit();
      sm100::tc_fence_after();
      mma_steps(tmem, [&](int k) { return mndesc(sp, C, k); }, [&](int k) { return mndesc(Sb + B1S_DYD, C, k); }, C / 16,
                sm100::idesc_bf16(128, 64, true, true), false);
      sm100::umma_commit(bars + 2);
    }
    if (!wait_bar(bars + 2, it & 1, err, 0x5322)) *abort_flag = 1;
    sm100::tc_fence_after();
    {
      const float* clp = reinterpret_cast<const float*>(smem + B1S_CL + st * 256);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float x[32];
        tmem_ld32(tmem_at(tmem, warp, 32 * half), x);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int p = 32 * half + e;
          G[p] = x[e] + __expf(fmaxf(clp[p], -20.f)) * G[p];
        }
      }
    }
    if (tid == 0) bulk_wait_read();  // the gradient image is rewritten in the next step
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0 && it + 2 < NC) issue(it + 2);
  }
  if (ds0 && it == NC)
#pragma unroll
    for (int p = 0; p < P; ++p) ds0[(bh * P + p) * N + s] = G[p];
  if (tid == 0) bulk_wait_all();
  if (*abort_flag && tid == 0) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 64);
}

// ============================================================ chunk-parallel backward
// One CTA per (chunk, batch, head group), 128 threads; the heads of the group run in turn.
// Shared by the heads: B, C tiles, the causal CB = C B^T (as rows and transposed), the fp32 sum
// of dCB over the heads, and dC, dB accumulated in TMEM over the heads.  Per head
// (reference MB1-MB4, `atomic_ops/kernel_mamba2_bwd_b2_intra.py:32-180`,
// `kernel_mamba2_bwd_b1_state.py:132-249`, `mamba2_bwd_a_dA_reference.py:60-115`):
//   dC  += (dy e^{max(c,-20)}) S_in            dB += (dBx e^{max(cl-c,-20)}) dS_end
//   dds^T = dS_end B^T   (state part of d(dBx), per channel)
//   dCB[i][j] += sum_p (dy e^{c_i - c_r})[i][p] (dBx e^{c_r - c_j})[j][p]   per row block (r = 16 I)
//   ddd^T[p][j] = sum_{i >= 16 J + 16} (dy e^{c_i - c_s})[i][p] CB[i][j]  per key block (s = 16 J + 15),
//            plus the diagonal block exactly per channel
//   y_off^T = S_in C^T ; then per channel p, rows i = 63 .. 0: dc, its reverse cumulative sum g,
//   ddt = d(dBx) x + g A [unclipped], dx = d(dBx) dt, dA_h += g dt
// and after the heads dC += dCB B, dB += dCB^T C (dCB summed over the heads), written per group.
constexpr int SB_THREADS = 256;
constexpr int SB_B = 0, SB_C = 16384, SB_CB = 32768, SB_CBT = 40960, SB_DCB = 49152, SB_X = 65536, SB_DT = 73728,
              SB_DY = 81920, SB_S = 90112, SB_DS = 106496, SB_CUM = 122880, SB_DYR = 139264, SB_BI0 = 147456,
              SB_BI1 = 155648, SB_DYD = 163840, SB_V = 172032, SB_DYS0 = 180224, SB_DYS1 = 188416, SB_YD = 196608,
              SB_BAR = 212992;
// per-head outputs dx, ddt staged as plain [i][p] bf16 rows over the dead phase-1 operands, and the
// diagonal part of ddd (fp32 [p][j]) after them
constexpr int SB_OX = SB_DYR, SB_ODT = SB_DYR + T_CP, SB_DDG = SB_BI1, SB_XCH = SB_DDG + 16384;
constexpr size_t SB_SMEM = 1024 + SB_BAR + 256;
// TMEM columns: dC [0,128) and dB [128,256) (M = 64, N = 128); dCB per row block I at 256 + 8 I (I + 1)
// (widths 16, 32, 48, 64); dds^T [416, 480); later ddd^T per key block J < 3 at 256 + 16 J and
// y_off^T [320, 384)
constexpr int TM_DC = 0, TM_DB = 128, TM_DCB = 256, TM_DDS = 416, TM_DDD = 256, TM_YO = 320;

AHB_DEVICE int dcb_off(int I) { return 8 * I * (I + 1); }
// fp32 dCB sum [i][j], row i rotated by i words: the 16 rows of a readout warp hit 16 banks
AHB_DEVICE int dcb_at(int i, int j) { return i * C + ((i + j) & (C - 1)); }
// key operand buffer of dCB row block I (rows j <= 16 I + 15)
AHB_DEVICE int dcb_buf(int I) { return I == 0 ? SB_BI0 : (I == 1 ? SB_BI1 : (I == 2 ? SB_DYS0 : SB_DYS1)); }
// hi / lo operand bases of ddd block J (K steps J + 1 .. 3 stored from 6 KB, 10 KB, 12 KB down:
// regions DYS0 and DYR, 12 KB each)
AHB_DEVICE int ddd_hi(int J) { return SB_DYS0 + (J == 0 ? 0 : (J == 1 ? 6144 : 10240)) - 2048 * (J + 1); }
AHB_DEVICE int ddd_lo(int J) { return SB_DYR + (J == 0 ? 0 : (J == 1 ? 6144 : 10240)) - 2048 * (J + 1); }

// Exact per-channel sum of the diagonal block J for the intra part of d(dBx) at row i, channel p:
// sum over rows i2 >= i of the block of CB[i2][i] dy[i2][p] e^{max(c_i2 - c_i, -20)}, in fp32 like
// the forward's diagonal blocks (the decay gradient cancels the two).
__device__ __noinline__ float sb_exact_ddd(const unsigned char* smem, const float* CUM, int p, int i, int J);

__global__ void __launch_bounds__(SB_THREADS, 1) ssd_chunk_bwd_tc(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dt,
    const __grid_constant__ CUtensorMap tm_dy, const float* __restrict__ A, const unsigned char* __restrict__ sin_t,
    const unsigned char* __restrict__ dse_t, const float* __restrict__ yd_t, int L, int H, bf16* __restrict__ dx_o,
    bf16* __restrict__ ddt_o, float* __restrict__ dA_o, float* __restrict__ dB_part, float* __restrict__ dC_part,
    int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t S = smem_u32(smem);
  float* CUM = reinterpret_cast<float*>(smem + SB_CUM);  // [i][p]
  float* DCB = reinterpret_cast<float*>(smem + SB_DCB);  // [i][j]
  // barriers: 0 B/C, 1 CB, 2 head loads, 3 phase 1, 4 dCB blocks, 8 ddd blocks and y_off, 13 final
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SB_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0..3] exact diagonal blocks of this head, [4] abort
  float* span_w = reinterpret_cast<float*>(flags + 8);  // [2][4]
  PhaseClock pc(16);

  const int n = blockIdx.x, b = blockIdx.y, NC = gridDim.x;
  const int hpg = H / gridDim.z, h0 = blockIdx.z * hpg;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, quarter = warp & 3, wg = warp >> 2;
  const int row0 = b * L + n * C;
  if (tid == 0) {
    for (int i = 0; i < 14; ++i) sm100::mbar_init(bars + i, 1);
    flags[4] = 0;
    sm100::fence_barrier_init();
    sm100::mbar_expect_tx(bars, 2 * T_CN);
    sm100::tma_load_2d(smem + SB_B, &tm_b, bars, 0, row0);
    sm100::tma_load_2d(smem + SB_B + T_CN / 2, &tm_b, bars, 64, row0);
    sm100::tma_load_2d(smem + SB_C, &tm_c, bars, 0, row0);
    sm100::tma_load_2d(smem + SB_C + T_CN / 2, &tm_c, bars, 64, row0);
  }
  if (warp == 0) sm100::tmem_alloc(tmem_slot, 512);
  for (int e = tid; e < C * C; e += SB_THREADS) DCB[e] = 0.f;
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (!wait_bar(bars, 0, err, 0x5331)) flags[4] = 1;
  if (tid == 0 && !flags[4]) {  // CB = C B^T into the (not yet used) dCB columns
    sm100::tc_fence_after();
    mma_steps(tmem + TM_DCB, [&](int s) { return kdesc(S + SB_C, C, s); }, [&](int s) { return kdesc(S + SB_B, C, s); },
              N / 16, sm100::idesc_bf16(64, 64, false, false), false);
    sm100::umma_commit(bars + 1);
  }
  if (!wait_bar(bars + 1, 0, err, 0x5332)) flags[4] = 1;
  sm100::tc_fence_after();
  if (wg == 0) {  // causal CB -> rows tile (i, j) and transposed tile (j, i)
    const int i = 16 * warp + lane;
    float x[64];
    tmem_ld32(tmem_at(tmem, warp, TM_DCB), x);
    tmem_ld32(tmem_at(tmem, warp, TM_DCB + 32), x + 32);
    if (lane < 16) {
#pragma unroll
      for (int j = 0; j < 64; ++j) x[j] = j <= i ? clip4(x[j]) : 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 8) st_chunk8(S + SB_CB + sw_off16(C, i, c), x + c);
#pragma unroll
      for (int j = 0; j < 64; ++j)
        *reinterpret_cast<bf16*>(smem + SB_CBT + sw_off(C, j, i)) = __float2bfloat16_rn(x[j]);
    }
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  pc.mark(0);
  if (flags[4]) goto sb_teardown;
  for (int hh = 0; hh < hpg; ++hh) {
    const int h = h0 + hh;
    const uint32_t ph = hh & 1;
    const int64_t ch = ((int64_t)b * H + h) * NC + n;
    const float Ah = A[h];
    if (tid == 0) {
      sm100::mbar_expect_tx(bars + 2, 3 * T_CP + 2 * T_NP + C * P * 4);
      tma_load_3d(smem + SB_X, &tm_x, bars + 2, 0, h, row0);
      tma_load_3d(smem + SB_DT, &tm_dt, bars + 2, 0, h, row0);
      tma_load_3d(smem + SB_DY, &tm_dy, bars + 2, 0, h, row0);
      bulk_g2s(smem + SB_S, sin_t + ch * T_NP, T_NP, bars + 2);
      bulk_g2s(smem + SB_DS, dse_t + ch * T_NP, T_NP, bars + 2);
      bulk_g2s(smem + SB_YD, yd_t + ch * (C * P), C * P * 4, bars + 2);  // intra-chunk y rows [i][p]
    }
    if (!wait_bar(bars + 2, ph, err, 0x5333)) flags[4] = 1;
    pc.mark(1);
    // decay cumsum (block totals exchanged in the DYR buffer, written only after it)
    chunk_cumsum(smem + SB_DT, Ah, CUM, reinterpret_cast<float*>(smem + SB_DYR), tid);
    if (tid < P) {  // span of each 16-row block
      const int p = tid;
      float sp[4];
#pragma unroll
      for (int I = 0; I < 4; ++I) sp[I] = warp_max(CUM[16 * I * P + p] - CUM[(16 * I + 15) * P + p]);
      if (lane == 0)
#pragma unroll
        for (int I = 0; I < 4; ++I) span_w[warp * 4 + I] = sp[I];
    }
    __syncthreads();
    pc.mark(2);
    if (tid < 4) flags[tid] = !(fmaxf(span_w[tid], span_w[4 + tid]) <= 60.f);
    // DYR = dy e^{c - c_r(i)}, DYD = dy e^{max(c,-20)}, V = dBx e^{max(cl - c, -20)}  (rows, columns p)
    // outputs of both units kept until the stores after the loop (the units' loads come first)
    float r8[2][8], d8[2][8], v8[2][8];
#pragma unroll
    for (int it = 0; it < (C * P / 8) / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int i = u_ >> 3, c = (u_ & 7) << 3;
      float dy[8], xv[8], dv[8];
      unpack8(*reinterpret_cast<const uint4*>(smem + SB_DY + sw_off16(C, i, c)), dy);
      unpack8(*reinterpret_cast<const uint4*>(smem + SB_X + sw_off16(C, i, c)), xv);
      unpack8(*reinterpret_cast<const uint4*>(smem + SB_DT + sw_off16(C, i, c)), dv);
      float c8[8], cr8[8], cl8[8];
      ld8f_x(CUM + i * P + c, c8);
      ld8f_x(CUM + (i & ~15) * P + c, cr8);
      ld8f_x(CUM + (C - 1) * P + c, cl8);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        r8[it][e] = dy[e] * __expf(c8[e] - cr8[e]);
        d8[it][e] = dy[e] * __expf(fmaxf(c8[e], -20.f));
        v8[it][e] = clip4(dv[e] * xv[e]) * __expf(fmaxf(cl8[e] - c8[e], -20.f));
      }
    }
#pragma unroll
    for (int it = 0; it < (C * P / 8) / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int i = u_ >> 3, c = (u_ & 7) << 3;
      st_chunk8(S + SB_DYR + sw_off16(C, i, c), r8[it]);
      st_chunk8(S + SB_DYD + sw_off16(C, i, c), d8[it]);
      st_chunk8(S + SB_V + sw_off16(C, i, c), v8[it]);
    }
    pc.mark(3);
    // dCB of this head per row block I: keys (dBx e^{c_r - c_j}) for j <= 16 I + 15, the four blocks'
    // operands (BI0, BI1, DYS0, DYS1; 1280 16-byte units) in the same pass as the tiles above (the
    // exact-block flags read from the span maxima: flags[] is written by threads 0-3 above)
    float ob[1280 / SB_THREADS][8];  // stored after the loop (the units' loads come first)
#pragma unroll
    for (int it = 0; it < 1280 / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int I = u_ < 128 ? 0 : (u_ < 384 ? 1 : (u_ < 768 ? 2 : 3));
      const int lu = u_ - 64 * I * (I + 1);
      const int j = lu >> 3, c = (lu & 7) << 3;
      float xv[8], dv[8];
      float* o = ob[it];
      unpack8(*reinterpret_cast<const uint4*>(smem + SB_X + sw_off16(C, j, c)), xv);
      unpack8(*reinterpret_cast<const uint4*>(smem + SB_DT + sw_off16(C, j, c)), dv);
      const bool zero = !(fmaxf(span_w[I], span_w[4 + I]) <= 60.f) && j >= 16 * I;
      float cj[8], cr8[8];
      ld8f_x(CUM + j * P + c, cj);
      ld8f_x(CUM + 16 * I * P + c, cr8);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = zero ? 0.f : clip4(dv[e] * xv[e]) * __expf(cr8[e] - cj[e]);
    }
#pragma unroll
    for (int it = 0; it < 1280 / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int I = u_ < 128 ? 0 : (u_ < 384 ? 1 : (u_ < 768 ? 2 : 3));
      const int lu = u_ - 64 * I * (I + 1);
      st_chunk8(S + dcb_buf(I) + sw_off16(C, lu >> 3, (lu & 7) << 3), ob[it]);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0 && !flags[4]) {  // dCB first (its readout comes next), then dC, dB and dds
      sm100::tc_fence_after();
#pragma unroll
      for (int I = 0; I < 4; ++I)
        mma_steps(tmem + TM_DCB + dcb_off(I), [&](int k) { return kdesc(S + SB_DYR, C, k); },
                  [&](int k) { return kdesc(S + dcb_buf(I), C, k); }, P / 16,
                  sm100::idesc_bf16(64, 16 * (I + 1), false, false), false);
      sm100::umma_commit(bars + 4);
      const bool acc = hh > 0;
      mma_steps(tmem + TM_DC, [&](int k) { return kdesc(S + SB_DYD, C, k); }, [&](int k) { return kdesc(S + SB_S, N, k); },
                P / 16, sm100::idesc_bf16(64, 128, false, false), acc);
      mma_steps(tmem + TM_DB, [&](int k) { return kdesc(S + SB_V, C, k); }, [&](int k) { return kdesc(S + SB_DS, N, k); },
                P / 16, sm100::idesc_bf16(64, 128, false, false), acc);
      mma_steps(tmem + TM_DDS, [&](int k) { return mndesc(S + SB_DS, N, k); }, [&](int k) { return kdesc(S + SB_B, C, k); },
                N / 16, sm100::idesc_bf16(64, 64, true, false), false);
      sm100::umma_commit(bars + 3);
      pc.mark(14);
    }
    pc.mark(4);
    if (!wait_bar(bars + 4, ph, err, 0x5335)) flags[4] = 1;
    pc.mark(5);
    sm100::tc_fence_after();
    {  // dCB rows i = 16 quarter + lane (block I = quarter) into the fp32 sum over the heads; the
       // warpgroups take alternate 16-column blocks
      const int i = 16 * quarter + lane, I = quarter;
#pragma unroll
      for (int p4 = wg; p4 < 4; p4 += 2)
        if (p4 <= I) {
          float x[16];
          tmem_ld16(tmem_at(tmem, quarter, TM_DCB + dcb_off(I) + 16 * p4), x);
          if (lane < 16)
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int j = 16 * p4 + e;
              if (j <= i) DCB[dcb_at(i, j)] += x[e];
            }
        }
      if (wg == (I & 1) && lane < 16) {  // the warp that added block p4 = I
        if (flags[I]) {  // exact per-channel sums on the diagonal block
          for (int j = 16 * I; j <= i; ++j) {
            float acc = 0.f;
            for (int p = 0; p < P; ++p) {
              const float dyv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DY + sw_off(C, i, p)));
              const float xv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_X + sw_off(C, j, p)));
              const float dv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DT + sw_off(C, j, p)));
              acc += dyv * clip4(dv * xv) * __expf(fmaxf(CUM[i * P + p] - CUM[j * P + p], -20.f));
            }
            DCB[dcb_at(i, j)] += acc;
          }
        }
      }
    }
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(6);
    if (flags[4]) break;
    // phase 2: ddd^T per key block J (reference s = 16 J + 15) and y_off^T
    // ddd^T blocks J = 0..2 below the diagonal block (rows i >= 16 J + 16; block 3 has none) as bf16
    // hi + lo operands, packed: block J's K steps J + 1 .. 3 (2 KB each) at hi / lo bases shifted
    // down by 2 KB (J + 1); one pass (768 units), then the MMAs and y_off^T
    float hb[768 / SB_THREADS][8], lb[768 / SB_THREADS][8];  // stored after the loop
#pragma unroll
    for (int it = 0; it < 768 / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int J = u_ < 384 ? 0 : (u_ < 640 ? 1 : 2);
      const int lu = u_ - (J == 0 ? 0 : (J == 1 ? 384 : 640));
      const int i = 16 * (J + 1) + (lu >> 3), c = (lu & 7) << 3;
      float dy[8];
      float* o = hb[it];
      float* lo = lb[it];
      unpack8(*reinterpret_cast<const uint4*>(smem + SB_DY + sw_off16(C, i, c)), dy);
      float ci[8], cs8[8];
      ld8f_x(CUM + i * P + c, ci);
      ld8f_x(CUM + (16 * J + 15) * P + c, cs8);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = dy[e] * __expf(ci[e] - cs8[e]);
        lo[e] = o[e] - __bfloat162float(__float2bfloat16_rn(o[e]));
      }
    }
#pragma unroll
    for (int it = 0; it < 768 / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int J = u_ < 384 ? 0 : (u_ < 640 ? 1 : 2);
      const int lu = u_ - (J == 0 ? 0 : (J == 1 ? 384 : 640));
      const int i = 16 * (J + 1) + (lu >> 3), c = (lu & 7) << 3;
      st_chunk8(S + ddd_hi(J) + sw_off16(C, i, c), hb[it]);
      st_chunk8(S + ddd_lo(J) + sw_off16(C, i, c), lb[it]);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0 && !flags[4]) {
      sm100::tc_fence_after();
      constexpr uint32_t ID = sm100::idesc_bf16(64, 16, true, false);
#pragma unroll
      for (int J = 0; J < 3; ++J) {
        for (int k = J + 1; k < 4; ++k)
          sm100::umma_bf16(tmem + TM_DDD + 16 * J, mndesc(S + ddd_hi(J), C, k), kdesc(S + SB_CBT + 2048 * J, C, k),
                           ID, k > J + 1 ? 1u : 0u);
        for (int k = J + 1; k < 4; ++k)
          sm100::umma_bf16(tmem + TM_DDD + 16 * J, mndesc(S + ddd_lo(J), C, k), kdesc(S + SB_CBT + 2048 * J, C, k),
                           ID, 1u);
      }
      mma_steps(tmem + TM_YO, [&](int k) { return mndesc(S + SB_S, N, k); },
                [&](int k) { return kdesc(S + SB_C, C, k); }, N / 16, sm100::idesc_bf16(64, 64, true, false), false);
      sm100::umma_commit(bars + 8);
    }
    pc.mark(7);
    // the dC / dB / dds products read DYD and V, over which DDG and XCH are written below
    if (!wait_bar(bars + 3, ph, err, 0x5336)) flags[4] = 1;
    {
      // diagonal blocks of ddd, four threads per channel, one block each, while the MMAs run:
      // ddd[j] = e^{c_s - c_j} sum_{i>=j} CB[i][j] (dy_i e^{c_i - c_s}) with s the block's last row
      float* DDG = reinterpret_cast<float*>(smem + SB_DDG);  // [j][p]
      const int p = tid & 63;
      {
        const int J = tid >> 6;
        const int r = 16 * J;
        const float cs = CUM[(r + 15) * P + p];
        float u[16];
#pragma unroll
        for (int t = 0; t < 16; ++t)
          u[t] = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DY + sw_off(C, r + t, p)));
        const bool wide = !(CUM[r * P + p] - cs <= 80.f);
        if (!wide) {
#pragma unroll
          for (int t = 0; t < 16; ++t) u[t] *= __expf(CUM[(r + t) * P + p] - cs);
          // column j of the block = row r + j of CB^T: two 16-byte chunks (rows i < j are the
          // causal mask's zeros), read by every thread of the block (broadcast)
          float dv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float cb[16];
            unpack8(*reinterpret_cast<const uint4*>(smem + SB_CBT + sw_off16(C, r + j, r)), cb);
            unpack8(*reinterpret_cast<const uint4*>(smem + SB_CBT + sw_off16(C, r + j, r + 8)), cb + 8);
            float acc = 0.f;
#pragma unroll
            for (int i = j; i < 16; ++i) acc += cb[i] * u[i];
            dv[j] = __expf(cs - CUM[(r + j) * P + p]) * acc;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) DDG[(r + j) * P + p] = dv[j];  // after all the loads above
        } else {
          for (int j = 0; j < 16; ++j) DDG[(r + j) * P + p] = sb_exact_ddd(smem, CUM, p, r + j, J);
        }
      }
    }
    pc.mark(8);
    if (!wait_bar(bars + 8, ph, err, 0x5337)) flags[4] = 1;
    sm100::tc_fence_after();
    __syncthreads();
    pc.mark(9);
    {
      // four threads per channel p = 16 quarter + (lane & 15), one 16-row block each, in descending
      // row order k = 2 wg + (lane >> 4): block J = 3 - k (warpgroup 0 rows 32-63, lanes 0-15 the
      // upper block).  The M = 64 accumulators hold channel p in lane p & 15 of the quarter, so the
      // lower block's values reach lanes 16-31 by shuffle.  Pass 1 (descending rows): dc without the
      // last row's extra term and its local suffix sums, d(dBx), dx; the four threads then exchange
      // their suffix totals and the parts of that extra term (state carry and the state part of
      // d(dBx)); pass 2: g, ddt and dA.
      const int hf = lane >> 4, cl16 = lane & 15;
      const int p = 16 * quarter + cl16;
      const int jb = wg == 0 ? 2 : 0;       // lower of the warpgroup's two blocks
      const int J = jb + 1 - hf;            // this thread's block
      const int kq = 2 * wg + hf;           // position in the descending row order
      float* XCH = reinterpret_cast<float*>(smem + SB_XCH);  // [k][p]: suffix totals; [4 + k][p]: dcl parts
      float dds[16], ddd[16], yo[16];
      {
        float a32[32], lo16[16], hi16[16];
        tmem_ld32(tmem_at(tmem, quarter, TM_DDS + 16 * jb), a32);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, a32[e], cl16);
          dds[e] = hf ? sh : a32[16 + e];
        }
        tmem_ld16(tmem_at(tmem, quarter, TM_DDD + 16 * jb), lo16);
        tmem_ld16(tmem_at(tmem, quarter, TM_DDD + 16 * (jb + 1)), hi16);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, lo16[e], cl16);
          ddd[e] = hf ? sh : (J == 3 ? 0.f : hi16[e]);  // block 3 is all diagonal: no MMA part
        }
        tmem_ld16(tmem_at(tmem, quarter, TM_YO + 16 * jb), lo16);
        tmem_ld16(tmem_at(tmem, quarter, TM_YO + 16 * (jb + 1)), hi16);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float sh = __shfl_sync(0xffffffffu, lo16[e], cl16);
          yo[e] = hf ? sh : hi16[e];
        }
      }
      float suf[16], ddbx[16], oxv[16];
      float dclp = 0.f, local = 0.f;
      const float cl = CUM[(C - 1) * P + p];
      bf16* OX = reinterpret_cast<bf16*>(smem + SB_OX);
      {
        float car = 0.f;
        for (int s = 32 * kq; s < 32 * kq + 32; ++s)
          car += __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DS + sw_off(N, s, p))) *
                 __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_S + sw_off(N, s, p)));
        if (cl > -20.f) dclp += car * __expf(cl);
      }
      {
        const float* ydr = reinterpret_cast<const float*>(smem + SB_YD);  // [i][p]
        const float cs = CUM[(16 * J + 15) * P + p];
#pragma unroll
        for (int r = 15; r >= 0; --r) {
          const int i = 16 * J + r;
          const float ci = CUM[i * P + p];
          const float dyv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DY + sw_off(C, i, p)));
          const float xv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_X + sw_off(C, i, p)));
          const float dtv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DT + sw_off(C, i, p)));
          const float bx = clip4(dtv * xv);
          const float dd = ddd[r] * __expf(cs - ci) + reinterpret_cast<const float*>(smem + SB_DDG)[i * P + p];
          const float dlt = cl - ci;
          const float ds = dds[r] * __expf(fmaxf(dlt, -20.f));
          float dc = dyv * ydr[i * P + p] - bx * dd;
          if (ci > -20.f) dc += dyv * yo[r] * __expf(ci);
          if (dlt > -20.f) {
            dc -= bx * ds;
            dclp += bx * ds;
          }
          local += dc;
          suf[r] = local;
          ddbx[r] = dd + ds;
          oxv[r] = ddbx[r] * dtv;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r)  // stores after all the loads of the loop above
          OX[(16 * J + r) * P + p] = __float2bfloat16_rn(oxv[r]);
      }
      XCH[kq * 64 + p] = local;
      XCH[(4 + kq) * 64 + p] = dclp;
      __syncthreads();
      pc.mark(10);
      float dAh = 0.f;
      {
        float off = XCH[4 * 64 + p] + XCH[5 * 64 + p] + XCH[6 * 64 + p] + XCH[7 * 64 + p];
        for (int k2 = 0; k2 < kq; ++k2) off += XCH[k2 * 64 + p];
        bf16* ODT = reinterpret_cast<bf16*>(smem + SB_ODT);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const int i = 16 * J + r;
          const float xv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_X + sw_off(C, i, p)));
          const float dtv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DT + sw_off(C, i, p)));
          const float g = off + suf[r];
          const float pre = dtv * Ah;
          const float gA = (pre > -20.f && pre < 20.f) ? g : 0.f;
          oxv[r] = ddbx[r] * xv + gA * Ah;
          dAh += gA * dtv;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) ODT[(16 * J + r) * P + p] = __float2bfloat16_rn(oxv[r]);
      }
      dAh = warp_sum(dAh);
      if (lane == 0) atomicAdd(dA_o + h, dAh);
    }
    sm100::tc_fence_before();
    __syncthreads();
    pc.mark(11);
#pragma unroll
    for (int it = 0; it < (C * P / 8) / SB_THREADS; ++it) {
      const int u_ = it * SB_THREADS + tid;
      const int i = u_ >> 3, c8 = (u_ & 7) << 3;
      const int64_t gi = (((int64_t)b * L + (int64_t)n * C + i) * H + h) * P + c8;
      *reinterpret_cast<uint4*>(dx_o + gi) = *reinterpret_cast<const uint4*>(smem + SB_OX + (i * P + c8) * 2);
      *reinterpret_cast<uint4*>(ddt_o + gi) = *reinterpret_cast<const uint4*>(smem + SB_ODT + (i * P + c8) * 2);
    }
    __syncthreads();
    pc.mark(12);
  }
  if (flags[4]) goto sb_teardown;
  // dC += dCB B and dB += dCB^T C with dCB summed over the group's heads
#pragma unroll
  for (int it = 0; it < (C * C / 8) / SB_THREADS; ++it) {
    const int u_ = it * SB_THREADS + tid;
    const int i = u_ >> 3, c = (u_ & 7) << 3;
    float r8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) r8[e] = DCB[dcb_at(i, c + e)];
    st_chunk8(S + SB_CB + sw_off16(C, i, c), r8);
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    sm100::tc_fence_after();
    mma_steps(tmem + TM_DC, [&](int k) { return kdesc(S + SB_CB, C, k); }, [&](int k) { return mndesc(S + SB_B, C, k); },
              C / 16, sm100::idesc_bf16(64, 128, false, true), true);
    mma_steps(tmem + TM_DB, [&](int k) { return mndesc(S + SB_CB, C, k); }, [&](int k) { return mndesc(S + SB_C, C, k); },
              C / 16, sm100::idesc_bf16(64, 128, true, true), true);
    sm100::umma_commit(bars + 13);
  }
  if (!wait_bar(bars + 13, 0, err, 0x5338)) goto sb_teardown;
  sm100::tc_fence_after();
  {
    // warpgroup 0 reads dC, warpgroup 1 dB (rows i = 16 quarter + lane, lanes 0-15)
    const int i = 16 * quarter + lane;
    const int64_t off = (((int64_t)blockIdx.z * gridDim.y + b) * L + (int64_t)n * C + i) * N;
#pragma unroll 1
    for (int q = 4 * wg; q < 4 * wg + 4; ++q) {
      float x[32];
      tmem_ld32(tmem_at(tmem, quarter, (q < 4 ? TM_DC : TM_DB) + 32 * (q & 3)), x);
      if (lane < 16) {
        float* dst = (q < 4 ? dC_part : dB_part) + off + 32 * (q & 3);
#pragma unroll
        for (int e = 0; e < 32; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
      }
    }
  }
sb_teardown:
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  pc.mark(13);
  if (warp == 0) sm100::tmem_dealloc(tmem, 512);
  pc.done();
}

__global__ void sum_groups_tc(const float* __restrict__ part, int G, int64_t n, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int g = 0; g < G; ++g) s += part[g * n + i];
    out[i] = s;
  }
}

__device__ __noinline__ float sb_exact_ddd(const unsigned char* smem, const float* CUM, int p, int i, int J) {
  float acc = 0.f;
  const float ci = CUM[i * P + p];
  for (int i2 = i; i2 < 16 * J + 16; ++i2) {
    const float cb = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_CB + sw_off(C, i2, i)));
    const float dy = __bfloat162float(*reinterpret_cast<const bf16*>(smem + SB_DY + sw_off(C, i2, p)));
    acc += cb * dy * __expf(fmaxf(CUM[i2 * P + p] - ci, -20.f));
  }
  return acc;
}

template <class K>
int set_smem_tc(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess ? 0 : -3;
}

// S1 + S2 on the given scratch (per chunk-head: S_end^T image, y_diag^T rows, decay image, last
// cumsum)
int ssd_forward(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, int B, int L, int H,
                unsigned char* send_t, float* yd_t, unsigned char* dec_t, float* cl, const float* s0, float* s_final,
                void* y, unsigned char* sin_t, int* err, cudaStream_t st) {
  static int i1 = set_smem_tc(ssd_chunk_fwd_tc, S1_SMEM);
  static int i2 = set_smem_tc(ssd_state_fwd_tc, S2_SMEM);
  if (i1 || i2) return -3;
  CUtensorMap tb, tc, tx, tdt;
  if (tmap_2d_bf16(&tb, Bm, (int64_t)B * L, N, C) || tmap_2d_bf16(&tc, Cm, (int64_t)B * L, N, C) ||
      tmap_seq_bf16(&tx, x, (int64_t)B * L, H, P, C) || tmap_seq_bf16(&tdt, dt, (int64_t)B * L, H, P, C))
    return -20;
  const int NC = L / C;
  ssd_chunk_fwd_tc<<<dim3(NC, H, B), S1_THREADS, S1_SMEM, st>>>(tb, tc, tx, tdt, A, L, H, send_t, yd_t, dec_t, cl, err);
  if (cudaGetLastError() != cudaSuccess) return -4;
  ssd_state_fwd_tc<<<dim3(H, B), S2_THREADS, S2_SMEM, st>>>(tc, send_t, yd_t, dec_t, cl, L, H, NC, s0, (bf16*)y, sin_t,
                                                           s_final, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace

int ahb_ssd_supported(int P_, int N_) { return (P_ == P && N_ == N) ? C : 0; }

int ahb_ssd_fwd_tc(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, int B, int L, int H,
                   void* send_t, void* yd_t, void* dec_t, float* cl, const float* s0, float* s_final, void* y,
                   void* sin_t, int* err, cudaStream_t st) {
  return ssd_forward(x, dt, A, Bm, Cm, B, L, H, (unsigned char*)send_t, (float*)yd_t, (unsigned char*)dec_t, cl, s0,
                     s_final, y, (unsigned char*)sin_t, err, st);
}

AHB_PHASE_PROF_SETTER(ahb_ssd_phase_prof)

int ahb_ssd_head_groups(int H) {
  // eight heads per CTA where there are 32 or more: the chunk's B / C tiles, C B^T and the dB / dC
  // epilogue are shared by more heads and there are fewer partial sums to add
  if (H >= 32 && H % 8 == 0) return H / 8;
  for (int g : {8, 4, 2}) if (H % g == 0) return g;
  return 1;
}

int ahb_ssd_bwd_chunk_tc(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, const void* dy,
                         int B, int L, int H, const void* sin_t, const void* dse_t, const void* yd_t, void* dx, void* ddt,
                         float* dB, float* dC, float* dA, float* dB_part, float* dC_part, int* err, cudaStream_t st) {
  static int i1 = set_smem_tc(ssd_chunk_bwd_tc, SB_SMEM);
  if (i1) return -3;
  CUtensorMap tb, tc, tx, tdt, tdy;
  if (tmap_2d_bf16(&tb, Bm, (int64_t)B * L, N, C) || tmap_2d_bf16(&tc, Cm, (int64_t)B * L, N, C) ||
      tmap_seq_bf16(&tx, x, (int64_t)B * L, H, P, C) || tmap_seq_bf16(&tdt, dt, (int64_t)B * L, H, P, C) ||
      tmap_seq_bf16(&tdy, dy, (int64_t)B * L, H, P, C))
    return -20;
  const int G = ahb_ssd_head_groups(H);
  ssd_chunk_bwd_tc<<<dim3(L / C, B, G), SB_THREADS, SB_SMEM, st>>>(
      tb, tc, tx, tdt, tdy, A, (const unsigned char*)sin_t, (const unsigned char*)dse_t, (const float*)yd_t, L, H,
      (bf16*)dx, (bf16*)ddt, dA, dB_part, dC_part, err);
  if (cudaGetLastError() != cudaSuccess) return -4;
  const int64_t n = (int64_t)B * L * N;
  const int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
  sum_groups_tc<<<blocks, 256, 0, st>>>(dB_part, G, n, dB);
  sum_groups_tc<<<blocks, 256, 0, st>>>(dC_part, G, n, dC);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

int ahb_ssd_state_bwd_tc(const void* Cm, const void* dy, const void* dec_t, const float* cl, int B, int L, int H,
                         const float* ds_final, void* dse_t, float* ds0, int* err, cudaStream_t st) {
  static int i1 = set_smem_tc(ssd_state_bwd_tc, B1S_SMEM);
  if (i1) return -3;
  CUtensorMap tc, tdy;
  if (tmap_2d_bf16(&tc, Cm, (int64_t)B * L, N, C) || tmap_seq_bf16(&tdy, dy, (int64_t)B * L, H, P, C)) return -20;
  ssd_state_bwd_tc<<<dim3(H, B), B1S_THREADS, B1S_SMEM, st>>>(tc, tdy, (const unsigned char*)dec_t, cl, L, H, L / C,
                                                              ds_final, (unsigned char*)dse_t, ds0, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// ============================================================ allocation-free forward
// See ssd_noalloc.h: the forward's per-chunk intermediates live in this fixed device array.
#include <cstdio>
#include <mutex>
#include "ssd_noalloc.h"

static __device__ __align__(256) unsigned char g_ssd_noalloc_scratch[AHB_SSD_NOALLOC_SCRATCH_BYTES];
static __device__ int g_ssd_noalloc_err;  // device-side timeout word of the forward kernels

namespace {
constexpr int kMaxDevices = 64;
void* g_noalloc_ptr[kMaxDevices] = {};
int* g_noalloc_err[kMaxDevices] = {};
std::mutex g_noalloc_mu;
static_assert(T_NP + C * P * 4 + T_CP + P * 4 == AHB_SSD_NOALLOC_BYTES_PER_CHUNK_HEAD, "scratch per chunk-head");
}  // namespace

extern "C" int ahb_ssd_fwd_noalloc(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm,
                                   int B, int L, int H, void* y, cudaStream_t stream) {
  if (!x || !dt || !A || !Bm || !Cm || !y || B <= 0 || L <= 0 || H <= 0 || L % C != 0) return AHB_NOALLOC_EINVAL;
  const unsigned long long chunk_heads = (unsigned long long)B * H * (L / C);
  if (chunk_heads > AHB_SSD_NOALLOC_MAX_CHUNK_HEADS) {
    fprintf(stderr,
            "ahb_ssd_fwd_noalloc: B*H*(L/64) = %llu exceeds the fixed scratch limit of %u chunk-heads (%u bytes)\n",
            chunk_heads, (unsigned)AHB_SSD_NOALLOC_MAX_CHUNK_HEADS, (unsigned)AHB_SSD_NOALLOC_SCRATCH_BYTES);
    return AHB_NOALLOC_ETOOBIG;
  }
  // an error left pending by earlier work is reported, not cleared: it is not this call's
  if (cudaPeekAtLastError() != cudaSuccess) return AHB_NOALLOC_EPENDING;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AHB_NOALLOC_ESETUP;
  unsigned char* base = nullptr;
  int* errp = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      void* e = nullptr;
      if (cudaGetSymbolAddress(&p, g_ssd_noalloc_scratch) != cudaSuccess || !p) return AHB_NOALLOC_ESETUP;
      if (cudaGetSymbolAddress(&e, g_ssd_noalloc_err) != cudaSuccess || !e) return AHB_NOALLOC_ESETUP;
      g_noalloc_ptr[dev] = p;
      g_noalloc_err[dev] = static_cast<int*>(e);
    }
    base = static_cast<unsigned char*>(g_noalloc_ptr[dev]);
    errp = g_noalloc_err[dev];
  }
  unsigned char* send_t = base;
  float* yd_t = reinterpret_cast<float*>(send_t + chunk_heads * T_NP);
  unsigned char* dec_t = reinterpret_cast<unsigned char*>(yd_t) + chunk_heads * (C * P * 4);
  float* cl = reinterpret_cast<float*>(dec_t + chunk_heads * T_CP);
  const int rc = ssd_forward(x, dt, A, Bm, Cm, B, L, H, send_t, yd_t, dec_t, cl, nullptr, nullptr, y, nullptr, errp,
                             stream);
  if (rc == -4) return AHB_NOALLOC_ELAUNCH;
  return rc == 0 ? AHB_NOALLOC_OK : AHB_NOALLOC_ESETUP;
}
