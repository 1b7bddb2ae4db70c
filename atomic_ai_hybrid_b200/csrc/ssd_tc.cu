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
//     (M = 128 state rows) and y_diag^T per 16-row reference block (the pairwise decay split at
//     r = 16 I, rows e^{c_i - c_r} <= 1, keys e^{c_r - c_j}; blocks whose decay span exceeds 60
//     are summed exactly per channel); writes S_end^T and the decay e^{max(c,-20)} as swizzled
//     tile images, y_diag^T rows and the chunk's last cumsum.
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

using namespace ahb;
using namespace ahb::umma;
using bf16 = __nv_bfloat16;

namespace {

constexpr int C = 64, P = 64, N = 128;
constexpr int T_CP = C * P * 2;   // 64 x 64 bf16 tile (8 KB)
constexpr int T_CN = C * N * 2;   // 64 x 128 bf16 tile (16 KB)
constexpr int T_NP = N * P * 2;   // 128 x 64 bf16 tile (16 KB)

AHB_DEVICE float clip4(float x) { return sanitize(x, 1e4f); }

// ============================================================ chunk-parallel forward
constexpr int S1_THREADS = 128;
constexpr int S1_B = 0, S1_C = 16384, S1_X = 32768, S1_DT = 40960, S1_CB = 49152, S1_V = 57344, S1_W0 = 65536,
              S1_W1 = 73728, S1_CUM = 81920, S1_BAR = 98304;
constexpr size_t S1_SMEM = 1024 + S1_BAR + 256;

__global__ void __launch_bounds__(S1_THREADS, 2) ssd_chunk_fwd_tc(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dt, const float* __restrict__ A,
    int L, int H, unsigned char* __restrict__ send_t, bf16* __restrict__ yd_t, unsigned char* __restrict__ dec_t,
    float* __restrict__ cl_o, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t S = smem_u32(smem);
  float* CUM = reinterpret_cast<float*>(smem + S1_CUM);  // [i][p]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S1_BAR);  // 0 load, 1 CB, 2 S_end, 3-6 y_diag blocks
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0..3] exact diagonal block, [4] abort
  float* span_w = reinterpret_cast<float*>(flags + 8);  // [2 warps][4]

  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, NC = gridDim.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
  if (!wait_bar(bars, 0, err, 0x5301)) flags[4] = 1;
  if (tid == 0 && !flags[4]) {  // CB = C B^T  (M = 64 rows i, N = 64 keys j)
    sm100::tc_fence_after();
    mma_steps(tmem, [&](int s) { return kdesc(S + S1_C, C, s); }, [&](int s) { return kdesc(S + S1_B, C, s); }, N / 16,
              sm100::idesc_bf16(64, 64, false, false), false);
    sm100::umma_commit(bars + 1);
  }
  const float Ah = A[h];
  if (tid < P) {  // decay cumsum of channel p; span of each 16-row block
    const int p = tid;
    float s = 0.f;
    for (int i = 0; i < C; ++i) {
      const float dtv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_DT + sw_off(C, i, p)));
      s += fminf(fmaxf(dtv * Ah, -20.f), 20.f);
      CUM[i * P + p] = fminf(fmaxf(s, -1e4f), 1e4f);
    }
    cl_o[ch * P + p] = CUM[(C - 1) * P + p];
    float sp[4];
#pragma unroll
    for (int I = 0; I < 4; ++I) sp[I] = warp_max(CUM[16 * I * P + p] - CUM[(16 * I + 15) * P + p]);
    if (lane == 0)
#pragma unroll
      for (int I = 0; I < 4; ++I) span_w[warp * 4 + I] = sp[I];
  }
  __syncthreads();
  if (tid < 4) flags[tid] = !(fmaxf(span_w[tid], span_w[4 + tid]) <= 60.f);
  // V = dBx e^{max(cl - c, -20)}  (rows j, columns p)
#pragma unroll
  for (int it = 0; it < (C * P / 8) / S1_THREADS; ++it) {
    const int u_ = it * S1_THREADS + tid;
    const int j = u_ >> 3, c = (u_ & 7) << 3;
    float xv[8], dv[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(smem + S1_X + sw_off16(C, j, c)), xv);
    unpack8(*reinterpret_cast<const uint4*>(smem + S1_DT + sw_off16(C, j, c)), dv);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      o[e] = clip4(dv[e] * xv[e]) * __expf(fmaxf(CUM[(C - 1) * P + c + e] - CUM[j * P + c + e], -20.f));
    st_chunk8(S + S1_V + sw_off16(C, j, c), o);
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
  if (!wait_bar(bars + 1, 0, err, 0x5302)) flags[4] = 1;
  sm100::tc_fence_after();
  {  // causal CB rows (lanes 0-15 of each quarter) -> bf16 K-major tile (rows i, columns j <= i)
    const int i = 16 * warp + lane;
    float x[64];
    tmem_ld32(tmem_at(tmem, warp, 0), x);
    tmem_ld32(tmem_at(tmem, warp, 32), x + 32);
    if (lane < 16) {
#pragma unroll
      for (int j = 0; j < 64; ++j) x[j] = j <= i ? clip4(x[j]) : 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 8) st_chunk8(S + S1_CB + sw_off16(C, i, c), x + c);
    }
  }
  fence_async_smem();
  sm100::tc_fence_before();
  __syncthreads();
  // y_diag^T per reference block I (r = 16 I): W[j][p] = dBx e^{c_r - c_j} for keys j <= 16 I + 15,
  // D[p][i in block I] += W^T CB^T  -> TMEM columns [128 + 16 I, +16)
#pragma unroll
  for (int I = 0; I < 4; ++I) {
    const uint32_t buf = S + ((I & 1) ? S1_W1 : S1_W0);
    if (I >= 2 && !wait_bar(bars + 3 + I - 2, 0, err, 0x5303)) flags[4] = 1;
    const bool exact = flags[I];
#pragma unroll
    for (int it = 0; it <= I; ++it) {
      const int u_ = it * S1_THREADS + tid;
      const int j = u_ >> 3, c = (u_ & 7) << 3;
      float xv[8], dv[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(smem + S1_X + sw_off16(C, j, c)), xv);
      unpack8(*reinterpret_cast<const uint4*>(smem + S1_DT + sw_off16(C, j, c)), dv);
      const bool zero = exact && j >= 16 * I;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e] = zero ? 0.f : clip4(dv[e] * xv[e]) * __expf(CUM[16 * I * P + c + e] - CUM[j * P + c + e]);
      st_chunk8(buf + sw_off16(C, j, c), o);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0 && !flags[4]) {
      sm100::tc_fence_after();
      mma_steps(tmem + 128 + 16 * I, [&](int k) { return mndesc(buf, C, k); },
                [&](int k) { return kdesc(S + S1_CB + 2048 * I, C, k); }, I + 1, sm100::idesc_bf16(64, 16, true, false),
                false);
      sm100::umma_commit(bars + 3 + I);
    }
  }
  if (!wait_bar(bars + 2, 0, err, 0x5304) || !wait_bar(bars + 5, 0, err, 0x5304) || !wait_bar(bars + 6, 0, err, 0x5304))
    flags[4] = 1;
  sm100::tc_fence_after();
  __syncthreads();
  if (flags[4]) goto s1_teardown;
  {
    // S_end^T rows (lane = state row s) -> tile image (rows s, columns p)
    const int s = 32 * warp + lane;
    unsigned char* dst = send_t + ch * T_NP;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float x[32];
      tmem_ld32(tmem_at(tmem, warp, 64 + 32 * half), x);
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float y[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = clip4(x[c + e]);
        *reinterpret_cast<uint4*>(dst + sw_off16(N, s, 32 * half + c)) = pack8(y);
      }
    }
    // y_diag^T row p (lanes 0-15 of each quarter): fp32 rows into the dead W buffers, then the
    // exact diagonal sums where needed, then bf16 rows out
    float* YD = reinterpret_cast<float*>(smem + S1_W0);  // [p][i]
    const int p = 16 * warp + lane;
    float y[64];
    tmem_ld32(tmem_at(tmem, warp, 128), y);
    tmem_ld32(tmem_at(tmem, warp, 160), y + 32);
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 64; ++i) YD[p * C + i] = y[i] * __expf(CUM[i * P + p] - CUM[(i & ~15) * P + p]);
      for (int I = 0; I < 4; ++I) {
        if (!flags[I]) continue;
        for (int i = 16 * I; i < 16 * I + 16; ++i) {
          float acc = 0.f;
          for (int j = 16 * I; j <= i; ++j) {
            const float cb = __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_CB + sw_off(C, i, j)));
            const float xv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_X + sw_off(C, j, p)));
            const float dv = __bfloat162float(*reinterpret_cast<const bf16*>(smem + S1_DT + sw_off(C, j, p)));
            acc += cb * clip4(dv * xv) * __expf(fmaxf(CUM[i * P + p] - CUM[j * P + p], -20.f));
          }
          YD[p * C + i] += acc;
        }
      }
      bf16* dst2 = yd_t + ch * (C * P) + p * C;
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = clip4(YD[p * C + c + e]);
        *reinterpret_cast<uint4*>(dst2 + c) = pack8(o);
      }
    }
    // decay e^{max(c, -20)} as a tile image (rows i, columns p)
#pragma unroll
    for (int it = 0; it < (C * P / 8) / S1_THREADS; ++it) {
      const int u_ = it * S1_THREADS + tid;
      const int i = u_ >> 3, c = (u_ & 7) << 3;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __expf(fmaxf(CUM[i * P + c + e], -20.f));
      *reinterpret_cast<uint4*>(dec_t + ch * T_CP + sw_off16(C, i, c)) = pack8(o);
    }
  }
s1_teardown:
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 256);
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
    const bf16* __restrict__ yd_t, const unsigned char* __restrict__ dec_t, const float* __restrict__ cl,
    int L, int H, int NC, const float* __restrict__ s0, bf16* __restrict__ y, unsigned char* __restrict__ sin_t,
    float* __restrict__ s_final, int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t Sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S2_BAR);  // full[2], mma
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
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
      if (sin_t) *reinterpret_cast<uint4*>(sin_t + c * T_NP + sw_off16(N, s, p)) = pack8(S + p);
    }
    fence_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      if (!wait_bar(bars + st, (n >> 1) & 1, err, 0x5311)) *abort_flag = 1;
      sm100::tc_fence_after();
      if (!*abort_flag)
        mma_steps(tmem, [&](int k) { return mndesc(Sb + S2_S, N, k); }, [&](int k) { return kdesc(sc, C, k); }, N / 16,
                  sm100::idesc_bf16(64, 64, true, false), false);
      sm100::umma_commit(bars + 2);
    }
    // carry the state: S <- clip(S e^{max(cl, -20)} + S_end)   (S_end^T row s from the image)
    const int p0 = 16 * warp + lane;  // channel of this lane in the y epilogue (lanes 0-15)
    uint4 ydr[8];
    if (lane < 16)
#pragma unroll
      for (int q8 = 0; q8 < 8; ++q8) ydr[q8] = *reinterpret_cast<const uint4*>(yd_t + c * (C * P) + p0 * C + 8 * q8);
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
    if (!wait_bar(bars + 2, n & 1, err, 0x5313)) *abort_flag = 1;
    sm100::tc_fence_after();
    {
      float yo[64];
      tmem_ld32(tmem_at(tmem, warp, 0), yo);
      tmem_ld32(tmem_at(tmem, warp, 32), yo + 32);
      if (lane < 16) {
        const unsigned char* dec = smem + st * S2_STAGE + T_CN + T_NP;
        bf16* Y = reinterpret_cast<bf16*>(smem + S2_Y);
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
          float yd[8];
          unpack8(ydr[q8], yd);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int i = 8 * q8 + e;
            const float dh = __bfloat162float(*reinterpret_cast<const bf16*>(dec + sw_off(C, i, p0)));
            Y[i * P + p0] = __float2bfloat16_rn(clip4(yd[e] + clip4(yo[i] * dh)));
          }
        }
      }
    }
    sm100::tc_fence_before();
    __syncthreads();
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
  if (*abort_flag && tid == 0) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 64);
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
constexpr int B1S_BAR = B1S_DYD + T_CP;
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
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
      *reinterpret_cast<uint4*>(dse_t + c * T_NP + sw_off16(N, s, p)) = pack8(G + p);
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
    sm100::tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;
    if (tid == 0 && it + 2 < NC) issue(it + 2);
  }
  if (ds0 && it == NC)
#pragma unroll
    for (int p = 0; p < P; ++p) ds0[(bh * P + p) * N + s] = G[p];
  if (*abort_flag && tid == 0) {
    const uint64_t t0 = sm100::globaltimer();
    while (sm100::globaltimer() - t0 < 2000000ull) {}
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (warp == 0) sm100::tmem_dealloc(tmem, 64);
}

template <class K>
int set_smem_tc(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess ? 0 : -3;
}

// S1 + S2 on the given scratch (per chunk-head: S_end^T image, y_diag^T rows, decay image, last
// cumsum; these are SSD_SCRATCH_PER_CHUNK_HEAD bytes in this order within one chunk-head's slot)
int ssd_forward(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, int B, int L, int H,
                unsigned char* send_t, bf16* yd_t, unsigned char* dec_t, float* cl, const float* s0, float* s_final,
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
  return ssd_forward(x, dt, A, Bm, Cm, B, L, H, (unsigned char*)send_t, (bf16*)yd_t, (unsigned char*)dec_t, cl, s0,
                     s_final, y, (unsigned char*)sin_t, err, st);
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
static_assert(T_NP + C * P * 2 + T_CP + P * 4 == (64 * 128 + 64) * 4, "scratch per chunk-head");
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
  bf16* yd_t = reinterpret_cast<bf16*>(send_t + chunk_heads * T_NP);
  unsigned char* dec_t = reinterpret_cast<unsigned char*>(yd_t) + chunk_heads * (C * P * 2);
  float* cl = reinterpret_cast<float*>(dec_t + chunk_heads * T_CP);
  const int rc = ssd_forward(x, dt, A, Bm, Cm, B, L, H, send_t, yd_t, dec_t, cl, nullptr, nullptr, y, nullptr, errp,
                             stream);
  if (rc == -4) return AHB_NOALLOC_ELAUNCH;
  return rc == 0 ? AHB_NOALLOC_OK : AHB_NOALLOC_ESETUP;
}
