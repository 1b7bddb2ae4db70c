// Label-smoothed cross entropy of the tied LM head without stored logits (reference
// `optimizer.py:244-312`).
//
// For row i with label y (label -100 = masked), z = clip(nan_to_num(bf16(h_i W^T)), +-1e4):
//   lse = log sum_v e^{z_v}
//   loss_i = (sp - sn) (lse - z_y) - sn (sum_v z_v - V lse),  sp = 1 - ls, sn = ls/(V-1)
//   d loss_i / d z_v = softmax_v - (sp - sn) [v == y] - sn
// The head GEMM's epilogue (moe_gemm.cu, EPI_CE_FWD) reduces each 256-column vocabulary tile of a
// row to (max, sum of e^{z - max}, z_y, sum z); this kernel combines a row's tiles into lse and its
// loss.  The backward recomputes the logits tile by tile (EPI_CE_BWD) into dlogits for the dh and
// dW GEMMs, one chunk of rows at a time.
#include "common.cuh"
#include "launchers.h"

using namespace ahb;

namespace {

constexpr int THREADS = 256, ROWS_PER_WARP = 4;

// one warp per row (four rows in turn); the block's losses and valid-row counts are summed
// before one atomic add each
__global__ void __launch_bounds__(THREADS) ce_combine_kernel(const float4* __restrict__ part, int ntiles,
                                                             const int64_t* __restrict__ labels, int64_t T, int V,
                                                             float ls, float* __restrict__ lse_out,
                                                             float* __restrict__ loss_sum, float* __restrict__ count) {
  __shared__ float sh_l[THREADS / 32], sh_c[THREADS / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const float sn = ls > 0.f ? ls / (float)(V - 1) : 0.f;
  const float sp = 1.f - ls;
  float wl = 0.f, wc = 0.f;
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    const int64_t row = ((int64_t)blockIdx.x * (THREADS / 32) + wid) * ROWS_PER_WARP + r;
    if (row >= T) break;
    const float4* pr = part + row * ntiles;
    float m = -INFINITY, s = 0.f, zy = 0.f, zs = 0.f;
    for (int t = lane; t < ntiles; t += 32) {
      const float4 q = pr[t];
      const float mm = fmaxf(m, q.x);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (q.x == -INFINITY ? 0.f : q.y * __expf(q.x - mm));
      m = mm;
      zy += q.z;
      zs += q.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
      m = mm;
    }
    zy = warp_sum(zy);
    zs = warp_sum(zs);
    if (lane == 0) {
      const float lse = m + logf(s);
      lse_out[row] = lse;
      if (labels[row] != -100) {
        const float nll = lse - zy;
        wl += ls > 0.f ? nll * (sp - sn) - sn * (zs - (float)V * lse) : nll;
        wc += 1.f;
      }
    }
  }
  if (lane == 0) {
    sh_l[wid] = wl;
    sh_c[wid] = wc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float l = 0.f, c = 0.f;
    for (int w = 0; w < THREADS / 32; ++w) {
      l += sh_l[w];
      c += sh_c[w];
    }
    if (c > 0.f) {
      atomicAdd(loss_sum, l);
      atomicAdd(count, c);
    }
  }
}

}  // namespace

void ahb_ce_combine(const void* partials, int ntiles, const int64_t* labels, int64_t T, int V, float ls, float* lse,
                    float* loss_sum, float* count, cudaStream_t st) {
  if (T == 0) return;
  const int64_t rows_per_block = (THREADS / 32) * ROWS_PER_WARP;
  ce_combine_kernel<<<(unsigned)((T + rows_per_block - 1) / rows_per_block), THREADS, 0, st>>>(
      (const float4*)partials, ntiles, labels, T, V, ls, lse, loss_sum, count);
}
