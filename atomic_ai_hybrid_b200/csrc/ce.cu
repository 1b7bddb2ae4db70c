// Label-smoothed cross entropy over bf16 logit rows (reference `optimizer.py:244-312`).
//
// For row i with label y (label -100 = masked):
//   z = clip(nan_to_num(logits), +-1e4) in fp32; lse = log sum_v e^{z_v}
//   loss_i = (sp - sn) (lse - z_y) - sn (sum_v z_v - V lse),  sp = 1 - ls, sn = ls/(V-1)
//   d loss_i / d z_v = softmax_v - (sp - sn) [v == y] - sn
// The gradient overwrites the logits in place (bf16), so the LM-head backward
// GEMMs read it directly; masked rows get a zero gradient.  One CTA per row,
// two passes (online max/sum, then the gradient).
#include "common.cuh"
#include "launchers.h"

using bf16 = __nv_bfloat16;
using namespace ahb;

namespace {

constexpr int THREADS = 256;

AHB_DEVICE float clean(float x) { return sanitize(x, 1e4f); }

__global__ void __launch_bounds__(THREADS) ce_rows_kernel(bf16* __restrict__ logits, const int64_t* __restrict__ labels,
                                                          int V, float ls, float* __restrict__ loss_sum,
                                                          float* __restrict__ count) {
  __shared__ float sh_m[THREADS / 32], sh_s[THREADS / 32], sh_z[THREADS / 32];
  __shared__ float s_lse, s_sum;
  const int64_t row = blockIdx.x;
  bf16* z = logits + row * V;
  const int64_t lab = labels[row];
  const bool valid = lab != -100;
  const int y = (int)(lab < 0 ? 0 : (lab >= V ? V - 1 : lab));
  // pass 1: online max / sum-exp and plain sum
  float m = -INFINITY, s = 0.f, zs = 0.f;
  const int nv = V / 8;  // V % 8 == 0 (checked on the host)
  for (int i = threadIdx.x; i < nv; i += THREADS) {
    uint4 u = reinterpret_cast<const uint4*>(z)[i];
    const bf16* e = reinterpret_cast<const bf16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = clean(__bfloat162float(e[j]));
      zs += x;
      if (x > m) {
        s = s * __expf(m - x) + 1.f;
        m = x;
      } else {
        s += __expf(x - m);
      }
    }
  }
  // combine (m, s) across the block
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  zs = warp_sum(zs);
  if (lane == 0) { sh_m[wid] = m; sh_s[wid] = s; sh_z[wid] = zs; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY, Ssum = 0.f, Z = 0.f;
    for (int w = 0; w < THREADS / 32; ++w) M = fmaxf(M, sh_m[w]);
    for (int w = 0; w < THREADS / 32; ++w) {
      Ssum += sh_m[w] == -INFINITY ? 0.f : sh_s[w] * __expf(sh_m[w] - M);
      Z += sh_z[w];
    }
    s_lse = M + logf(Ssum);
    s_sum = Z;
  }
  __syncthreads();
  const float lse = s_lse;
  const float sn = ls > 0.f ? ls / (float)(V - 1) : 0.f;
  const float sp = 1.f - ls;
  if (threadIdx.x == 0) {
    if (valid) {
      const float zy = clean(__bfloat162float(z[y]));
      const float nll = lse - zy;
      const float l = ls > 0.f ? nll * (sp - sn) - sn * (s_sum - (float)V * lse) : nll;
      atomicAdd(loss_sum, l);
      atomicAdd(count, 1.f);
    }
  }
  __syncthreads();  // everyone has read z[y] before it is overwritten
  // pass 2: gradient in place
  for (int i = threadIdx.x; i < nv; i += THREADS) {
    uint4 u = reinterpret_cast<const uint4*>(z)[i];
    bf16* e = reinterpret_cast<bf16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float g = 0.f;
      if (valid) {
        const int v = i * 8 + j;
        g = __expf(clean(__bfloat162float(e[j])) - lse) - sn - (v == y ? (sp - sn) : 0.f);
      }
      e[j] = __float2bfloat16_rn(g);
    }
    reinterpret_cast<uint4*>(z)[i] = u;
  }
}

}  // namespace

void ahb_ce_rows(void* logits, const int64_t* labels, int64_t R, int V, float ls, float* loss_sum, float* count,
                 cudaStream_t st) {
  if (R == 0) return;
  ce_rows_kernel<<<(unsigned)R, THREADS, 0, st>>>((bf16*)logits, labels, V, ls, loss_sum, count);
}
