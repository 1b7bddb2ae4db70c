// Source-softmax mixing of the BlockDAR layers (reference `model.py:707-765`:
// IntraBlockAttention mixes the block input with the deltas of the earlier
// sublayers, HybridDARAttention mixes the history of block deltas):
//   score_i = scale * <q, k_i>,  w = softmax_i(score),  out = sum_i w_i s_i
// for n sources per token.  The projections q = Dense(x), k_i = Dense_i(s_i) stay
// library GEMMs; this kernel replaces the stack / multiply / sum / softmax /
// weighted-sum chain (one pass over the sources).  One warp per token; source and
// key pointers come in device tables (n <= 32).
// Backward (per token, g = d out): dot_i = <g, s_i>, dscore_i = w_i (dot_i - sum_j w_j dot_j),
//   d s_i = w_i g,  dq = scale sum_i dscore_i k_i,  d k_i = scale dscore_i q.
#include "common.cuh"
#include "launchers.h"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

constexpr int NMAX = 32;

__global__ void source_mix_fwd_kernel(const bf16* __restrict__ q, const bf16* const* __restrict__ ks,
                                      const bf16* const* __restrict__ ss, int n, int64_t T, int dl, int d,
                                      float scale, bf16* __restrict__ out, float* __restrict__ wts) {
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  float sc[NMAX];
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) {
    float p = 0.f;
    for (int c = lane; c < dl; c += 32) p += __bfloat162float(q[t * dl + c]) * __bfloat162float(ks[i][t * dl + c]);
    p = warp_sum(p) * scale;
    sc[i] = p;
    mx = fmaxf(mx, p);
  }
  float z = 0.f;
  for (int i = 0; i < n; ++i) {
    sc[i] = __expf(sc[i] - mx);
    z += sc[i];
  }
  for (int i = 0; i < n; ++i) {
    sc[i] /= z;
    if (lane == 0) wts[(int64_t)i * T + t] = sc[i];
  }
  for (int c = lane; c < d; c += 32) {
    float a = 0.f;
    for (int i = 0; i < n; ++i) a += sc[i] * __bfloat162float(ss[i][t * d + c]);
    out[t * d + c] = __float2bfloat16_rn(a);
  }
}

__global__ void source_mix_bwd_kernel(const bf16* __restrict__ g, const bf16* __restrict__ q,
                                      const bf16* const* __restrict__ ks, const bf16* const* __restrict__ ss,
                                      const float* __restrict__ wts, int n, int64_t T, int dl, int d, float scale,
                                      bf16* __restrict__ dq, bf16* const* __restrict__ dks,
                                      bf16* const* __restrict__ dss) {
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  float w[NMAX], ds[NMAX];
  float wd = 0.f;
  for (int i = 0; i < n; ++i) {
    w[i] = wts[(int64_t)i * T + t];
    float p = 0.f;
    for (int c = lane; c < d; c += 32) p += __bfloat162float(g[t * d + c]) * __bfloat162float(ss[i][t * d + c]);
    p = warp_sum(p);
    ds[i] = p;
    wd += w[i] * p;
  }
  for (int i = 0; i < n; ++i) ds[i] = w[i] * (ds[i] - wd) * scale;  // d score_i, times the score scale
  for (int c = lane; c < d; c += 32) {
    const float gv = __bfloat162float(g[t * d + c]);
    for (int i = 0; i < n; ++i) dss[i][t * d + c] = __float2bfloat16_rn(w[i] * gv);
  }
  for (int c = lane; c < dl; c += 32) {
    const float qv = __bfloat162float(q[t * dl + c]);
    float a = 0.f;
    for (int i = 0; i < n; ++i) {
      a += ds[i] * __bfloat162float(ks[i][t * dl + c]);
      dks[i][t * dl + c] = __float2bfloat16_rn(ds[i] * qv);
    }
    dq[t * dl + c] = __float2bfloat16_rn(a);
  }
}

}  // namespace

int ahb_source_mix_max() { return NMAX; }

void ahb_source_mix_fwd(const void* q, const void* const* ks, const void* const* ss, int n, int64_t T, int dl, int d,
                        float scale, void* out, float* wts, cudaStream_t st) {
  if (T <= 0) return;
  source_mix_fwd_kernel<<<(unsigned)((T + 7) / 8), 256, 0, st>>>((const bf16*)q, (const bf16* const*)ks,
                                                                 (const bf16* const*)ss, n, T, dl, d, scale,
                                                                 (bf16*)out, wts);
}

void ahb_source_mix_bwd(const void* g, const void* q, const void* const* ks, const void* const* ss, const float* wts,
                        int n, int64_t T, int dl, int d, float scale, void* dq, void* const* dks, void* const* dss,
                        cudaStream_t st) {
  if (T <= 0) return;
  source_mix_bwd_kernel<<<(unsigned)((T + 7) / 8), 256, 0, st>>>(
      (const bf16*)g, (const bf16*)q, (const bf16* const*)ks, (const bf16* const*)ss, wts, n, T, dl, d, scale,
      (bf16*)dq, (bf16* const*)dks, (bf16* const*)dss);
}
