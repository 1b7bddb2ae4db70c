// Fused optimizer step over the owned shard of the flat parameter store
// (reference `train_setup.py:490-550` apply step + `optimizer.py:84-239`).
//
// optim_prepare: avg = grad/n_accum; sum(avg^2) (global norm, NaN-propagating);
//   per diagnostic-group non-finite flags; g = nan_to_num(avg, 0) * grad_scale;
//   sum(g^2) (the clip_by_global_norm input); was_clipped = any |p| >= 100.
// optim_apply: per segment label -- muon (direction precomputed), lion,
//   adamw (decay / no decay), frozen -- then clip +-100 + nan_to_num, the
//   router_temp decay-to-init and the expert_bias sign update, and writes the
//   fp32 master plus the compute copy (bf16 or fp32) in the same pass.
// Blocks cover CHUNK elements of one segment; a block finds its segment by
// binary search over the per-segment chunk prefix.
//
// Data parallelism over NVLink peer memory: given the table of every rank's
// full-size gradient buffer, prepare sums the owned slice over the ranks while
// it reads it (the reduce-scatter fused into the first pass; the sum is written
// to the local slice for apply), and given the table of every rank's compute
// buffer, apply stores each updated weight into all of them (the all-gather
// fused into the update).  Plain loads/stores only; the caller orders the
// phases with peer barriers.
#include "common.cuh"
#include "launchers.h"

using namespace ahb;
using bf16 = __nv_bfloat16;

namespace {

constexpr int CHUNK = 4096;
constexpr int THREADS = 256;

AHB_DEVICE int find_seg(const int* cstart, int S, int b) {
  int lo = 0, hi = S;  // cstart[lo] <= b < cstart[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cstart[mid] <= b) lo = mid; else hi = mid;
  }
  return lo;
}

AHB_DEVICE void put_g(float* p, float v) { *p = v; }
AHB_DEVICE void put_g(bf16* p, float v) { *p = __float2bfloat16_rn(v); }

// G: gradient element type (fp32, or bf16 for a store whose accumulators are 16-bit)
template <typename G>
__global__ void __launch_bounds__(THREADS) optim_prepare_kernel(const AhbSegInfo* __restrict__ segs,
                                                                const int* __restrict__ cstart, int S,
                                                                G* __restrict__ grad,
                                                                const float* __restrict__ master, float inv,
                                                                double* __restrict__ red, int* __restrict__ flags,
                                                                const float* const* __restrict__ gpeers, int npeers,
                                                                int64_t lo) {
  __shared__ float sh[THREADS / 32];
  const int b = blockIdx.x;
  const int s = find_seg(cstart, S, b);
  const AhbSegInfo sg = segs[s];
  const int64_t base = (int64_t)(b - cstart[s]) * CHUNK;
  const int64_t rem = sg.len - base;
  const int n = (int)(rem < CHUNK ? rem : CHUNK);
  float sa = 0.f, sgq = 0.f;
  int nonfin = 0, clipped = 0;
  const bool rg = sg.flags & AHB_SEG_REQUIRES_GRAD;
  for (int i = threadIdx.x; i < n; i += THREADS) {
    const int64_t idx = sg.off + base + i;
    if (rg) {
      float a;
      if (npeers > 0) {
        a = 0.f;
        for (int r = 0; r < npeers; ++r) a += gpeers[r][lo + idx];
        a *= inv;
      } else {
        a = to_f(grad[idx]) * inv;
      }
      sa += a * a;
      const bool fin = isfinite(a);
      nonfin |= !fin;
      const float g = (fin ? a : 0.f) * sg.gscale;
      put_g(grad + idx, g);
      sgq += g * g;
    }
    clipped |= fabsf(master[idx]) >= 100.f;
  }
  sa = block_sum(sa, sh);
  sgq = block_sum(sgq, sh);
  if (threadIdx.x == 0) {
    atomicAdd(red, (double)sa);
    atomicAdd(red + 1, (double)sgq);
  }
  if (__syncthreads_or(clipped) && threadIdx.x == 0) atomicOr(flags, 1);
  if (__syncthreads_or(nonfin) && threadIdx.x == 0) atomicOr(flags + 1 + sg.group, 1);
}

AHB_DEVICE float signf_(float x) { return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f); }

template <typename G>
__global__ void __launch_bounds__(THREADS) optim_apply_kernel(const AhbSegInfo* __restrict__ segs,
                                                              const int* __restrict__ cstart, int S,
                                                              float* __restrict__ master, float* __restrict__ m,
                                                              float* __restrict__ v, const G* __restrict__ grad,
                                                              const float* __restrict__ coef_p,
                                                              uint16_t* __restrict__ compute,
                                                              const float* __restrict__ frac, int fracE,
                                                              AhbOptimArgs a, uint16_t* const* __restrict__ cpeers,
                                                              int npeers) {
  const int b = blockIdx.x;
  const int s = find_seg(cstart, S, b);
  const AhbSegInfo sg = segs[s];
  const int64_t base = (int64_t)(b - cstart[s]) * CHUNK;
  const int64_t rem = sg.len - base;
  const int n = (int)(rem < CHUNK ? rem : CHUNK);
  const float coef = *coef_p;
  const int lab = sg.label;
  const float lr = a.lr[lab], wd = a.wd[lab];
  const bool rg = sg.flags & AHB_SEG_REQUIRES_GRAD;
  for (int i = threadIdx.x; i < n; i += THREADS) {
    const int64_t j = base + i;
    const int64_t idx = sg.off + j;
    float p = master[idx];
    if (lab == AHB_LABEL_MUON) {
      if (rg) p += -lr * to_f(grad[idx]) - lr * wd * p;
    } else if (lab == AHB_LABEL_LION) {
      if (rg) {
        const float g = to_f(grad[idx]) * coef;
        const float mm = m[idx];
        const float u = signf_(0.1f * g + 0.9f * mm) + wd * p;
        m[idx] = 0.99f * mm + 0.01f * g;
        p -= lr * u;
      }
    } else if (lab == AHB_LABEL_ADAMW_DECAY || lab == AHB_LABEL_ADAMW_NODECAY) {
      const float g = rg ? to_f(grad[idx]) * coef : 0.f;
      const float mm = 0.9f * m[idx] + 0.1f * g;
      const float vv = 0.999f * v[idx] + 0.001f * g * g;
      m[idx] = mm;
      v[idx] = vv;
      const float u = (mm / a.bc1) / (sqrtf(vv / a.bc2) + 1e-8f) + wd * p;
      p -= lr * u;
    }
    p = sanitize(p, 100.f);
    if (sg.flags & AHB_SEG_ROUTER_TEMP) p -= 0.02f * (p - 10.f);
    if ((sg.flags & AHB_SEG_EXPERT_BIAS) && frac) {
      const float f = frac[(int64_t)sg.bias_row * fracE + j];
      p += 0.02f * (f > 1.f / (float)sg.len ? -1.f : 1.f);
    }
    master[idx] = p;
    if (npeers > 0) {
      if (sg.flags & AHB_SEG_COMPUTE_FP32)
        for (int r = 0; r < npeers; ++r) reinterpret_cast<float*>(cpeers[r] + sg.coff)[j] = p;
      else {
        const bf16 pb = __float2bfloat16_rn(p);
        for (int r = 0; r < npeers; ++r) reinterpret_cast<bf16*>(cpeers[r] + sg.coff)[j] = pb;
      }
    } else if (sg.flags & AHB_SEG_COMPUTE_FP32) {
      reinterpret_cast<float*>(compute + sg.coff)[j] = p;
    } else {
      reinterpret_cast<bf16*>(compute + sg.coff)[j] = __float2bfloat16_rn(p);
    }
  }
}

// Muon's Newton-Schulz step after its two GEMMs (reference optimizer.py:65-75): X <- 1.5 X - 0.5 Y
// in fp32, a non-finite result set to zero (the reference's nan_to_num after every step), and the
// bf16 image of X that the next step's GEMMs read.  Without Y it only writes the image.  Four
// elements per thread (the matrices are multiples of 64 columns).
__global__ void __launch_bounds__(THREADS) ns_update_kernel(float* __restrict__ X, const bf16* __restrict__ Y,
                                                            bf16* __restrict__ Xb, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)THREADS + threadIdx.x; i < n4; i += (int64_t)gridDim.x * THREADS) {
    float4 x = reinterpret_cast<float4*>(X)[i];
    float v[4] = {x.x, x.y, x.z, x.w};
    if (Y) {
      const uint2 yr = reinterpret_cast<const uint2*>(Y)[i];
      const bf16* y = reinterpret_cast<const bf16*>(&yr);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float t = 1.5f * v[k] - 0.5f * __bfloat162float(y[k]);
        v[k] = isfinite(t) ? t : 0.f;
      }
      reinterpret_cast<float4*>(X)[i] = make_float4(v[0], v[1], v[2], v[3]);
    }
    __align__(8) bf16 o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __float2bfloat16_rn(v[k]);
    reinterpret_cast<uint2*>(Xb)[i] = *reinterpret_cast<const uint2*>(o);
  }
}

}  // namespace

void ahb_optim_prepare(const AhbSegInfo* segs, const int* cstart, int S, int nblocks, void* grad, bool grad_bf16,
                       const float* master, float inv, double* red, int* flags, const float* const* gpeers,
                       int npeers, int64_t lo, cudaStream_t st) {
  if (nblocks <= 0) return;
  if (grad_bf16)
    optim_prepare_kernel<bf16><<<nblocks, THREADS, 0, st>>>(segs, cstart, S, (bf16*)grad, master, inv, red, flags,
                                                            gpeers, npeers, lo);
  else
    optim_prepare_kernel<float><<<nblocks, THREADS, 0, st>>>(segs, cstart, S, (float*)grad, master, inv, red, flags,
                                                             gpeers, npeers, lo);
}

void ahb_optim_apply(const AhbSegInfo* segs, const int* cstart, int S, int nblocks, float* master, float* m, float* v,
                     const void* grad, bool grad_bf16, const float* coef, void* compute, const float* frac, int fracE,
                     AhbOptimArgs args, void* const* cpeers, int npeers, cudaStream_t st) {
  if (nblocks <= 0) return;
  if (grad_bf16)
    optim_apply_kernel<bf16><<<nblocks, THREADS, 0, st>>>(segs, cstart, S, master, m, v, (const bf16*)grad, coef,
                                                          (uint16_t*)compute, frac, fracE, args,
                                                          (uint16_t* const*)cpeers, npeers);
  else
    optim_apply_kernel<float><<<nblocks, THREADS, 0, st>>>(segs, cstart, S, master, m, v, (const float*)grad, coef,
                                                           (uint16_t*)compute, frac, fracE, args,
                                                           (uint16_t* const*)cpeers, npeers);
}

int ahb_optim_chunk() { return CHUNK; }

void ahb_ns_update(float* X, const void* Y, void* Xb, int64_t n, int num_sms, cudaStream_t st) {
  const int64_t n4 = n / 4;
  if (n4 <= 0) return;
  const int64_t want = (n4 + THREADS - 1) / THREADS;
  const int grid = (int)(want < (int64_t)num_sms * 8 ? want : (int64_t)num_sms * 8);
  ns_update_kernel<<<grid, THREADS, 0, st>>>(X, static_cast<const bf16*>(Y), static_cast<bf16*>(Xb), n4);
}
