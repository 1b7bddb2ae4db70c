// Shared helpers for the sm_100a kernels of atomic_ai_hybrid_b200.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#define AHB_DEVICE __device__ __forceinline__

namespace ahb {

AHB_DEVICE float to_f(float x) { return x; }
AHB_DEVICE float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> AHB_DEVICE T from_f(float x);
template <> AHB_DEVICE float from_f<float>(float x) { return x; }
template <> AHB_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

AHB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
AHB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `sh` needs blockDim.x/32 floats.  All threads get the result.
AHB_DEVICE float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  float t = lane < nw ? sh[lane] : 0.f;
  return warp_sum(t);
}

// nan_to_num(clip(x, -c, c)): NaN -> 0, +-inf -> +-c.
AHB_DEVICE float sanitize(float x, float c) {
  if (x != x) return 0.f;
  return fminf(fmaxf(x, -c), c);
}

AHB_DEVICE float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }
AHB_DEVICE float siluf_(float x) { return x * sigmoidf_(x); }
// softplus with the usual large-input cutoff (torch/jax agree to fp32 rounding)
AHB_DEVICE float softplusf_(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// 16-byte vector of 8 bf16
struct alignas(16) bf16x8 { __nv_bfloat162 v[4]; };

}  // namespace ahb
