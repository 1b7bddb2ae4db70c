// Data-parallel collectives over NVLink / NVSwitch peer memory.
//
// Buffers are plain cudaMalloc allocations shared between the ranks of one node
// through CUDA IPC handles (one process per GPU); every rank holds the peer
// pointers of all ranks (its own included).  Peer memory is only touched with
// ordinary loads and stores -- no TMA, no multicast.
//
// * symm_barrier: thread r stores the epoch into slot `rank` of rank r's signal
//   pad (release, system scope) and then waits until slot r of its own pad holds
//   the epoch (acquire).  The wait is bounded by %globaltimer; on timeout the
//   kernel records 100 + r in the error word and returns.
// * reduce_scatter: out[i] = sum_r peers[r][lo + i] (fp32) -- used when the
//   optimizer runs in PyTorch ops; the fused path sums inside the optimizer's
//   prepare kernel instead (optim.cu).
// * copy_out: the local slice [off, off + n) is stored at the same offset of
//   every peer buffer -- the stand-alone all-gather; the fused path stores from
//   the optimizer's apply kernel.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include "common.cuh"
#include "launchers.h"

namespace {

AHB_DEVICE uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
AHB_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
AHB_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void symm_barrier_kernel(uint32_t* const* __restrict__ pads, int rank, int world, uint32_t epoch,
                                    int* __restrict__ err, uint64_t timeout_ns) {
  const int r = threadIdx.x;
  if (r >= world) return;
  __threadfence_system();
  st_release_sys(pads[r] + rank, epoch);
  const uint32_t* mine = pads[rank] + r;
  const uint64_t t0 = gtimer();
  // epochs only grow; the signed difference tolerates wrap-around
  while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
    if (gtimer() - t0 > timeout_ns) {
      atomicCAS(err, 0, 100 + r);
      return;
    }
    __nanosleep(64);
  }
}

// `out` may be this rank's own slice of the summed buffers (in-place reduce)
__global__ void rs_kernel(const float* const* __restrict__ peers, int world, int64_t lo, int64_t n4, float* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 v = reinterpret_cast<const float4*>(peers[r] + lo)[i];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = s;
  }
}

__global__ void copy_out_kernel(const uint4* __restrict__ src, uint4* const* __restrict__ peers, int world,
                                int64_t off16, int64_t n16) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    for (int r = 0; r < world; ++r) peers[r][off16 + i] = v;
  }
}

// out[i] = sum_s slots[s * stride + i] (bf16 in, fp32 sum in slot order, bf16 out); 8 per thread
__global__ void sum_slots_kernel(const uint4* __restrict__ slots, int nslots, int64_t stride16, int64_t n16,
                                 uint4* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < nslots; ++s) {
      const uint4 v = slots[s * stride16 + i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        a[2 * j] += f.x;
        a[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
    out[i] = o;
  }
}

int grid_for(int64_t n) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t b = (n + 255) / 256;
  const int64_t cap = (int64_t)sms * 8;
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace

int ahb_ipc_alloc(int64_t nbytes, void** ptr) {
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, (size_t)nbytes);
  if (e != cudaSuccess) {
    fprintf(stderr, "ahb_ipc_alloc(%lld): %s\n", (long long)nbytes, cudaGetErrorString(e));
    return -1;
  }
  e = cudaMemset(*ptr, 0, (size_t)nbytes);
  return e == cudaSuccess ? 0 : -1;
}

int ahb_ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : -1; }

int ahb_ipc_handle(void* ptr, void* handle64) {
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return -1;
  memcpy(handle64, &h, sizeof(h));
  return 0;
}

int ahb_ipc_open(const void* handle64, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    fprintf(stderr, "ahb_ipc_open: %s\n", cudaGetErrorString(e));
    return -1;
  }
  return 0;
}

int ahb_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : -1; }

void ahb_symm_barrier(uint32_t* const* pads_dev, int rank, int world, uint32_t epoch, int* err, double timeout_s,
                      cudaStream_t st) {
  symm_barrier_kernel<<<1, 32, 0, st>>>(pads_dev, rank, world, epoch, err, (uint64_t)(timeout_s * 1e9));
}

void ahb_reduce_scatter_f32(const float* const* peers_dev, int world, int64_t lo, int64_t n, float* out,
                            cudaStream_t st) {
  const int64_t n4 = n / 4;
  if (n4 == 0) return;
  rs_kernel<<<grid_for(n4), 256, 0, st>>>(peers_dev, world, lo, n4, out);
}

void ahb_copy_out(const void* src, void* const* peers_dev, int world, int64_t off_bytes, int64_t nbytes,
                  cudaStream_t st) {
  const int64_t n16 = nbytes / 16;
  if (n16 == 0) return;
  copy_out_kernel<<<grid_for(n16), 256, 0, st>>>((const uint4*)src, (uint4* const*)peers_dev, world, off_bytes / 16,
                                                 n16);
}

void ahb_sum_slots_bf16(const void* slots, int nslots, int64_t stride, int64_t n, void* out, cudaStream_t st) {
  const int64_t n16 = n / 8;
  if (n16 == 0) return;
  sum_slots_kernel<<<grid_for(n16), 256, 0, st>>>((const uint4*)slots, nslots, stride / 8, n16, (uint4*)out);
}

int ahb_memcpy_async(void* dst, const void* src, int64_t nbytes, cudaStream_t st) {
  return cudaMemcpyAsync(dst, src, (size_t)nbytes, cudaMemcpyDefault, st) == cudaSuccess ? 0 : -1;
}
