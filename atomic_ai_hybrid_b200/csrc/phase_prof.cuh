// Per-phase cycle counters of the scan kernels (a diagnostic; off unless a buffer is set).
//
// Every translation unit that includes this header owns one device pointer.  The host points it at a
// zeroed uint64 array with the setter that AHB_PHASE_PROF_SETTER defines; thread 0 of every CTA then
// adds the SM cycles (clock64) between consecutive marks to the counter of each phase, and one to the
// kernel's CTA counter at the end.  Summed cycles over CTAs divided by the CTA count give the mean
// latency of each phase in one CTA.  With the pointer null (the default) a mark costs one predicated
// branch of thread 0.  The setter copies to a device symbol, so it is not called during capture.
#pragma once
#include <cuda_runtime.h>

namespace ahb {

static __device__ unsigned long long* g_phase_prof = nullptr;

struct PhaseClock {
  unsigned long long* p;
  long long t;
  __device__ __forceinline__ explicit PhaseClock(int base) {
    p = g_phase_prof;
    if (p) p += base;
    t = clock64();
  }
  // cycles since the previous mark -> counter k of this kernel's block of 16
  __device__ __forceinline__ void mark(int k) {
    if (p && threadIdx.x == 0) {
      const long long n = clock64();
      atomicAdd(p + k, (unsigned long long)(n - t));
      t = n;
    }
  }
  // lane 0 of every warp: cycles since `since` -> counter k + warp (a per-warp arrival time)
  __device__ __forceinline__ void warp_mark(int k, long long since) {
    if (p && (threadIdx.x & 31) == 0) atomicAdd(p + k + (threadIdx.x >> 5), (unsigned long long)(clock64() - since));
  }
  // counter 15: the number of CTAs that reached the end
  __device__ __forceinline__ void done() {
    if (p && threadIdx.x == 0) atomicAdd(p + 15, 1ull);
  }
};

}  // namespace ahb

#define AHB_PHASE_PROF_SETTER(fn)                                                                  \
  int fn(void* counters) {                                                                         \
    unsigned long long* ptr = static_cast<unsigned long long*>(counters);                          \
    return cudaMemcpyToSymbol(ahb::g_phase_prof, &ptr, sizeof(ptr)) == cudaSuccess ? 0 : -1;       \
  }
