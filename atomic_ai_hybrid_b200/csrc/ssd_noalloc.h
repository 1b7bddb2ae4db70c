// Allocation-free entry point of the Mamba2 SSD forward.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that must not allocate device memory while they run:
// code that executes while another framework is capturing a CUDA graph in a
// mode where cudaMalloc is illegal, serving engines that reserve all HBM at
// start-up and forbid later allocations, and allocator or stream callbacks that
// would re-enter their own allocator.  The caller passes inputs and the output
// buffer; the chunk-state scratch the forward needs comes from a fixed array in
// device memory that every GPU loading this library holds until process exit.
//
//   Limit: B * H * (L / 64) <= AHB_SSD_NOALLOC_MAX_CHUNK_HEADS (the 32 MiB scratch holds,
//   per (batch, head, chunk), the chunk's end state and decay factors in bf16, its intra-chunk
//   output in fp32 and its 64 last decay sums: 41,216 bytes, so 814 chunk-heads).
//   Shapes: x, dt (B, L, H, 64) bf16; A (H,) fp32; Bm, Cm (B, L, 128) bf16;
//   y (B, L, H, 64) bf16; L a multiple of 64; all pointers on the current device.
//
// The first call on each device looks up the device addresses of the scratch array and
// of a fixed timeout word (cudaGetSymbolAddress) and sets the kernels' shared-memory
// limits; make that first call before any stream capture begins.  Every call shares the one
// scratch array, so calls whose executions overlap on the GPU (different
// streams without ordering, or concurrent host threads) race on it; calls
// ordered on one stream are safe.  Nothing in the scratch needs to start at
// zero: the forward writes every element it later reads.
#pragma once
#include <cuda_runtime.h>

#define AHB_NOALLOC_OK 0
#define AHB_NOALLOC_EINVAL -1   // null pointer or invalid shape
#define AHB_NOALLOC_ETOOBIG -2  // problem needs more scratch than the fixed array holds
#define AHB_NOALLOC_ESETUP -3   // device query / symbol lookup failed
#define AHB_NOALLOC_ELAUNCH -4  // a kernel launch of this call failed
#define AHB_NOALLOC_EPENDING -5  // a CUDA error from earlier work was pending on entry (left uncleared)
#define AHB_SSD_NOALLOC_SCRATCH_BYTES (32u << 20)
#define AHB_SSD_NOALLOC_BYTES_PER_CHUNK_HEAD (128u * 64u * 2u + 64u * 64u * 4u + 64u * 64u * 2u + 64u * 4u)
#define AHB_SSD_NOALLOC_MAX_CHUNK_HEADS (AHB_SSD_NOALLOC_SCRATCH_BYTES / AHB_SSD_NOALLOC_BYTES_PER_CHUNK_HEAD)

#ifdef __cplusplus
extern "C" {
#endif
int ahb_ssd_fwd_noalloc(const void* x, const void* dt, const float* A, const void* Bm, const void* Cm, int B, int L,
                        int H, void* y, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
