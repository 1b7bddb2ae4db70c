// Raw-pointer launchers of the sm_100a kernels (no framework types).
// dtype codes: AHB_F32 = 0, AHB_BF16 = 1.  All launches go to `st`.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#define AHB_F32 0
#define AHB_BF16 1

// elementwise.cu
void ahb_sanitize(void* out, const void* in, int64_t n, int dtype, float clip, cudaStream_t st);
void ahb_rmsnorm_fwd(const void* x, const float* scale, void* y, float* rstd, int64_t M, int D, int dtype, float eps,
                     cudaStream_t st);
void ahb_rmsnorm_bwd(const void* dy, const void* x, const float* scale, const float* rstd, void* dx, float* dscale_acc,
                     int64_t M, int D, int dtype, cudaStream_t st);
void ahb_conv1d_fwd(const void* x, int64_t xs, const void* w, int wdtype, const float* bias, void* y, int B, int L,
                    int C, int dtype, int silu, float clip, cudaStream_t st);
void ahb_conv1d_bwd(const void* x, int64_t xs, const void* w, int wdtype, const float* bias, const void* dy, void* dx,
                    float* dw_acc, float* db_acc, int B, int L, int C, int dtype, int silu, float clip,
                    cudaStream_t st);
void ahb_accumulate(float* acc, const void* g, int64_t n, int dtype, float scale, cudaStream_t st);
void ahb_embedding_fwd(const int64_t* ids, const void* emb, int edtype, void* out, int odtype, int64_t T, int D,
                       int64_t V, cudaStream_t st);
void ahb_embedding_bwd(const int64_t* ids, const void* dout, int dtype, float* acc, int64_t T, int D, int64_t V,
                       cudaStream_t st);
