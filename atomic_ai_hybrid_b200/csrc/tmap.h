// Host-side TMA tensor-map encoding (driver entry point looked up through the runtime).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ahb {

typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline TmapEncodeFn tmap_encode_fn() {
  static TmapEncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TmapEncodeFn>(p);
  }
  return fn;
}

// bf16 tensor (B, L, H, D) as a 3-D map {D, H, B*L}; box {64, 1, box_t} with 128-byte swizzle:
// one box is a box_t x 64 tile of one head, landing as a swizzled 64-column slab.
inline int tmap_seq_bf16(CUtensorMap* m, const void* ptr, int64_t BL, int64_t H, int64_t D, int box_t) {
  TmapEncodeFn fn = tmap_encode_fn();
  if (!fn || !ptr) return -1;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)BL};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(H * D * 2)};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_t};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

}  // namespace ahb

namespace ahb {

// bf16 row-major (rows, cols) matrix as a 2-D map; box {64, box_rows} with 128-byte swizzle
// (one box = a box_rows x 64 slab).
inline int tmap_2d_bf16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  TmapEncodeFn fn = tmap_encode_fn();
  if (!fn || !ptr) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

}  // namespace ahb
