// Expert-parallel token exchange over NVLink peer memory (no counterpart in the
// reference, whose experts are replicated: `atomic_ops/moe_gmm.py:84-89` leaves EP
// as a follow-up).
//
// Each rank owns E/W consecutive experts.  Every rank has three peer-mapped
// buffers: a receive buffer of token rows grouped by (local expert, source rank),
// a row-metadata array (source rank, assignment index) for those rows, and a
// return buffer of rows in its own assignment order a = j*T + t.
//
// * ep_publish: write this rank's per-expert assignment counts into slot `rank`
//   of every peer's count table (the host then derives the receive layout).
// * ep_dispatch: for assignment a with expert e -> rank r = e / El, store the
//   source row (x[a % T], or rows[a]) at row dst_base[e] + rank_in_expert(a) of
//   rank r's receive buffer, and the metadata beside it.  One warp per row,
//   16-byte stores straight into the peer's memory.
// * ep_return: every received row with metadata (s, a) is stored into row a of
//   rank s's return buffer (the combine direction).
// * ep_zero_pad: zero the padding rows of the local receive buffer so that the
//   grouped GEMM tiles and the weight-gradient sums see zeros there.
// Ordering between phases is the caller's (peer barriers).  Only ordinary
// loads/stores touch peer memory.
#include <cstdint>
#include "common.cuh"
#include "launchers.h"

namespace {

__global__ void ep_publish_kernel(const int* __restrict__ counts, int E, int* const* __restrict__ peers, int W,
                                  int rank) {
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) {
    const int r = i / E, e = i % E;
    peers[r][rank * E + e] = counts[e];
  }
}

// one warp per assignment a
__global__ void ep_dispatch_kernel(const uint4* __restrict__ src, int src_by_token, int T, int k, int d16,
                                   const int* __restrict__ eidx, const int* __restrict__ pos_local,
                                   const int* __restrict__ off_local, const int* __restrict__ dst_base, int El,
                                   uint4* const* __restrict__ recv_peers, int2* const* __restrict__ meta_peers,
                                   int rank, int* __restrict__ dst_pos) {
  const int64_t a = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (a >= (int64_t)T * k) return;
  const int lane = threadIdx.x & 31;
  const int e = eidx[a];
  const int r = e / El;
  const int p = dst_base[e] + (pos_local[a] - off_local[e]);
  const uint4* s = src + (src_by_token ? (a % T) : a) * d16;
  uint4* dst = recv_peers[r] + (int64_t)p * d16;
  for (int c = lane; c < d16; c += 32) dst[c] = s[c];
  if (lane == 0) {
    if (meta_peers) meta_peers[r][p] = make_int2(rank, (int)a);
    if (dst_pos) dst_pos[a] = p;
  }
}

// rows of the local buffer -> row meta.y of rank meta.x's return buffer
__global__ void ep_return_kernel(const uint4* __restrict__ rows, const int2* __restrict__ meta, int64_t R, int d16,
                                 uint4* const* __restrict__ ret_peers) {
  const int64_t p = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (p >= R) return;
  const int2 m = meta[p];
  if (m.x < 0) return;
  const uint4* s = rows + p * d16;
  uint4* dst = ret_peers[m.x] + (int64_t)m.y * d16;
  for (int c = threadIdx.x & 31; c < d16; c += 32) dst[c] = s[c];
}

// zero rows [off[e] + seg[e], off[e + 1]) of each local expert segment; meta of those rows = -1
__global__ void ep_zero_pad_kernel(uint4* __restrict__ rows, int2* __restrict__ meta, const int* __restrict__ off,
                                   const int* __restrict__ seg, int El, int d16) {
  const int e = blockIdx.x;
  const int64_t b = (int64_t)off[e] + seg[e], end = off[e + 1];
  for (int64_t p = b; p < end; ++p) {
    for (int c = threadIdx.x; c < d16; c += blockDim.x) rows[p * d16 + c] = make_uint4(0, 0, 0, 0);
    if (meta && threadIdx.x == 0) meta[p] = make_int2(-1, -1);
  }
}

int rows_grid(int64_t rows) { return (int)((rows + 7) / 8); }

}  // namespace

void ahb_ep_publish(const int* counts, int E, int* const* peers_dev, int W, int rank, cudaStream_t st) {
  ep_publish_kernel<<<1, 256, 0, st>>>(counts, E, peers_dev, W, rank);
}

void ahb_ep_dispatch(const void* src, int src_by_token, int T, int k, int d, const int* eidx, const int* pos_local,
                     const int* off_local, const int* dst_base, int El, void* const* recv_peers,
                     void* const* meta_peers, int rank, int* dst_pos, cudaStream_t st) {
  const int64_t n = (int64_t)T * k;
  if (n == 0) return;
  ep_dispatch_kernel<<<rows_grid(n), 256, 0, st>>>((const uint4*)src, src_by_token, T, k, d / 8, eidx, pos_local,
                                                   off_local, dst_base, El, (uint4* const*)recv_peers,
                                                   (int2* const*)meta_peers, rank, dst_pos);
}

void ahb_ep_return(const void* rows, const void* meta, int64_t R, int d, void* const* ret_peers, cudaStream_t st) {
  if (R == 0) return;
  ep_return_kernel<<<rows_grid(R), 256, 0, st>>>((const uint4*)rows, (const int2*)meta, R, d / 8,
                                                 (uint4* const*)ret_peers);
}

void ahb_ep_zero_pad(void* rows, void* meta, const int* off, const int* seg, int El, int d, cudaStream_t st) {
  if (El == 0) return;
  ep_zero_pad_kernel<<<El, 256, 0, st>>>((uint4*)rows, (int2*)meta, off, seg, El, d / 8);
}
