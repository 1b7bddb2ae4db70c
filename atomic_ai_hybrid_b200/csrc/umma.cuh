// Shared-memory operand tiles and tcgen05 helpers for the chunked-scan kernels.
//
// Operand tiles are bf16, stored in the 128-byte-swizzled canonical layout that
// tcgen05.mma reads through a shared-memory descriptor:
//   a tile of R rows x K columns is K/64 "slabs" of R x 128 bytes; inside a slab,
//   8-row groups of 1024 bytes; 16-byte chunk c of row r sits at chunk c ^ (r % 8).
// The same bytes serve two roles:
//   * K-major operand  (rows = M or N, columns = K): K-step s (16 columns) starts at
//     slab s/4, byte 32*(s%4) of the row; SBO = 1024.
//   * MN-major operand (rows = K, columns = M or N): K-step s starts at row 16*s
//     (byte 2048*s); LBO = slab stride (distance between 64-column groups), SBO = 1024.
// Threads write such tiles with st.shared and make them visible to the tensor core
// with fence.proxy.async before the issuing thread's barrier.
//
// Accumulator (TMEM) layout, cta_group::1: for M = 128, row m is lane m; for M = 64,
// row 16*q + r is lane 32*q + r (the first 16 lanes of each 32-lane quarter).  Column n
// is column n in both cases.  A warp reads the lanes of its own quarter (warp % 4).
#pragma once
#include <cuda.h>
#include <cstdint>
#include "common.cuh"
#include "sm100.cuh"

namespace ahb {
namespace umma {

using bf16 = __nv_bfloat16;
using sm100::smem_u32;

// byte offset of element (row, col) in an R-row swizzled bf16 tile
AHB_DEVICE uint32_t sw_off(int R, int row, int col) {
  return (uint32_t)((col >> 6) * (R * 128) + (row >> 3) * 1024 + (row & 7) * 128 +
                    ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}
// byte offset of the 16-byte chunk holding columns [c8, c8 + 8) of `row`
AHB_DEVICE uint32_t sw_off16(int R, int row, int c8) {
  return (uint32_t)((c8 >> 6) * (R * 128) + (row >> 3) * 1024 + (row & 7) * 128 + ((((c8 & 63) >> 3) ^ (row & 7)) << 4));
}

// Shared-memory matrix descriptors (128-byte swizzle) for K step s.  The start-address field is
// (base >> 4) plus the step's offset >> 4, masked to its 14 bits (both are multiples of 16; a base
// shifted below the window by whole K steps wraps and comes back in the sum); written this way a
// fully unrolled step loop costs an add and a mask per descriptor instead of rebuilding it from the
// byte address.
AHB_DEVICE uint64_t desc_const(uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
AHB_DEVICE uint64_t kdesc(uint32_t base, int R, int s) {
  return desc_const(16, 1024) |
         static_cast<uint64_t>(((base >> 4) + (uint32_t)(((s >> 2) * R * 128 + (s & 3) * 32) >> 4)) & 0x3FFFu);
}
AHB_DEVICE uint64_t mndesc(uint32_t base, int Krows, int s) {
  return desc_const((uint32_t)(Krows * 128), 1024) | static_cast<uint64_t>(((base >> 4) + (uint32_t)(s * 128)) & 0x3FFFu);
}

// 8 consecutive fp32 of a shared-memory row as two 16-byte loads, the halves in swapped order on
// lanes with bit 2 set: where 8 or 16 lanes read consecutive 32-byte pieces of a row, each load then
// meets every bank group once per row instead of half of them twice
AHB_DEVICE void ld8f_x(const float* src, float* o) {
  const int sw = (threadIdx.x >> 2) & 1;
  const float4 a = *reinterpret_cast<const float4*>(src + 4 * sw);
  const float4 b = *reinterpret_cast<const float4*>(src + 4 - 4 * sw);
  const float4 lo = sw ? b : a, hi = sw ? a : b;
  o[0] = lo.x; o[1] = lo.y; o[2] = lo.z; o[3] = lo.w; o[4] = hi.x; o[5] = hi.y; o[6] = hi.z; o[7] = hi.w;
}

// 16-byte asynchronous copy global -> shared that holds no registers; cp_async_wait_all waits for
// this thread's copies
AHB_DEVICE void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
AHB_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

AHB_DEVICE void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

AHB_DEVICE uint32_t pack_bf2(float a, float b) {
  __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&p);
}
AHB_DEVICE void st_shared16(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// 8 floats -> one swizzled 16-byte chunk
AHB_DEVICE void st_chunk8(uint32_t addr, const float* v) {
  st_shared16(addr, pack_bf2(v[0], v[1]), pack_bf2(v[2], v[3]), pack_bf2(v[4], v[5]), pack_bf2(v[6], v[7]));
}
AHB_DEVICE void ld_shared16(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr) : "memory");
}
AHB_DEVICE void unpack8(uint4 w, float* v) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(p[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
AHB_DEVICE uint4 pack8(const float* v) {
  uint4 w;
  w.x = pack_bf2(v[0], v[1]);
  w.y = pack_bf2(v[2], v[3]);
  w.z = pack_bf2(v[4], v[5]);
  w.w = pack_bf2(v[6], v[7]);
  return w;
}

// 16 consecutive fp32 columns of the warp's lanes
AHB_DEVICE void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
using sm100::tmem_ld32;

// TMEM address of column `col` in the lanes of warp quarter `q`
AHB_DEVICE uint32_t tmem_at(uint32_t base, int q, int col) { return base + ((uint32_t)(32 * q) << 16) + (uint32_t)col; }

// Issue D (+)= A x B^T over `ks` K-steps; A/B descriptors come from functors of the step.
template <class FA, class FB>
AHB_DEVICE void mma_steps(uint32_t d, FA&& fa, FB&& fb, int ks, uint32_t idesc, bool acc) {
#pragma unroll 8
  for (int s = 0; s < ks; ++s) sm100::umma_bf16(d, fa(s), fb(s), idesc, (acc || s > 0) ? 1u : 0u);
}

// 1-D bulk copy global -> shared (16-byte aligned, size multiple of 16), completion on `bar`
AHB_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 1-D bulk copy shared -> global (16-byte aligned, size multiple of 16) in the issuing thread's
// bulk group; bulk_commit closes the group, bulk_wait_read lets the thread reuse the source once
// the copies have read it, bulk_wait_all waits for the writes too
AHB_DEVICE void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
AHB_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
AHB_DEVICE void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
AHB_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 3-D TMA tile store from a swizzled shared-memory box (coordinates non-negative), in the issuing
// thread's bulk group
AHB_DEVICE void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// 3-D TMA tile load (no multicast)
AHB_DEVICE void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Bounded mbarrier wait for kernels without role-abort plumbing: records `code` in `err`
// and returns false after ~2 s.
AHB_DEVICE bool wait_bar(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (sm100::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = sm100::globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 0 && sm100::globaltimer() - t0 > 2000000000ull) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

}  // namespace umma
}  // namespace ahb
