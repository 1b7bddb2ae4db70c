// Warp-level tensor-core tiles for the chunked scan kernels.
//
// The chunk-local products of the GDN-2 / SSD scans are small (64x64x128
// tiles) and their operands are transformed on the way in (per-channel decay
// factors e^{gc_i - gc_r}, gates, transposes), so they are issued as warp-wide
// m16n8k16 bf16 MMAs with fp32 accumulation, with operand fragments assembled by
// small "pair loader" functors:
//   A-loader  pa(r, c) -> bf16x2 of (A[r][c], A[r][c+1])
//   B-loader  pb(k, n) -> bf16x2 of (B[k][n], B[k+1][n])
// Accumulator element map of one 16x8 tile for lane (g = lane/4, t = lane%4):
//   c[0] = (g, 2t)  c[1] = (g, 2t+1)  c[2] = (g+8, 2t)  c[3] = (g+8, 2t+1)
#pragma once
#include "common.cuh"

namespace ahb {

AHB_DEVICE uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

AHB_DEVICE uint32_t pack2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  __nv_bfloat162 v;
  v.x = lo;
  v.y = hi;
  return *reinterpret_cast<uint32_t*>(&v);
}

AHB_DEVICE void mma16816(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <class FA>
AHB_DEVICE void load_a(uint32_t a[4], const FA& fa, int m0, int k0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  a[0] = fa(m0 + g, k0 + 2 * t);
  a[1] = fa(m0 + g + 8, k0 + 2 * t);
  a[2] = fa(m0 + g, k0 + 2 * t + 8);
  a[3] = fa(m0 + g + 8, k0 + 2 * t + 8);
}

template <class FB>
AHB_DEVICE void load_b(uint32_t b[2], const FB& fb, int k0, int n0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  b[0] = fb(k0 + 2 * t, n0 + g);
  b[1] = fb(k0 + 2 * t + 8, n0 + g);
}

// acc[j] (+)= A[m0:m0+16, k_lo:k_hi] * B[k_lo:k_hi, n0+8j : n0+8j+8]
template <int NT, class FA, class FB>
AHB_DEVICE void warp_mma(float (*acc)[4], const FA& fa, const FB& fb, int m0, int n0, int k_lo, int k_hi) {
  for (int k0 = k_lo; k0 < k_hi; k0 += 16) {
    uint32_t a[4];
    load_a(a, fa, m0, k0);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      uint32_t b[2];
      load_b(b, fb, k0, n0 + 8 * j);
      mma16816(acc[j], a, b);
    }
  }
}

// fp32 pair -> bf16 hi pair + bf16 lo pair (hi + lo = v to ~2^-16 relative)
AHB_DEVICE void split2(float2 v, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  const float2 hf = __bfloat1622float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack2(v.x - hf.x, v.y - hf.y);
}

// warp_mma with fp32 operands split into two bf16 terms: A B ~ Ah Bh + Ah Bl + Al Bh.
// Loaders return float2: fa(r, c) = (A[r][c], A[r][c+1]), fb(k, n) = (B[k][n], B[k+1][n]).
template <int NT, class FA, class FB>
AHB_DEVICE void warp_mma_split(float (*acc)[4], const FA& fa, const FB& fb, int m0, int n0, int k_lo, int k_hi) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  for (int k0 = k_lo; k0 < k_hi; k0 += 16) {
    uint32_t ah[4], al[4];
    split2(fa(m0 + g, k0 + 2 * t), ah[0], al[0]);
    split2(fa(m0 + g + 8, k0 + 2 * t), ah[1], al[1]);
    split2(fa(m0 + g, k0 + 2 * t + 8), ah[2], al[2]);
    split2(fa(m0 + g + 8, k0 + 2 * t + 8), ah[3], al[3]);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      uint32_t bh[2], bl[2];
      split2(fb(k0 + 2 * t, n0 + 8 * j + g), bh[0], bl[0]);
      split2(fb(k0 + 2 * t + 8, n0 + 8 * j + g), bh[1], bl[1]);
      mma16816(acc[j], ah, bh);
      mma16816(acc[j], ah, bl);
      mma16816(acc[j], al, bh);
    }
  }
}

template <int NT>
AHB_DEVICE void zero_acc(float (*acc)[4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
}

// Visit every accumulator element: f(row, col, value&)
template <int NT, class F>
AHB_DEVICE void for_acc(float (*acc)[4], int m0, int n0, const F& f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int c = n0 + 8 * j + 2 * t;
    f(m0 + g, c, acc[j][0]);
    f(m0 + g, c + 1, acc[j][1]);
    f(m0 + g + 8, c, acc[j][2]);
    f(m0 + g + 8, c + 1, acc[j][3]);
  }
}

// ---- common pair loaders over shared memory -------------------------------
// row-major bf16 matrix S[r][c] (ld in elements, even): A(r,c) = S[r][c]
struct RowA16 {
  const __nv_bfloat16* p; int ld;
  AHB_DEVICE uint32_t operator()(int r, int c) const { return *reinterpret_cast<const uint32_t*>(p + r * ld + c); }
};
// A(r,c) = S[c][r] for a row-major bf16 S (transposed access)
struct ColA16 {
  const __nv_bfloat16* p; int ld;
  AHB_DEVICE uint32_t operator()(int r, int c) const { return pack2(p[c * ld + r], p[(c + 1) * ld + r]); }
};
// A(r,c) = S[r][c] for fp32 S
struct RowA32 {
  const float* p; int ld;
  AHB_DEVICE uint32_t operator()(int r, int c) const { return pack2(p[r * ld + c], p[r * ld + c + 1]); }
};
// A(r,c) = S[c][r] for fp32 S
struct ColA32 {
  const float* p; int ld;
  AHB_DEVICE uint32_t operator()(int r, int c) const { return pack2(p[c * ld + r], p[(c + 1) * ld + r]); }
};
// B(k,n) = S[n][k] for bf16 S (k contiguous)
struct NKB16 {
  const __nv_bfloat16* p; int ld;
  AHB_DEVICE uint32_t operator()(int k, int n) const { return *reinterpret_cast<const uint32_t*>(p + n * ld + k); }
};
// B(k,n) = S[k][n] for bf16 S (n contiguous)
struct KNB16 {
  const __nv_bfloat16* p; int ld;
  AHB_DEVICE uint32_t operator()(int k, int n) const { return pack2(p[k * ld + n], p[(k + 1) * ld + n]); }
};
// B(k,n) = S[k][n] for fp32 S
struct KNB32 {
  const float* p; int ld;
  AHB_DEVICE uint32_t operator()(int k, int n) const { return pack2(p[k * ld + n], p[(k + 1) * ld + n]); }
};
// B(k,n) = S[n][k] for fp32 S
struct NKB32 {
  const float* p; int ld;
  AHB_DEVICE uint32_t operator()(int k, int n) const { return pack2(p[n * ld + k], p[n * ld + k + 1]); }
};

}  // namespace ahb
