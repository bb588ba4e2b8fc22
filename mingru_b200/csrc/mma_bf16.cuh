// mma_bf16.cuh -- warp-level bf16 tensor-core products with split (hi + lo)
// operands, for the chunk matrices of the delta rule.
//
// Every chunk matrix lives in shared memory as bf16 with a padded leading
// dimension (kLd = 72 elements = 144 bytes: the 8 rows an ldmatrix phase reads
// fall in 8 distinct 16-byte bank groups). A matrix computed in fp32 is kept
// as two bf16 tiles, hi = bf16(x) and lo = bf16(x - hi), so x = hi + lo to
// ~16 significant bits; a product of two such operands is formed as
// hi*hi + hi*lo + lo*hi (the lo*lo term is below fp32 accumulation noise),
// and inputs that are exact in bf16 use one term. With fp32 accumulation this
// keeps each product within a few ulp of fp32 (the recurrence state stays fp32
// in registers between chunks).
//
// Operand orientation: A(m, k) is read from a tile stored either row-major
// [m][k] ("row") or as its transpose [k][m] ("col", ldmatrix .trans); B(k, n)
// from a tile stored [n][k] ("nk") or [k][n] ("kn", ldmatrix .trans). The
// fragment layouts are those of mma.m16n8k16 .row.col.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace mgs {
namespace tc {

constexpr int kLd = 72;  // bf16 elements per shared-memory row of a 64-wide tile

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void ldsm4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p))
               : "memory");
}

__device__ __forceinline__ void ldsm4t(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p))
               : "memory");
}

__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                    uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float x0, float x1) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  return *reinterpret_cast<uint32_t*>(&h);
}

// (x0, x1) -> hi pair and lo pair with x = hi + lo (each rounded to nearest).
__device__ __forceinline__ void split_pack(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  const float2 hf = __bfloat1622float2(h);
  __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
  hi = *reinterpret_cast<uint32_t*>(&h);
  lo = *reinterpret_cast<uint32_t*>(&l);
}

// A split operand: hi tile and (optional) lo tile, both [rows][kLd] bf16.
struct Op {
  const __nv_bfloat16* hi;
  const __nv_bfloat16* lo;  // nullptr: exact in bf16 (one term)
};

// Per-lane ldmatrix source of the A fragment rows m0..m0+15, cols k0..k0+15.
template <bool COL>
__device__ __forceinline__ const __nv_bfloat16* a_src(const __nv_bfloat16* t, int m0, int k0) {
  const int lane = threadIdx.x & 31, r = lane & 7, q = lane >> 3;
  if (!COL)  // stored [m][k]
    return t + (m0 + r + ((q & 1) << 3)) * kLd + k0 + ((q >> 1) << 3);
  // stored [k][m]
  return t + (k0 + r + ((q >> 1) << 3)) * kLd + m0 + ((q & 1) << 3);
}

// Per-lane ldmatrix source of the B fragments of two n-tiles (n0..n0+15), k0..k0+15.
template <bool KN>
__device__ __forceinline__ const __nv_bfloat16* b_src(const __nv_bfloat16* t, int k0, int n0) {
  const int lane = threadIdx.x & 31, r = lane & 7, q = lane >> 3;
  if (!KN)  // stored [n][k]
    return t + (n0 + r + ((q >> 1) << 3)) * kLd + k0 + ((q & 1) << 3);
  // stored [k][n]
  return t + (k0 + r + ((q & 1) << 3)) * kLd + n0 + ((q >> 1) << 3);
}

__device__ __forceinline__ void ldsm2(const void* p, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_addr(p))
               : "memory");
}

__device__ __forceinline__ void ldsm2t(const void* p, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_addr(p))
               : "memory");
}

// B fragment of one n-tile (n0..n0+7), k0..k0+15 (lanes 0-15 supply the addresses).
template <bool KN>
__device__ __forceinline__ void load_b1(const __nv_bfloat16* t, int k0, int n0, uint32_t (&r)[2]) {
  const int lane = threadIdx.x & 31, rr = lane & 7, q = (lane >> 3) & 1;
  if (KN)
    ldsm2t(t + (k0 + rr + (q << 3)) * kLd + n0, r);  // stored [k][n]
  else
    ldsm2(t + (n0 + rr) * kLd + k0 + (q << 3), r);   // stored [n][k]
}

template <bool COL>
__device__ __forceinline__ void load_a(const __nv_bfloat16* t, int m0, int k0, uint32_t (&r)[4]) {
  if (COL)
    ldsm4t(a_src<true>(t, m0, k0), r);
  else
    ldsm4(a_src<false>(t, m0, k0), r);
}

template <bool KN>
__device__ __forceinline__ void load_b(const __nv_bfloat16* t, int k0, int n0, uint32_t (&r)[4]) {
  if (KN)
    ldsm4t(b_src<true>(t, k0, n0), r);
  else
    ldsm4(b_src<false>(t, k0, n0), r);
}

// c[NT] (a 16 x 8*NT tile at rows m0, cols n0) += A(m0.., k) * B(k, n0..) for
// k in [k_begin, k_end) (multiples of 16). NT even.
// Only the first np_end n-tile pairs are computed (the rest of c is untouched).
// NT = 1 is a single 8-column tile.
template <int NT, bool ACOL, bool BKN>
__device__ __forceinline__ void gemm(float (&c)[NT][4], Op A, int m0, Op B, int n0, int k_begin,
                                     int k_end, int np_end = NT / 2) {
  if constexpr (NT == 1) {
    for (int k0 = k_begin; k0 < k_end; k0 += 16) {
      uint32_t ah[4], al[4], bh[2], bl[2];
      load_a<ACOL>(A.hi, m0, k0, ah);
      if (A.lo) load_a<ACOL>(A.lo, m0, k0, al);
      load_b1<BKN>(B.hi, k0, n0, bh);
      mma(c[0], ah, bh[0], bh[1]);
      if (B.lo) {
        load_b1<BKN>(B.lo, k0, n0, bl);
        mma(c[0], ah, bl[0], bl[1]);
      }
      if (A.lo) mma(c[0], al, bh[0], bh[1]);
    }
  } else {
  static_assert(NT % 2 == 0, "n-tiles come in pairs");
  for (int k0 = k_begin; k0 < k_end; k0 += 16) {
    uint32_t ah[4], al[4];
    load_a<ACOL>(A.hi, m0, k0, ah);
    if (A.lo) load_a<ACOL>(A.lo, m0, k0, al);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      if (j / 2 >= np_end) break;
      uint32_t bh[4], bl[4];
      load_b<BKN>(B.hi, k0, n0 + 8 * j, bh);
      mma(c[j], ah, bh[0], bh[1]);
      mma(c[j + 1], ah, bh[2], bh[3]);
      if (B.lo) {
        load_b<BKN>(B.lo, k0, n0 + 8 * j, bl);
        mma(c[j], ah, bl[0], bl[1]);
        mma(c[j + 1], ah, bl[2], bl[3]);
      }
      if (A.lo) {
        mma(c[j], al, bh[0], bh[1]);
        mma(c[j + 1], al, bh[2], bh[3]);
      }
    }
  }
  }
}

template <int NT>
__device__ __forceinline__ void zero(float (&c)[NT][4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
}

// Element coordinates of fragment value v (0..3) of n-tile j.
__device__ __forceinline__ int frag_row(int m0, int v) {
  return m0 + ((threadIdx.x & 31) >> 2) + ((v >> 1) << 3);
}
__device__ __forceinline__ int frag_col(int n0, int j, int v) {
  return n0 + 8 * j + ((threadIdx.x & 3) << 1) + (v & 1);
}

// Store a 16 x 8*NT fp32 tile as split bf16 (hi, lo) tiles at rows m0, cols n0,
// applying f(row, col, x) first (f returns the value to store).
template <int NT, class F>
__device__ __forceinline__ void store_split(const float (&c)[NT][4], __nv_bfloat16* hi,
                                            __nv_bfloat16* lo, int m0, int n0, F f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = m0 + g + 8 * h, col = n0 + 8 * j + 2 * t;
      const float x0 = f(row, col, c[j][2 * h]), x1 = f(row, col + 1, c[j][2 * h + 1]);
      uint32_t ph, pl;
      split_pack(x0, x1, ph, pl);
      *reinterpret_cast<uint32_t*>(hi + row * kLd + col) = ph;
      if (lo) *reinterpret_cast<uint32_t*>(lo + row * kLd + col) = pl;
    }
}

// Write a 64 x 64 fp32 matrix held row-major in shared memory (leading
// dimension ld) as split bf16 tiles, all threads of the block, rows x cols.
__device__ __forceinline__ void f32_to_split(const float* src, int ld, __nv_bfloat16* hi,
                                             __nv_bfloat16* lo, int nthreads) {
  for (int i = threadIdx.x; i < 64 * 32; i += nthreads) {
    const int row = i >> 5, col = (i & 31) << 1;
    uint32_t ph, pl;
    split_pack(src[row * ld + col], src[row * ld + col + 1], ph, pl);
    *reinterpret_cast<uint32_t*>(hi + row * kLd + col) = ph;
    *reinterpret_cast<uint32_t*>(lo + row * kLd + col) = pl;
  }
}

}  // namespace tc
}  // namespace mgs
