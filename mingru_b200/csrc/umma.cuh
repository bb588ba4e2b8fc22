// umma.cuh -- tcgen05 (5th-generation tensor core) building blocks for the
// 64 x 64 chunk products of the delta rule: blocked shared-memory tiles,
// matrix descriptors, MMA issue and commit, TMEM allocation and loads.
//
// Tile layout ("blocked"): a 64 x 64 bf16 tile is 8 x 8 core matrices of
// 8 rows x 16 bytes; core matrix (r/8, c/8) sits at byte (r/8)*1024 + (c/8)*128
// and row r%8 of it at +16*(r%8). The same bytes serve as a K-major operand
// (contraction over the tile's columns: LBO = 128, SBO = 1024) and as an
// MN-major operand (contraction over its rows: LBO = 1024, SBO = 128), so a
// matrix and its transpose are both read from one copy. Products are
// D[m][n] (+)= sum_k A(m, k) B(n, k) with M = N = 64, K = 64 in four 16-deep
// MMAs, fp32 accumulators in TMEM: row m of D lives in TMEM lane
// 32*(m/16) + m%16, column n in column n of the accumulator.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace mgs {
namespace umma {

constexpr int kTileBytes = 64 * 64 * 2;  // 8192

// Element offset of (r, c) in a blocked 64-column tile.
__device__ __forceinline__ int boff(int r, int c) {
  return (r >> 3) * 512 + (c >> 3) * 64 + (r & 7) * 8 + (c & 7);
}

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory matrix descriptor (no swizzle, sm_100 descriptor version 1).
__device__ __forceinline__ uint64_t desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
// 16-deep k-step kk of a tile used K-major / MN-major.
__device__ __forceinline__ uint64_t desc_k(uint32_t tile, int kk) {
  return desc(tile + kk * 256, 128, 1024);
}
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, int kk) {
  return desc(tile + kk * 2048, 1024, 128);
}

// Instruction descriptor: bf16 x bf16 -> fp32, N columns (a multiple of 16,
// default 64), M = 64 (or 128: two blocked tiles stacked in consecutive
// memory, row m of D in TMEM lane m), operand majors.
__host__ __device__ constexpr uint32_t idesc64(bool a_mn, bool b_mn, bool m128 = false,
                                               uint32_t n = 64) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((n >> 3) << 17) | ((m128 ? 128u >> 4 : 64u >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)acc), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// A split operand tile pair in shared memory, as matrix descriptors of its
// first k-step: hi, lo (lo == 0: exact in bf16), the per-k-step descriptor
// increment (256 B K-major, 2048 B MN-major, in 16-byte units) and whether the
// product contracts over the tile's rows (MN-major) or columns (K-major).
struct Opnd {
  uint64_t hi, lo;
  uint32_t step;
  bool mn;
  uint64_t lo2 = 0;  // third level (0: none): x = hi + lo + lo2 for fp32-grade operands
};

// MN-major operand from a blocked tile of `cols` columns (a multiple of 8;
// rows are the contraction dimension, 64 of them): row-block stride cols*16 B.
__device__ __forceinline__ Opnd opnd_mn(uint32_t hi_addr, uint32_t lo_addr, int cols) {
  Opnd o;
  o.mn = true;
  const uint32_t rb = (uint32_t)cols * 16;
  o.step = 2 * rb / 16;
  o.hi = desc(hi_addr, rb, 128);
  o.lo = lo_addr == 0 ? 0 : desc(lo_addr, rb, 128);
  return o;
}

// Element offset of (r, c) in a blocked tile of `cols` columns.
__device__ __forceinline__ int boff_n(int r, int c, int cols) {
  return (r >> 3) * (cols * 8) + (c >> 3) * 64 + (r & 7) * 8 + (c & 7);
}

// Operand from tile addresses (lo_addr == 0: no lo term).
__device__ __forceinline__ Opnd opnd(uint32_t hi_addr, uint32_t lo_addr, bool mn) {
  Opnd o;
  o.mn = mn;
  o.step = mn ? 2048 / 16 : 256 / 16;
  o.hi = mn ? desc(hi_addr, 1024, 128) : desc(hi_addr, 128, 1024);
  o.lo = lo_addr == 0 ? 0 : (mn ? desc(lo_addr, 1024, 128) : desc(lo_addr, 128, 1024));
  return o;
}
// Three-level operand (64-column blocked tiles; a zero address drops a level).
__device__ __forceinline__ Opnd opnd3(uint32_t hi_addr, uint32_t lo_addr, uint32_t lo2_addr, bool mn) {
  Opnd o = opnd(hi_addr, lo_addr, mn);
  o.lo2 = lo2_addr == 0 ? 0 : (mn ? desc(lo2_addr, 1024, 128) : desc(lo2_addr, 128, 1024));
  return o;
}
// Three-level MN-major operand of a blocked tile of `cols` columns.
__device__ __forceinline__ Opnd opnd_mn3(uint32_t hi_addr, uint32_t lo_addr, uint32_t lo2_addr,
                                         int cols) {
  Opnd o = opnd_mn(hi_addr, lo_addr, cols);
  o.lo2 = lo2_addr == 0 ? 0 : desc(lo2_addr, (uint32_t)cols * 16, 128);
  return o;
}

// One product of a batch: D (+)= A B^T over K = 64 with the hi*hi, hi*lo and
// lo*hi terms; where either operand has a third level, also hi*lo2, lo2*hi
// and lo*lo (every term down to 2^-16 of the leading one: the dropped terms
// are below 2^-24 relative, fp32 rounding).
struct Prod {
  uint32_t d;
  Opnd A, B;
  bool accumulate;
  bool m128 = false;
  uint32_t n = 64;  // columns of D (B's MN extent)
};

// Issue a batch of independent products (one thread) k-step by k-step,
// round-robin over the products, so that consecutive MMAs go to different
// accumulators. Descriptors only advance by a constant per k-step, which keeps
// the issuing thread's instruction count per MMA small (issue, not the tensor
// pipe, bounds 64 x 64 x 16 MMAs).
template <int N>
__device__ __forceinline__ void products(const Prod (&ps)[N]) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const Prod& p = ps[i];
      const uint32_t id = idesc64(p.A.mn, p.B.mn, p.m128, p.n);
      const uint64_t oa = (uint64_t)(kk * p.A.step), ob = (uint64_t)(kk * p.B.step);
      mma(p.d, p.A.hi + oa, p.B.hi + ob, id, kk > 0 || p.accumulate);
      if (p.B.lo) mma(p.d, p.A.hi + oa, p.B.lo + ob, id, true);
      if (p.A.lo) mma(p.d, p.A.lo + oa, p.B.hi + ob, id, true);
      if (p.B.lo2) mma(p.d, p.A.hi + oa, p.B.lo2 + ob, id, true);
      if (p.A.lo2) mma(p.d, p.A.lo2 + oa, p.B.hi + ob, id, true);
      if ((p.A.lo2 || p.B.lo2) && p.A.lo && p.B.lo) mma(p.d, p.A.lo + oa, p.B.lo + ob, id, true);
    }
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          saddr(bar))
      : "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Warp-collective TMEM allocation of `ncols` columns (a power of two >= 32);
// the base address is written to shared memory at `dst`.
__device__ __forceinline__ void alloc(uint32_t* dst, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc(uint32_t base, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols)
               : "memory");
}

// Warp-collective load of 16 consecutive accumulator columns of this warp's
// 32-lane quarter (lane i of the warp gets TMEM lane 32*(warp%4) + i).
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// As ld16 without the wait: the registers are valid only after ld_wait()
// has been passed the same arrays (several loads share one wait).
__device__ __forceinline__ void ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// Wait for this thread's outstanding TMEM loads; the empty asm statements that
// follow tie the loaded registers to the wait so no use moves above it.
__device__ __forceinline__ void ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void ld_bind(uint32_t (&r)[16], float (&v)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Split 16 consecutive values of row r (columns c0..c0+15, c0 % 8 == 0) into
// bf16 hi / lo and store them into blocked tiles.
__device__ __forceinline__ void store_split16(__nv_bfloat16* hi, __nv_bfloat16* lo, int r, int c0,
                                              const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t ph[4], pl[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = v[8 * h + 2 * i], x1 = v[8 * h + 2 * i + 1];
      __nv_bfloat162 b = __floats2bfloat162_rn(x0, x1);
      const float2 f = __bfloat1622float2(b);
      __nv_bfloat162 l = __floats2bfloat162_rn(x0 - f.x, x1 - f.y);
      ph[i] = *reinterpret_cast<uint32_t*>(&b);
      pl[i] = *reinterpret_cast<uint32_t*>(&l);
    }
    const int o = boff(r, c0 + 8 * h);
    *reinterpret_cast<uint4*>(hi + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
    if (lo) *reinterpret_cast<uint4*>(lo + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
  }
}

// store_split16 for a blocked tile of `cols` columns (chunks of 8 columns
// at c0 and c0 + 8; a chunk is written only if it starts below `valid`).
__device__ __forceinline__ void store_split16_n(__nv_bfloat16* hi, __nv_bfloat16* lo, int r, int c0,
                                                int cols, int valid, const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (c0 + 8 * h >= valid) continue;
    uint32_t ph[4], pl[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = v[8 * h + 2 * i], x1 = v[8 * h + 2 * i + 1];
      __nv_bfloat162 b = __floats2bfloat162_rn(x0, x1);
      const float2 f = __bfloat1622float2(b);
      __nv_bfloat162 l = __floats2bfloat162_rn(x0 - f.x, x1 - f.y);
      ph[i] = *reinterpret_cast<uint32_t*>(&b);
      pl[i] = *reinterpret_cast<uint32_t*>(&l);
    }
    const int o = boff_n(r, c0 + 8 * h, cols);
    *reinterpret_cast<uint4*>(hi + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
    *reinterpret_cast<uint4*>(lo + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
  }
}

// x -> bf16 levels h, m, l with x = h + m + l to within 2^-24 relative
// (each level is the bf16 rounding of what the previous ones leave; the
// differences are exact in fp32), for two values packed per 32-bit word.
__device__ __forceinline__ void split3_pack(float x0, float x1, uint32_t& h, uint32_t& m, uint32_t& l) {
  __nv_bfloat162 bh = __floats2bfloat162_rn(x0, x1);
  const float2 fh = __bfloat1622float2(bh);
  const float r0 = x0 - fh.x, r1 = x1 - fh.y;
  __nv_bfloat162 bm = __floats2bfloat162_rn(r0, r1);
  const float2 fm = __bfloat1622float2(bm);
  __nv_bfloat162 bl = __floats2bfloat162_rn(r0 - fm.x, r1 - fm.y);
  h = *reinterpret_cast<uint32_t*>(&bh);
  m = *reinterpret_cast<uint32_t*>(&bm);
  l = *reinterpret_cast<uint32_t*>(&bl);
}

// 8 consecutive values -> three levels at element offset o of tiles h, m, l.
__device__ __forceinline__ void store_split8_3(__nv_bfloat16* h, __nv_bfloat16* m, __nv_bfloat16* l,
                                               int o, const float* v) {
  uint32_t ph[4], pm[4], pl[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) split3_pack(v[2 * i], v[2 * i + 1], ph[i], pm[i], pl[i]);
  *reinterpret_cast<uint4*>(h + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
  *reinterpret_cast<uint4*>(m + o) = make_uint4(pm[0], pm[1], pm[2], pm[3]);
  *reinterpret_cast<uint4*>(l + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
}

}  // namespace umma
}  // namespace mgs
