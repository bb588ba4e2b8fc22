// common.cuh -- shared device machinery for the chunked look-back scans.
//
// Every scan in this library is a first-order affine recurrence over a time
// axis, x_t = M_t x_{t-1} + u_t, whose per-segment aggregates form a monoid
// under composition. The kernels tile (time x channels): a CTA takes one tile
// from an atomic tile counter (so every tile it waits on was handed out
// earlier and is already running), reduces its segment locally in registers,
// publishes the aggregate, and walks back over the preceding tiles of the same
// channel strip until it meets an inclusive prefix ("decoupled look-back",
// Merrill & Garland 2016). Waits are bounded: a wait that runs out records
// MGS_LOOKBACK_TIMEOUT in the per-call workspace header and in a sticky device
// word, then proceeds, so no launch can hang a GPU.
#pragma once

#include <type_traits>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mingru_scan.h"

namespace mgs {

// ---------------------------------------------------------------- dtypes --

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

template <int BYTES>
struct VecOf;
template <>
struct VecOf<16> { using type = uint4; };
template <>
struct VecOf<8> { using type = uint2; };
template <>
struct VecOf<4> { using type = unsigned; };
template <>
struct VecOf<2> { using type = unsigned short; };

// Load N consecutive elements (one vector access of N*sizeof(T) <= 16 bytes;
// the caller guarantees alignment) and widen to fp32. Streaming hint: every
// input element is read exactly once per kernel.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  static_assert(N * sizeof(T) <= 16, "vector too wide");
  using V = typename VecOf<N * sizeof(T)>::type;
  V v = __ldcs(reinterpret_cast<const V*>(p));
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = to_f32<T>(e[i]);
}

template <typename T, int N>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&in)[N]) {
  static_assert(N * sizeof(T) <= 16, "vector too wide");
  using V = typename VecOf<N * sizeof(T)>::type;
  V v;
  T* e = reinterpret_cast<T*>(&v);
#pragma unroll
  for (int i = 0; i < N; ++i) e[i] = from_f32<T>(in[i]);
  __stcs(reinterpret_cast<V*>(p), v);
}

// ------------------------------------------------------- memory ordering --

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------- workspace --
//
// Per-call look-back workspace (caller allocated, header + flags zeroed by
// the launcher with one cudaMemsetAsync):
//   [0]          u32 tile counter
//   [1]          u32 per-call error bits
//   [256 ..)     u32 flags[ntiles]              0 = empty, 1 = aggregate, 2 = inclusive
//   [..)         f32 agg[ntiles][NF][32]
//   [..)         f32 incl[ntiles][NF][32]
// NF = floats each lane of the look-back warp carries.

constexpr unsigned kFlagEmpty = 0u;
constexpr unsigned kFlagAgg = 1u;
constexpr unsigned kFlagIncl = 2u;
constexpr unsigned kErrTimeout = 1u << MGS_LOOKBACK_TIMEOUT;

// Upper bound on polls of one flag (~ a second with the backoff below).
constexpr long long kSpinLimit = 1ll << 24;

struct Lookback {
  unsigned* counter;
  unsigned* err;
  unsigned* flags;
  float* agg;
  float* incl;
  long long spin;  // poll bound of each wait (kSpinLimit; tests pass a small one)
};

// Sticky error word of this translation unit (each .cu file that includes
// this header owns one); read and cleared by the file's take_sticky_error().
static __device__ unsigned g_sticky_err = 0u;

static inline unsigned take_sticky_error(cudaStream_t stream) {
  unsigned v = 0u, zero = 0u;
  if (cudaMemcpyFromSymbolAsync(&v, g_sticky_err, sizeof(v), 0, cudaMemcpyDeviceToHost, stream) !=
      cudaSuccess)
    return 1u << MGS_LAUNCH_FAILED;
  if (cudaMemcpyToSymbolAsync(g_sticky_err, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice,
                              stream) != cudaSuccess)
    return 1u << MGS_LAUNCH_FAILED;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return 1u << MGS_LAUNCH_FAILED;
  return v;
}

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline size_t lookback_bytes(long long ntiles, int nf) {
  size_t flags = align_up((size_t)ntiles * 4, 256);
  size_t elem = (size_t)ntiles * nf * 32 * 4;
  return 256 + flags + 2 * elem;
}

inline size_t lookback_zero_bytes(long long ntiles) {
  return 256 + align_up((size_t)ntiles * 4, 256);
}

inline Lookback lookback_view(void* ws, long long ntiles, int nf) {
  char* base = static_cast<char*>(ws);
  Lookback lb;
  lb.counter = reinterpret_cast<unsigned*>(base);
  lb.err = reinterpret_cast<unsigned*>(base) + 1;
  lb.flags = reinterpret_cast<unsigned*>(base + 256);
  size_t flags = align_up((size_t)ntiles * 4, 256);
  lb.agg = reinterpret_cast<float*>(base + 256 + flags);
  lb.incl = lb.agg + (size_t)ntiles * nf * 32;
  lb.spin = kSpinLimit;
  return lb;
}

// Publish this lane's NF floats of `val` for `tile` and raise its flag.
template <int NF>
__device__ __forceinline__ void lb_publish(const Lookback& lb, long long tile, unsigned flag,
                                           const float (&val)[NF]) {
  const int lane = threadIdx.x & 31;
  float* dst = (flag == kFlagIncl ? lb.incl : lb.agg) + (size_t)tile * NF * 32;
#pragma unroll
  for (int f = 0; f < NF; ++f) __stcg(dst + f * 32 + lane, val[f]);
  __threadfence();
  __syncwarp();
  if (lane == 0) st_release_u32(lb.flags + tile, flag);
}

// Wait (bounded) until `tile` has published; returns the flag the whole warp
// agrees on (the minimum any lane acquired: an aggregate stays valid once the
// inclusive value also exists).
__device__ __forceinline__ unsigned lb_wait(const Lookback& lb, long long tile) {
  unsigned f = ld_acquire_u32(lb.flags + tile);
  long long it = 0;
  while (f == kFlagEmpty) {
    if (++it > lb.spin) {
      atomicOr(lb.err, kErrTimeout);
      atomicOr(&g_sticky_err, kErrTimeout);
      f = kFlagIncl;  // proceed with whatever is there; the host raises
      break;
    }
    if ((it & 255) == 0 && ld_relaxed_u32(lb.err) != 0u) {
      f = kFlagIncl;
      break;
    }
    __nanosleep(32);
    f = ld_acquire_u32(lb.flags + tile);
  }
  return __reduce_min_sync(0xffffffffu, f);
}

// Decoupled look-back run by one full warp. `Monoid` supplies
//   static void identity(float (&x)[NF]);
//   static void combine(const float (&earlier)[NF], const float (&later)[NF], float (&out)[NF]);
// where `out` may alias `earlier` (never `later`).
// `tile` is the tile's position in processing order, `stride` the distance to
// its predecessor in the same strip, `pos` its index along the strip (0 = the
// first segment: no predecessor). On return `excl` holds the composition of
// every earlier segment of the strip and the tile's inclusive value has been
// published.
template <class Monoid, int NF>
__device__ __forceinline__ void warp_lookback(const Lookback& lb, long long tile, long long stride,
                                              long long pos, const float (&agg)[NF],
                                              float (&excl)[NF]) {
  const int lane = threadIdx.x & 31;
  if (pos == 0) {
    Monoid::identity(excl);
    lb_publish<NF>(lb, tile, kFlagIncl, agg);
    return;
  }
  lb_publish<NF>(lb, tile, kFlagAgg, agg);
  float run[NF];
  Monoid::identity(run);
  long long p = tile - stride;
  while (true) {
    const unsigned f = lb_wait(lb, p);
    const float* src = (f == kFlagIncl ? lb.incl : lb.agg) + (size_t)p * NF * 32;
    float e[NF], tmp[NF];
#pragma unroll
    for (int i = 0; i < NF; ++i) e[i] = __ldcg(src + i * 32 + lane);
    Monoid::combine(e, run, tmp);
#pragma unroll
    for (int i = 0; i < NF; ++i) run[i] = tmp[i];
    if (f == kFlagIncl || p < stride) break;
    p -= stride;
  }
#pragma unroll
  for (int i = 0; i < NF; ++i) excl[i] = run[i];
  float inc[NF];
  Monoid::combine(excl, agg, inc);
  lb_publish<NF>(lb, tile, kFlagIncl, inc);
}

// Windowed decoupled look-back: lanes inspect up to 32 predecessors at once
// (lane i looks at predecessor i+1 of the strip), so the walk back to the
// nearest inclusive prefix costs one L2 round trip per 32 predecessors
// instead of one per predecessor. Same contract as warp_lookback.
// `seed` (optional, NF floats of this lane) is the element before the first
// segment of the strip (a carried-in state); the first segment's exclusive
// prefix is then the seed instead of the identity.
template <class Monoid, int NF>
__device__ __forceinline__ void warp_lookback_win(const Lookback& lb, long long tile,
                                                  long long stride, long long pos,
                                                  const float (&agg)[NF], float (&excl)[NF],
                                                  const float* seed = nullptr) {
  const int lane = threadIdx.x & 31;
  if (pos == 0) {
    if (seed == nullptr) {
      Monoid::identity(excl);
      lb_publish<NF>(lb, tile, kFlagIncl, agg);
    } else {
      float inc[NF];
#pragma unroll
      for (int i = 0; i < NF; ++i) excl[i] = seed[i];
      Monoid::combine(excl, agg, inc);
      lb_publish<NF>(lb, tile, kFlagIncl, inc);
    }
    return;
  }
  lb_publish<NF>(lb, tile, kFlagAgg, agg);
  float run[NF];
  Monoid::identity(run);
  long long remaining = pos;        // predecessors left: tile - k*stride, k = 1..remaining
  long long base = tile - stride;   // predecessor k = 1
  while (remaining > 0) {
    const int nwin = remaining < 32 ? (int)remaining : 32;
    const bool valid = lane < nwin;
    const unsigned* fp = lb.flags + (valid ? base - (long long)lane * stride : 0);
    unsigned f = valid ? ld_acquire_u32(fp) : kFlagIncl;
    int last;
    long long it = 0;
    while (true) {
      const unsigned im = __ballot_sync(0xffffffffu, valid && f == kFlagIncl);
      last = im ? (__ffs(im) - 1) : nwin - 1;
      const bool need = lane <= last;
      const unsigned em = __ballot_sync(0xffffffffu, need && f == kFlagEmpty);
      if (em == 0u) break;
      if (++it > lb.spin) {
        if (lane == 0) {
          atomicOr(lb.err, kErrTimeout);
          atomicOr(&g_sticky_err, kErrTimeout);
        }
        if (f == kFlagEmpty) f = kFlagIncl;  // proceed; the host raises
        continue;
      }
      if ((it & 255) == 0 && ld_relaxed_u32(lb.err) != 0u && f == kFlagEmpty) f = kFlagIncl;
      if (need && f == kFlagEmpty) {
        __nanosleep(32);
        f = ld_acquire_u32(fp);
      }
    }
    __syncwarp();
    // Compose predecessors nearest-first: run = e_i o run. Loads of G
    // predecessors are issued together so a small element costs one L2 round
    // trip per G predecessors instead of one per predecessor.
    constexpr int G = NF <= 4 ? 8 : (NF <= 8 ? 4 : (NF <= 16 ? 2 : 1));
#pragma unroll 1
    for (int i0 = 0; i0 <= last; i0 += G) {
      float e[G][NF];
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        const int i = i0 + gi < last ? i0 + gi : last;  // clamp: duplicates are never combined
        const unsigned fi = __shfl_sync(0xffffffffu, f, i);
        const float* src = (fi == kFlagIncl ? lb.incl : lb.agg) +
                           (size_t)(base - (long long)i * stride) * NF * 32;
#pragma unroll
        for (int q = 0; q < NF; ++q) e[gi][q] = __ldcg(src + q * 32 + lane);
      }
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        if (i0 + gi <= last) {
          Monoid::combine(e[gi], run, e[gi]);  // combine may write over its earlier operand
#pragma unroll
          for (int q = 0; q < NF; ++q) run[q] = e[gi][q];
        }
      }
    }
    const unsigned flast = __shfl_sync(0xffffffffu, f, last);
    if (flast == kFlagIncl) break;
    remaining -= nwin;
    base -= (long long)nwin * stride;
  }
#pragma unroll
  for (int i = 0; i < NF; ++i) excl[i] = run[i];
  float inc[NF];
  Monoid::combine(excl, agg, inc);
  lb_publish<NF>(lb, tile, kFlagIncl, inc);
}

// Same look-back for large elements: the tile aggregate is read from shared
// memory (agg_s[NF][32]) and the exclusive prefix is written back to shared
// memory (excl_s[NF][32]), so only two NF-float elements are live in
// registers at any time (the k x (k+1) maps of the block scans are 72 floats
// at k = 8).
template <class Monoid, int NF>
__device__ __forceinline__ void warp_lookback_win_smem(const Lookback& lb, long long tile,
                                                       long long stride, long long pos,
                                                       const float (*agg_s)[32],
                                                       float (*excl_s)[32]) {
  const int lane = threadIdx.x & 31;
  float run[NF];
#pragma unroll
  for (int q = 0; q < NF; ++q) run[q] = agg_s[q][lane];
  if (pos == 0) {
    lb_publish<NF>(lb, tile, kFlagIncl, run);
    Monoid::identity(run);
#pragma unroll
    for (int q = 0; q < NF; ++q) excl_s[q][lane] = run[q];
    return;
  }
  lb_publish<NF>(lb, tile, kFlagAgg, run);
  Monoid::identity(run);
  long long remaining = pos;
  long long base = tile - stride;
  while (remaining > 0) {
    const int nwin = remaining < 32 ? (int)remaining : 32;
    const bool valid = lane < nwin;
    const unsigned* fp = lb.flags + (valid ? base - (long long)lane * stride : 0);
    unsigned f = valid ? ld_acquire_u32(fp) : kFlagIncl;
    int last;
    long long it = 0;
    while (true) {
      const unsigned im = __ballot_sync(0xffffffffu, valid && f == kFlagIncl);
      last = im ? (__ffs(im) - 1) : nwin - 1;
      const bool need = lane <= last;
      const unsigned em = __ballot_sync(0xffffffffu, need && f == kFlagEmpty);
      if (em == 0u) break;
      if (++it > lb.spin) {
        if (lane == 0) {
          atomicOr(lb.err, kErrTimeout);
          atomicOr(&g_sticky_err, kErrTimeout);
        }
        if (f == kFlagEmpty) f = kFlagIncl;
        continue;
      }
      if ((it & 255) == 0 && ld_relaxed_u32(lb.err) != 0u && f == kFlagEmpty) f = kFlagIncl;
      if (need && f == kFlagEmpty) {
        __nanosleep(32);
        f = ld_acquire_u32(fp);
      }
    }
    __syncwarp();
#pragma unroll 1
    for (int i = 0; i <= last; ++i) {
      const unsigned fi = __shfl_sync(0xffffffffu, f, i);
      const float* src = (fi == kFlagIncl ? lb.incl : lb.agg) +
                         (size_t)(base - (long long)i * stride) * NF * 32;
      float e[NF];
#pragma unroll
      for (int q = 0; q < NF; ++q) e[q] = __ldcg(src + q * 32 + lane);
      Monoid::combine(e, run, e);
#pragma unroll
      for (int q = 0; q < NF; ++q) run[q] = e[q];
    }
    const unsigned flast = __shfl_sync(0xffffffffu, f, last);
    if (flast == kFlagIncl) break;
    remaining -= nwin;
    base -= (long long)nwin * stride;
  }
#pragma unroll
  for (int q = 0; q < NF; ++q) excl_s[q][lane] = run[q];
  {
    float a[NF];
#pragma unroll
    for (int q = 0; q < NF; ++q) a[q] = agg_s[q][lane];
    Monoid::combine(run, a, run);
  }
  lb_publish<NF>(lb, tile, kFlagIncl, run);
}

// ------------------------------------------------- TMA bulk copy + mbarrier --
//
// Tiles are streamed into shared memory with the bulk-copy engine
// (cp.async.bulk global -> shared, completion counted on an mbarrier; no
// tensor map and no multicast). Every wait on an mbarrier is bounded.

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

// Bounded wait for an mbarrier phase; returns false (after recording a
// timeout) if the phase never completes within `limit` polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned* err,
                                          long long limit = kSpinLimit) {
  long long it = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++it > limit) {
      atomicOr(err, kErrTimeout);
      atomicOr(&g_sticky_err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// One bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from global to this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads, so
// a group of warps can leave a loop together (no warp is ever left waiting
// at a barrier that another warp has abandoned).
__device__ __forceinline__ bool bar_any(int id, int nthreads, bool pred) {
  unsigned r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((unsigned)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0u;
}

// ------------------------------------------------------ TMA tensor maps --
//
// Host: encode a 3-D tiled tensor map for a C-contiguous (Z, Y, X) tensor
// (X innermost) with a box of (bx, by, 1), no swizzle, zero fill outside the
// tensor. The driver function is fetched through the runtime's entry-point
// query, so the library does not link libcuda directly.

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

template <typename E>
inline CUtensorMapDataType tma_dtype();
template <>
inline CUtensorMapDataType tma_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <>
inline CUtensorMapDataType tma_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <>
inline CUtensorMapDataType tma_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }

// Returns false if the map cannot be encoded (the caller reports MGS_LAUNCH_FAILED).
template <typename E>
inline bool make_tmap_3d(CUtensorMap* map, const void* base, long long X, long long Y, long long Z,
                         unsigned bx, unsigned by) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)X, (cuuint64_t)Y, (cuuint64_t)Z};
  const cuuint64_t strides[2] = {(cuuint64_t)(X * (long long)sizeof(E)),
                                 (cuuint64_t)(X * Y * (long long)sizeof(E))};
  const cuuint32_t box[3] = {bx, by, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(map, tma_dtype<E>(), 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Device: one tiled box load (no multicast) completing on `bar`. The x
// coordinate times the element size is always a multiple of 16 bytes here.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Device: one tiled box store from this CTA's shared memory (rows or columns
// outside the tensor are not written). Shared-memory writes of the generic
// proxy must be fenced (fence_proxy_async_smem) and the CTA synchronised
// before the store is issued; the source stays live until bulk_wait_read().
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int x, int y, int z,
                                             const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(src))
      : "memory");
}

// One bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory to global memory, in the current bulk group
// (bulk_commit / bulk_wait_read; shared writes fenced with fence_proxy_async_smem).
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until all but the most recent committed bulk group have read shared memory.
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Error-word helpers shared by the per-file launchers.
// On failure, clear the runtime's last-error state so the failure is
// reported once, by this call, and does not leak into the next launch check.
#define MGS_CUDA_OK(expr)              \
  do {                                 \
    if ((expr) != cudaSuccess) {       \
      (void)cudaGetLastError();        \
      return MGS_LAUNCH_FAILED;        \
    }                                  \
  } while (0)

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline int dtype_size(int dtype) {
  switch (dtype) {
    case MGS_F32: return 4;
    case MGS_BF16: return 2;
    case MGS_F16: return 2;
    default: return 0;
  }
}

// mgs_dtype code of a storage type.
template <typename E>
constexpr int dtype_of() {
  if constexpr (std::is_same_v<E, float>) return MGS_F32;
  else if constexpr (std::is_same_v<E, __nv_bfloat16>) return MGS_BF16;
  else return MGS_F16;
}

}  // namespace mgs
