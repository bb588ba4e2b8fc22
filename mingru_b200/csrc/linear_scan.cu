// linear_scan.cu -- diagonal affine scan h_t = a_t h_{t-1} + b_t (forward and
// backward) for (B, T, D) tensors, fp32 / bf16 / fp16 storage, fp32 math.
//
// Reference behaviour: min_gru.py:1454-1510 `linear_scan` returns
// (A_t = prod_{s<=t} a_s, Bc_t = a_t Bc_{t-1} + b_t) with A_0 = 1, Bc_0 = 0;
// its Triton kernels (triton_scans.py:702-751, 961-1036) walk T sequentially
// per channel. The backward adjoint (triton_scans.py:1013-1024):
//   G^A_t = gA_t + a_{t+1} G^A_{t+1},  G^B_t = gB_t + a_{t+1} G^B_{t+1},
//   da_t  = G^A_t A_{t-1} + G^B_t Bc_{t-1},  db_t = G^B_t.
//
// Three algorithms, chosen per shape (the same choice for forward and
// backward, since the forward's carries feed the backward):
//  * strip (wide problems, B*ceil(D/32) >= 2 x #SMs, rows 16-byte aligned):
//    32-channel strips walk all of T, one warp per strip running the
//    recurrence itself (one FMA per channel and step), their 32-step chunks
//    streamed by TMA into per-warp shared-memory rings (mbarrier completion)
//    and each chunk's results written back by TMA box stores; no global
//    synchronisation.
//  * direct-vec (narrow problems, rows 16-byte aligned): one tile (64 steps x
//    128 channels, 4 channels per lane, 16-byte accesses) per CTA, chunk
//    carries across CTAs by windowed decoupled look-back.
//  * direct-scalar (any D): the same with one channel per lane.
// The forward writes the state at every carry-chunk start ("carries", fp32,
// ~6% of one input); the backward's tiles are exactly those chunks, so it
// recomputes A_{t-1}, Bc_{t-1} in registers from them instead of reading the
// saved outputs: it reads a, b, gA, gBc and writes da, db -- the algorithmic
// minimum -- and carries the adjoint G in reverse time order.
#include "common.cuh"

#include <mutex>

namespace mgs {
namespace linear {

constexpr int kLc = 32;  // carry-chunk length = backward tile length (all algorithms)

// direct paths
constexpr int kVecCpt = 4;                       // channels per lane, direct-vec
constexpr int kVecFwdS = 8, kVecFwdNW = 8;       // forward tile 64 steps
constexpr int kSclFwdS = 8, kSclFwdNW = 4;       // forward tile 32 steps
constexpr int kBwdS = 4, kBwdNW = 8;             // backward tile 32 steps
static_assert(kBwdS * kBwdNW == kLc, "backward tile must be one carry chunk");
static_assert((kVecFwdS * kVecFwdNW) % kLc == 0 && kLc % kVecFwdS == 0, "vec carry grid");
static_assert((kSclFwdS * kSclFwdNW) % kLc == 0 && kLc % kSclFwdS == 0, "scalar carry grid");

// strip path

enum Algo { kStrip = 0, kDirectVec = 1, kDirectScalar = 2 };

inline int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

struct Geometry {
  Algo algo;
  int cpt;             // channels per lane
  long long sper;      // strips per batch row
  long long nstrips;   // B * sper
  long long nchunks;   // ceil(T / kLc): carry chunks = backward tiles per strip
  long long ntiles;    // nstrips * nchunks
  long long fchunks;   // forward tiles per strip (direct paths)
  long long ftiles;
};

inline Geometry geometry(long long B, long long T, long long D, int dtype) {
  Geometry g;
  const bool rows16 = ((D * dtype_size(dtype)) % 16) == 0;
  const long long strips32 = B * ((D + 31) / 32);
  if (rows16 && strips32 >= 2LL * sm_count())
    g.algo = kStrip;
  else
    g.algo = rows16 ? kDirectVec : kDirectScalar;
  g.cpt = g.algo == kDirectVec ? kVecCpt : 1;
  const long long w = 32LL * g.cpt;
  g.sper = (D + w - 1) / w;
  g.nstrips = B * g.sper;
  g.nchunks = (T + kLc - 1) / kLc;
  g.ntiles = g.nstrips * g.nchunks;
  const int fl = g.algo == kDirectVec ? kVecFwdS * kVecFwdNW : (g.algo == kDirectScalar ? kSclFwdS * kSclFwdNW : kLc);
  g.fchunks = (T + fl - 1) / fl;
  g.ftiles = g.nstrips * g.fchunks;
  return g;
}

// Forward monoid over (A, B) pairs, C channels per lane: x = [A0..A_{C-1}, B0..B_{C-1}].
template <int C>
struct FwdMonoid {
  static constexpr int NF = 2 * C;
  __device__ static void identity(float (&x)[NF]) {
#pragma unroll
    for (int c = 0; c < C; ++c) { x[c] = 1.f; x[C + c] = 0.f; }
  }
  // earlier then later: (A_l A_e, A_l B_e + B_l)
  __device__ static void combine(const float (&e)[NF], const float (&l)[NF], float (&o)[NF]) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      o[C + c] = fmaf(l[c], e[C + c], l[C + c]);
      o[c] = l[c] * e[c];
    }
  }
};

// Reverse monoid over the adjoint carries Y_t = a_t (g_t + Y_{t+1}), two
// adjoints (for A and for Bc) sharing the transition: x = [P, QA, QB] per channel.
template <int C>
struct RevMonoid {
  static constexpr int NF = 3 * C;
  __device__ static void identity(float (&x)[NF]) {
#pragma unroll
    for (int c = 0; c < C; ++c) { x[c] = 1.f; x[C + c] = 0.f; x[2 * C + c] = 0.f; }
  }
  __device__ static void combine(const float (&e)[NF], const float (&l)[NF], float (&o)[NF]) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      o[C + c] = fmaf(l[c], e[C + c], l[C + c]);
      o[2 * C + c] = fmaf(l[c], e[2 * C + c], l[2 * C + c]);
      o[c] = l[c] * e[c];
    }
  }
};

// acc <- acc then later (the monoids' combine may write over its earlier operand).
template <class M, int NF>
__device__ __forceinline__ void combine_into(float (&acc)[NF], const float (&later)[NF]) {
  M::combine(acc, later, acc);
}

template <typename E>
struct Args {
  const E* a;
  const E* b;
  E* A;
  E* Bc;
  const E* gA;
  const E* gB;
  E* da;
  E* db;
  float* carries;  // forward: written (may be null); backward: read
  // Sequence-parallel carry-in (null = none), fp32 [2][B][D]: forward, the
  // state (A, B) the slice starts from; backward, the adjoints (Y_A, Y_B)
  // entering the slice from the later slices.
  const float* cin;
  long long T_, D, sper, nstrips;
  long long nchunks;  // tiles (direct) or chunks (strip) per strip for this launch
  long long ntiles;
  Lookback lb;
};

// Strip-path tensor maps of the streamed inputs: (B, T, D) boxes of
// 32 channels x kLc steps (forward: a, b; backward: a, b, gA, gBc).
struct StripMaps {
  CUtensorMap m[4];
  CUtensorMap out[2];  // strip path: the two results (A, Bc or da, db), same boxes
};

// ------------------------------------------------------ shared step maths --

template <int C, int S>
__device__ __forceinline__ void fwd_agg(const float (&av)[S][C], const float (&bv)[S][C],
                                        float (&agg)[2 * C]) {
  FwdMonoid<C>::identity(agg);
#pragma unroll
  for (int s = 0; s < S; ++s)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      agg[C + c] = fmaf(av[s][c], agg[C + c], bv[s][c]);
      agg[c] *= av[s][c];
    }
}

template <int C, int S>
__device__ __forceinline__ void rev_agg(const float (&av)[S][C], const float (&ga)[S][C],
                                        const float (&gb)[S][C], float (&ragg)[3 * C]) {
  RevMonoid<C>::identity(ragg);
#pragma unroll
  for (int s = S - 1; s >= 0; --s)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      ragg[C + c] = av[s][c] * (ga[s][c] + ragg[C + c]);
      ragg[2 * C + c] = av[s][c] * (gb[s][c] + ragg[2 * C + c]);
      ragg[c] *= av[s][c];
    }
}

// Replay S forward steps from `cur`, storing A and Bc.
template <typename E, int C, int S>
__device__ __forceinline__ void fwd_emit(const Args<E>& p, const float (&av)[S][C],
                                         const float (&bv)[S][C], float (&cur)[2 * C], bool dok,
                                         long long t0, size_t base) {
#pragma unroll
  for (int s = 0; s < S; ++s) {
    float oa[C], ob[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      cur[C + c] = fmaf(av[s][c], cur[C + c], bv[s][c]);
      cur[c] *= av[s][c];
      oa[c] = cur[c];
      ob[c] = cur[C + c];
    }
    const long long t = t0 + s;
    if (dok && t < p.T_) {
      store_vec<E, C>(p.A + base + t * p.D, oa);
      store_vec<E, C>(p.Bc + base + t * p.D, ob);
    }
  }
}

// Per-thread backward of S steps given its forward start state (fcur) and
// the adjoint entering from later steps (ya, yb): writes da, db.
template <typename E, int C, int S>
__device__ __forceinline__ void bwd_emit(const Args<E>& p, const float (&av)[S][C],
                                         const float (&bv)[S][C], const float (&ga)[S][C],
                                         const float (&gb)[S][C], float (&fcur)[2 * C],
                                         float (&ya)[C], float (&yb)[C], bool dok, long long t0,
                                         size_t base) {
  float ap[S][C], bp[S][C];
#pragma unroll
  for (int s = 0; s < S; ++s)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      ap[s][c] = fcur[c];
      bp[s][c] = fcur[C + c];
      fcur[C + c] = fmaf(av[s][c], fcur[C + c], bv[s][c]);
      fcur[c] *= av[s][c];
    }
#pragma unroll
  for (int s = S - 1; s >= 0; --s) {
    float oda[C], odb[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float GA = ga[s][c] + ya[c];
      const float GB = gb[s][c] + yb[c];
      oda[c] = fmaf(GA, ap[s][c], GB * bp[s][c]);
      odb[c] = GB;
      ya[c] = av[s][c] * GA;
      yb[c] = av[s][c] * GB;
    }
    const long long t = t0 + s;
    if (dok && t < p.T_) {
      const size_t o = base + t * p.D;
      store_vec<E, C>(p.da + o, oda);
      store_vec<E, C>(p.db + o, odb);
    }
  }
}

// ------------------------------------------------------------ direct path --

template <typename E, int C, int S, int NW>
__global__ void __launch_bounds__(NW * 32) fwd_direct_kernel(Args<E> p) {
  using M = FwdMonoid<C>;
  constexpr int NF = M::NF;
  constexpr int L = S * NW;
  __shared__ unsigned s_tile;
  __shared__ float s_agg[NW][NF][32];
  __shared__ float s_ex[NF][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long tile = s_tile;
  if (tile >= p.ntiles) return;  // only when a test starts the counter past 0
  const long long chunk = tile / p.nstrips;
  const long long strip = tile - chunk * p.nstrips;
  const long long bi = strip / p.sper;
  const long long d0 = (strip - bi * p.sper) * (32LL * C) + (long long)lane * C;
  const bool dok = d0 < p.D;
  const long long t0 = chunk * L + (long long)warp * S;
  const size_t base = (size_t)bi * p.T_ * p.D + d0;

  float av[S][C], bv[S][C];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const long long t = t0 + s;
    if (dok && t < p.T_) {
      load_vec<E, C>(p.a + base + t * p.D, av[s]);
      load_vec<E, C>(p.b + base + t * p.D, bv[s]);
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) { av[s][c] = 1.f; bv[s][c] = 0.f; }
    }
  }
  float agg[NF];
  fwd_agg<C, S>(av, bv, agg);
#pragma unroll
  for (int f = 0; f < NF; ++f) s_agg[warp][f][lane] = agg[f];
  __syncthreads();

  if (warp == 0) {
    float tot[NF], w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) tot[f] = s_agg[0][f][lane];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
      combine_into<M, NF>(tot, w_);
    }
    float ex[NF], seed[NF];
    const bool seeded = p.cin != nullptr && chunk == 0;
    if (seeded) {  // the carried-in state (A_in, B_in) starts strip position 0
      const size_t bd = (size_t)(p.nstrips / p.sper) * p.D, o = (size_t)bi * p.D + d0;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const bool ok = dok && d0 + c < p.D;
        seed[c] = ok ? p.cin[o + c] : 1.f;
        seed[C + c] = ok ? p.cin[bd + o + c] : 0.f;
      }
    }
    warp_lookback_win<M, NF>(p.lb, tile, p.nstrips, chunk, tot, ex, seeded ? seed : nullptr);
#pragma unroll
    for (int f = 0; f < NF; ++f) s_ex[f][lane] = ex[f];
  }
  __syncthreads();

  float cur[NF], w_[NF];
#pragma unroll
  for (int f = 0; f < NF; ++f) cur[f] = s_ex[f][lane];
  for (int w = 0; w < warp; ++w) {
#pragma unroll
    for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
    combine_into<M, NF>(cur, w_);
  }
  if (p.carries != nullptr && ((warp * S) % kLc) == 0 && t0 < p.T_) {
    float* dst = p.carries + (size_t)((t0 / kLc) * p.nstrips + strip) * NF * 32;
#pragma unroll
    for (int f = 0; f < NF; ++f) __stcs(dst + f * 32 + lane, cur[f]);
  }
  fwd_emit<E, C, S>(p, av, bv, cur, dok, t0, base);
}

template <typename E, int C, int S, int NW>
__global__ void __launch_bounds__(NW * 32) bwd_direct_kernel(Args<E> p) {
  using FM = FwdMonoid<C>;
  using RM = RevMonoid<C>;
  constexpr int NFF = FM::NF, NFR = RM::NF;
  constexpr int L = S * NW;
  static_assert(L == kLc, "backward tile = carry chunk");
  __shared__ unsigned s_tile;
  __shared__ float s_fagg[NW][NFF][32];
  __shared__ float s_ragg[NW][NFR][32];
  __shared__ float s_fex[NFF][32];
  __shared__ float s_rex[NFR][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long tile = s_tile;                   // position in reverse processing order
  if (tile >= p.ntiles) return;  // only when a test starts the counter past 0
  const long long rchunk = tile / p.nstrips;
  const long long strip = tile - rchunk * p.nstrips;
  const long long chunk = p.nchunks - 1 - rchunk;  // time chunk
  const long long bi = strip / p.sper;
  const long long d0 = (strip - bi * p.sper) * (32LL * C) + (long long)lane * C;
  const bool dok = d0 < p.D;
  const long long t0 = chunk * L + (long long)warp * S;
  const size_t base = (size_t)bi * p.T_ * p.D + d0;

  float av[S][C], bv[S][C], ga[S][C], gb[S][C];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const long long t = t0 + s;
    if (dok && t < p.T_) {
      const size_t o = base + t * p.D;
      load_vec<E, C>(p.a + o, av[s]);
      load_vec<E, C>(p.b + o, bv[s]);
      load_vec<E, C>(p.gA + o, ga[s]);
      load_vec<E, C>(p.gB + o, gb[s]);
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) { av[s][c] = 1.f; bv[s][c] = 0.f; ga[s][c] = 0.f; gb[s][c] = 0.f; }
    }
  }
  float fagg[NFF], ragg[NFR];
  fwd_agg<C, S>(av, bv, fagg);
  rev_agg<C, S>(av, ga, gb, ragg);
#pragma unroll
  for (int f = 0; f < NFF; ++f) s_fagg[warp][f][lane] = fagg[f];
#pragma unroll
  for (int f = 0; f < NFR; ++f) s_ragg[warp][f][lane] = ragg[f];
  __syncthreads();

  if (warp == 0) {
    float tot[NFR], w_[NFR];
#pragma unroll
    for (int f = 0; f < NFR; ++f) tot[f] = s_ragg[NW - 1][f][lane];
#pragma unroll
    for (int w = NW - 2; w >= 0; --w) {
#pragma unroll
      for (int f = 0; f < NFR; ++f) w_[f] = s_ragg[w][f][lane];
      combine_into<RM, NFR>(tot, w_);
    }
    float ex[NFR], seed[NFR];
    const bool seeded = p.cin != nullptr && rchunk == 0;
    if (seeded) {  // the adjoints (Y_A, Y_B) entering from later slices
      const size_t bd = (size_t)(p.nstrips / p.sper) * p.D, o = (size_t)bi * p.D + d0;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const bool ok = dok && d0 + c < p.D;
        seed[c] = 1.f;
        seed[C + c] = ok ? p.cin[o + c] : 0.f;
        seed[2 * C + c] = ok ? p.cin[bd + o + c] : 0.f;
      }
    }
    warp_lookback_win<RM, NFR>(p.lb, tile, p.nstrips, rchunk, tot, ex, seeded ? seed : nullptr);
#pragma unroll
    for (int f = 0; f < NFR; ++f) s_rex[f][lane] = ex[f];
  } else if (warp == 1) {
    const float* src = p.carries + (size_t)(chunk * p.nstrips + strip) * NFF * 32;
#pragma unroll
    for (int f = 0; f < NFF; ++f) s_fex[f][lane] = __ldcs(src + f * 32 + lane);
  }
  __syncthreads();

  float fcur[NFF], rcur[NFR];
  {
    float w_[NFF];
#pragma unroll
    for (int f = 0; f < NFF; ++f) fcur[f] = s_fex[f][lane];
    for (int w = 0; w < warp; ++w) {
#pragma unroll
      for (int f = 0; f < NFF; ++f) w_[f] = s_fagg[w][f][lane];
      combine_into<FM, NFF>(fcur, w_);
    }
  }
  {
    float w_[NFR];
#pragma unroll
    for (int f = 0; f < NFR; ++f) rcur[f] = s_rex[f][lane];
    for (int w = NW - 1; w > warp; --w) {
#pragma unroll
      for (int f = 0; f < NFR; ++f) w_[f] = s_ragg[w][f][lane];
      combine_into<RM, NFR>(rcur, w_);
    }
  }
  float ya[C], yb[C];
#pragma unroll
  for (int c = 0; c < C; ++c) { ya[c] = rcur[C + c]; yb[c] = rcur[2 * C + c]; }
  bwd_emit<E, C, S>(p, av, bv, ga, gb, fcur, ya, yb, dok, t0, base);
}

// ------------------------------------------------------------- strip path --
//
// One warp per 32-channel strip walks all of T with the recurrence itself
// (lane = channel): no aggregates and no exchange between warps. Each warp
// streams its strip in IO chunks (TMA boxes of 32 channels x 32 or 64 steps;
// backward: plus the forward carry of each 32-step chunk inside) through a
// private ring of NST stages in shared memory; lane 0 refills a stage with
// the IO chunk NST ahead as soon as the warp has read it, and writes the
// chunk's results back by TMA box stores from two output buffers. Strips are dealt to warps CTA-first (strip =
// warp * gridDim.x + blockIdx.x, then + NW * gridDim.x), so the SMs' strip
// counts differ by at most one. The forward writes the strip state at every
// chunk start (the carries); the backward recomputes each chunk's states from
// them in registers and carries the adjoint in reverse.
//
// The walk is bound by one warp's serial path per chunk (ring wait, shared
// loads, 32 dependent steps, TMA issue) more than by the SM: 16-bit inputs,
// with half the bytes per chunk, stay below HBM bandwidth, fp32 reaches it.
//
// Each chunk's inputs are read into registers before any result is written:
// the stage and the output buffers are one shared array, so the compiler
// keeps every shared load behind the stores written before it, and a walk
// interleaving them would pay a load latency per step.
//
// Rows past T arrive zero-filled (TMA out-of-bounds fill). They come after
// every valid step of the strip and their results are clipped by the box
// stores; the backward walks only the valid rows of the chunk holding T's
// end, so an adjoint carried in from a later slice reaches step T - 1 intact.

constexpr int kWsWarps = 4;                  // warps (strips in flight) per CTA
constexpr size_t kWsRingPerWarp = 50 * 1024; // shared memory per warp: ring + output buffers

// Rows per TMA box ("IO chunk"). The 16-bit backward takes two 32-step carry
// chunks per box, so a chunk's fixed costs (ring wait, five copies, proxy
// fence, buffer turnaround) are paid every 64 steps (measured 152 -> 131 us
// at config 2); its forward is slower that way (118.7 vs 108.5 us), and an fp32 ring of
// 64-row boxes would not fit beside its output buffers.
template <typename E, bool BWD>
constexpr int ws_io() { return BWD && sizeof(E) == 2 ? 2 * kLc : kLc; }

// Per warp: NST input stages and two output buffers (an IO chunk's two result
// arrays, written back by TMA box stores while the next one is computed).
template <typename E, int NIN, bool WITH_CARRY, int NW>
struct WsStage {
  static constexpr int IO = ws_io<E, WITH_CARRY>(), NH = IO / kLc;  // rows per box, carry chunks per box
  static constexpr size_t kArrayBytes = (size_t)IO * 32 * sizeof(E);
  static constexpr size_t kCarryBytes = WITH_CARRY ? 2 * 32 * sizeof(float) : 0;  // per carry chunk
  static constexpr size_t kBytes = (NIN * kArrayBytes + NH * kCarryBytes + 127) / 128 * 128;
  static constexpr size_t kOutBytes = 2 * kArrayBytes;  // one output buffer (two arrays)
  static constexpr int kFit = (int)((kWsRingPerWarp - 2 * kOutBytes) / kBytes);
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr size_t kWarpBytes = kStages * kBytes + 2 * kOutBytes;
  static constexpr size_t kSmem = (size_t)NW * kWarpBytes;
  static_assert(kStages >= 2, "ring too shallow");
};

// Per-warp ring bookkeeping (lane 0 issues, every lane waits): IO chunk j of
// the warp's whole sequence uses slot j % NST with phase (j / NST) & 1.
template <int NST>
struct WsRing {
  uint64_t* full;
  unsigned pending = 0u, pend_ph = 0u;  // slots issued and not yet waited for
  __device__ void issued(int s, unsigned ph) {
    pending |= 1u << s;
    pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
  }
  __device__ bool wait(int s, unsigned ph, unsigned* err) {
    pending &= ~(1u << s);
    return mbar_wait(&full[s], ph, err);
  }
  // After a failed wait: let every copy still in flight land before exiting.
  __device__ void drain(unsigned* err) {
    for (int i = 0; i < NST; ++i)
      if (pending & (1u << i)) mbar_wait(&full[i], (pend_ph >> i) & 1u, err);
  }
};

template <typename E, int NW>
__global__ void __launch_bounds__(NW * 32, 1)
    fwd_strip_kernel(Args<E> p, const __grid_constant__ StripMaps maps) {
  using SS = WsStage<E, 2, false, NW>;
  constexpr int NST = SS::kStages, IO = SS::IO, NH = SS::NH;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t full[NW][NST];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    for (int i = 0; i < NST; ++i) mbar_init(&full[warp][i], 1);
    mbar_fence_init();
    tma_prefetch_desc(&maps.m[0]);
    tma_prefetch_desc(&maps.m[1]);
  }
  __syncwarp();
  unsigned char* wring = ring + (size_t)warp * SS::kWarpBytes;
  unsigned char* wout = wring + (size_t)NST * SS::kBytes;  // two output buffers
  WsRing<NST> rg;
  rg.full = full[warp];
  const long long nio = (p.nchunks + NH - 1) / NH;  // IO chunks per strip
  long long j0 = 0;  // IO chunks of earlier strips taken by this warp
  for (long long strip = (long long)warp * gridDim.x + blockIdx.x; strip < p.nstrips;
       strip += (long long)NW * gridDim.x) {
    const long long bi = strip / p.sper;
    const int d0 = (int)((strip - bi * p.sper) * 32);
    auto issue = [&](long long c) {  // lane 0: IO chunk c of this strip
      const long long j = j0 + c;
      const int s = (int)(j % NST);
      unsigned char* st = wring + (size_t)s * SS::kBytes;
      mbar_arrive_expect_tx(&rg.full[s], (unsigned)(2 * SS::kArrayBytes));
      tma_load_3d(st, &maps.m[0], d0, (int)(c * IO), (int)bi, &rg.full[s]);
      tma_load_3d(st + SS::kArrayBytes, &maps.m[1], d0, (int)(c * IO), (int)bi, &rg.full[s]);
      rg.issued(s, (unsigned)(j / NST) & 1u);
    };
    if (lane == 0)
      for (long long c = 0; c < NST && c < nio; ++c) issue(c);
    float A = 1.f, Bv = 0.f;
    if (p.cin != nullptr && d0 + lane < p.D) {  // carried-in state of the slice
      const size_t o = (size_t)bi * p.D + d0 + lane;
      A = p.cin[o];
      Bv = p.cin[(size_t)(p.nstrips / p.sper) * p.D + o];
    }
    for (long long c = 0; c < nio; ++c) {
      const long long j = j0 + c;
      const int s = (int)(j % NST);
      if (!rg.wait(s, (unsigned)(j / NST) & 1u, p.lb.err)) {
        if (lane == 0) {
          rg.drain(p.lb.err);
          bulk_wait_read();
        }
        return;
      }
      unsigned char* ob = wout + (size_t)(j & 1) * SS::kOutBytes;
#pragma unroll 1
      for (int h = 0; h < NH; ++h) {  // carry chunks of this IO chunk
        const long long cc = c * NH + h;
        if (p.carries != nullptr && cc < p.nchunks) {
          float* dst = p.carries + (size_t)(cc * p.nstrips + strip) * 2 * 32;
          __stcs(dst + lane, A);
          __stcs(dst + 32 + lane, Bv);
        }
        const E* sa = reinterpret_cast<const E*>(wring + (size_t)s * SS::kBytes) + h * kLc * 32 + lane;
        const E* sb = sa + SS::kArrayBytes / sizeof(E);
        E va[kLc], vb[kLc];
#pragma unroll
        for (int i = 0; i < kLc; ++i) {
          va[i] = sa[i * 32];
          vb[i] = sb[i * 32];
        }
        if (h == 0) {
          if (lane == 0) bulk_wait_read_1();  // the stores of IO chunk j - 2 have read this buffer
          __syncwarp();
        }
        E* oA = reinterpret_cast<E*>(ob) + h * kLc * 32 + lane;
        E* oB = oA + SS::kArrayBytes / sizeof(E);
#pragma unroll
        for (int i = 0; i < kLc; ++i) {
          const float a = to_f32<E>(va[i]);
          Bv = fmaf(a, Bv, to_f32<E>(vb[i]));
          A *= a;
          oA[i * 32] = from_f32<E>(A);
          oB[i * 32] = from_f32<E>(Bv);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (c + NST < nio) issue(c + NST);
        tma_store_3d(&maps.out[0], d0, (int)(c * IO), (int)bi, ob);
        tma_store_3d(&maps.out[1], d0, (int)(c * IO), (int)bi, ob + SS::kArrayBytes);
        bulk_commit();
      }
    }
    j0 += nio;
  }
  if (lane == 0) bulk_wait_read();
}

template <typename E, int NW>
__global__ void __launch_bounds__(NW * 32, 1)
    bwd_strip_kernel(Args<E> p, const __grid_constant__ StripMaps maps) {
  using SS = WsStage<E, 4, true, NW>;
  constexpr int NST = SS::kStages, IO = SS::IO, NH = SS::NH;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t full[NW][NST];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    for (int i = 0; i < NST; ++i) mbar_init(&full[warp][i], 1);
    mbar_fence_init();
    for (int i = 0; i < 4; ++i) tma_prefetch_desc(&maps.m[i]);
  }
  __syncwarp();
  unsigned char* wring = ring + (size_t)warp * SS::kWarpBytes;
  unsigned char* wout = wring + (size_t)NST * SS::kBytes;  // two output buffers
  WsRing<NST> rg;
  rg.full = full[warp];
  const long long nio = (p.nchunks + NH - 1) / NH;
  long long j0 = 0;
  for (long long strip = (long long)warp * gridDim.x + blockIdx.x; strip < p.nstrips;
       strip += (long long)NW * gridDim.x) {
    const long long bi = strip / p.sper;
    const int d0 = (int)((strip - bi * p.sper) * 32);
    auto issue = [&](long long c) {  // lane 0: step c handles IO chunk nio - 1 - c
      const long long io = nio - 1 - c;
      const long long j = j0 + c;
      const int s = (int)(j % NST);
      unsigned char* st = wring + (size_t)s * SS::kBytes;
      const int nc = (int)min((long long)NH, p.nchunks - io * NH);  // carry chunks inside T
      mbar_arrive_expect_tx(&rg.full[s], (unsigned)(4 * SS::kArrayBytes + nc * SS::kCarryBytes));
#pragma unroll
      for (int arr = 0; arr < 4; ++arr)
        tma_load_3d(st + arr * SS::kArrayBytes, &maps.m[arr], d0, (int)(io * IO), (int)bi,
                    &rg.full[s]);
      for (int h = 0; h < nc; ++h)
        bulk_g2s(st + 4 * SS::kArrayBytes + h * SS::kCarryBytes,
                 p.carries + (size_t)((io * NH + h) * p.nstrips + strip) * 2 * 32,
                 (unsigned)SS::kCarryBytes, &rg.full[s]);
      rg.issued(s, (unsigned)(j / NST) & 1u);
    };
    if (lane == 0)
      for (long long c = 0; c < NST && c < nio; ++c) issue(c);
    float ya = 0.f, yb = 0.f;  // adjoints entering from later steps
    if (p.cin != nullptr && d0 + lane < p.D) {  // ... and from later slices
      const size_t o = (size_t)bi * p.D + d0 + lane;
      ya = p.cin[o];
      yb = p.cin[(size_t)(p.nstrips / p.sper) * p.D + o];
    }
    for (long long c = 0; c < nio; ++c) {
      const long long io = nio - 1 - c;
      const long long j = j0 + c;
      const int s = (int)(j % NST);
      if (!rg.wait(s, (unsigned)(j / NST) & 1u, p.lb.err)) {
        if (lane == 0) {
          rg.drain(p.lb.err);
          bulk_wait_read();
        }
        return;
      }
      const unsigned char* st = wring + (size_t)s * SS::kBytes;
      unsigned char* ob = wout + (size_t)(j & 1) * SS::kOutBytes;
      if (lane == 0) bulk_wait_read_1();  // the stores of step j - 2 have read this buffer
      __syncwarp();
#pragma unroll 1
      for (int h = NH - 1; h >= 0; --h) {  // carry chunks of this IO chunk, in reverse
        if (io * NH + h >= p.nchunks) continue;  // past T: its rows are clipped by the stores
        const E* sa = reinterpret_cast<const E*>(st) + h * kLc * 32 + lane;
        const E* sb = sa + SS::kArrayBytes / sizeof(E);
        const E* sga = sb + SS::kArrayBytes / sizeof(E);
        const E* sgb = sga + SS::kArrayBytes / sizeof(E);
        const float* fc = reinterpret_cast<const float*>(st + 4 * SS::kArrayBytes + h * SS::kCarryBytes);
        float fA = fc[lane], fB = fc[32 + lane];
        E* oA = reinterpret_cast<E*>(ob) + h * kLc * 32 + lane;
        E* oB = oA + SS::kArrayBytes / sizeof(E);
        float ap[kLc], bp[kLc];  // states before each step of the carry chunk
#pragma unroll
        for (int i = 0; i < kLc; ++i) {
          const float a = to_f32<E>(sa[i * 32]);
          ap[i] = fA;
          bp[i] = fB;
          fB = fmaf(a, fB, to_f32<E>(sb[i * 32]));
          fA *= a;
        }
        // Reverse walk in groups of kGrp steps, each group's inputs read first.
        // In the chunk holding T's end, the zero-filled rows past T must not
        // touch the adjoint (it may carry another slice's adjoint in).
        constexpr int kGrp = 8;
        const long long nvalid = p.T_ - (io * NH + h) * kLc;
        if (nvalid >= kLc) {
#pragma unroll
          for (int g = kLc / kGrp - 1; g >= 0; --g) {
            E va[kGrp], vga[kGrp], vgb[kGrp];
#pragma unroll
            for (int k = 0; k < kGrp; ++k) {
              va[k] = sa[(g * kGrp + k) * 32];
              vga[k] = sga[(g * kGrp + k) * 32];
              vgb[k] = sgb[(g * kGrp + k) * 32];
            }
#pragma unroll
            for (int k = kGrp - 1; k >= 0; --k) {
              const int i = g * kGrp + k;
              const float a = to_f32<E>(va[k]);
              const float GA = to_f32<E>(vga[k]) + ya, GB = to_f32<E>(vgb[k]) + yb;
              ya = a * GA;
              yb = a * GB;
              oA[i * 32] = from_f32<E>(fmaf(GA, ap[i], GB * bp[i]));
              oB[i * 32] = from_f32<E>(GB);
            }
          }
        } else {  // unrolled with a predicate, so ap / bp keep static indices (registers)
#pragma unroll
          for (int i = kLc - 1; i >= 0; --i) {
            if (i < nvalid) {
              const float a = to_f32<E>(sa[i * 32]);
              const float GA = to_f32<E>(sga[i * 32]) + ya, GB = to_f32<E>(sgb[i * 32]) + yb;
              ya = a * GA;
              yb = a * GB;
              oA[i * 32] = from_f32<E>(fmaf(GA, ap[i], GB * bp[i]));
              oB[i * 32] = from_f32<E>(GB);
            }
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (c + NST < nio) issue(c + NST);
        tma_store_3d(&maps.out[0], d0, (int)(io * IO), (int)bi, ob);
        tma_store_3d(&maps.out[1], d0, (int)(io * IO), (int)bi, ob + SS::kArrayBytes);
        bulk_commit();
      }
    }
    j0 += nio;
  }
  if (lane == 0) bulk_wait_read();
}

// ---------------------------------------------------------------- launch --

template <class K>
int launch_persistent(K kernel, int threads, size_t dyn_smem, long long units, void** kargs,
                      cudaStream_t st) {
  // Static + dynamic shared memory above 48 KB needs the opt-in attribute.
  MGS_CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)dyn_smem));
  int per_sm = 0;
  MGS_CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, dyn_smem));
  if (per_sm < 1) return MGS_LAUNCH_FAILED;
  long long grid = (long long)per_sm * sm_count();
  if (grid > units) grid = units;
  MGS_CUDA_OK(cudaLaunchKernel((const void*)kernel, dim3((unsigned)grid), dim3(threads), kargs,
                               dyn_smem, st));
  return MGS_OK;
}

inline int nf_max(const Geometry& g) { return 3 * g.cpt; }

inline size_t workspace_bytes(const Geometry& g) {
  if (g.algo == kStrip) return 256;  // no look-back
  return lookback_bytes(g.ntiles > g.ftiles ? g.ntiles : g.ftiles, nf_max(g));
}

template <typename E>
int run(bool fwd, const void* a, const void* b, void* A, void* Bc, const void* gA,
        const void* gB, void* da, void* db, void* carries, long long B, long long T,
        long long D, int dtype, void* ws, size_t ws_bytes, cudaStream_t st,
        const float* cin = nullptr) {
  const Geometry g = geometry(B, T, D, dtype);
  if (g.ntiles == 0) return MGS_OK;
  if (g.ntiles > 0x7fffffffLL) return MGS_UNSUPPORTED;
  if (ws == nullptr || ws_bytes < workspace_bytes(g)) return MGS_WORKSPACE_TOO_SMALL;
  const size_t va = g.algo == kDirectScalar ? sizeof(E) : 16;
  const void* ptrs[6] = {a, b, fwd ? A : gA, fwd ? Bc : gB, fwd ? nullptr : da,
                         fwd ? nullptr : db};
  for (const void* q : ptrs)
    if (q != nullptr && !aligned(q, va)) return MGS_BAD_ALIGNMENT;
  if (!aligned(ws, 256) || (carries != nullptr && !aligned(carries, 16))) return MGS_BAD_ALIGNMENT;
  if (!fwd && carries == nullptr) return MGS_BAD_SHAPE;
  Args<E> p{};
  p.cin = cin;
  p.a = static_cast<const E*>(a);
  p.b = static_cast<const E*>(b);
  p.A = static_cast<E*>(A);
  p.Bc = static_cast<E*>(Bc);
  p.gA = static_cast<const E*>(gA);
  p.gB = static_cast<const E*>(gB);
  p.da = static_cast<E*>(da);
  p.db = static_cast<E*>(db);
  p.carries = static_cast<float*>(carries);
  p.T_ = T;
  p.D = D;
  p.sper = g.sper;
  p.nstrips = g.nstrips;
  if (g.algo == kStrip) {
    p.nchunks = g.nchunks;
    p.ntiles = g.ntiles;
    MGS_CUDA_OK(cudaMemsetAsync(ws, 0, 256, st));  // error word
    p.lb = lookback_view(ws, 0, 0);
    StripMaps maps;
    const unsigned io = fwd ? (unsigned)ws_io<E, false>() : (unsigned)ws_io<E, true>();
    const void* src[4] = {a, b, gA, gB};
    for (int i = 0; i < (fwd ? 2 : 4); ++i)
      if (!make_tmap_3d<E>(&maps.m[i], src[i], D, T, B, 32u, io)) return MGS_LAUNCH_FAILED;
    void* dst[2] = {fwd ? A : da, fwd ? Bc : db};
    for (int i = 0; i < 2; ++i)
      if (!make_tmap_3d<E>(&maps.out[i], dst[i], D, T, B, 32u, io)) return MGS_LAUNCH_FAILED;
    void* kargs[] = {&p, &maps};
    // one CTA of kWsWarps warps per SM (the rings fill its shared memory)
    const long long units = (g.nstrips + kWsWarps - 1) / kWsWarps;
    if (fwd)
      return launch_persistent(fwd_strip_kernel<E, kWsWarps>, kWsWarps * 32,
                               WsStage<E, 2, false, kWsWarps>::kSmem, units, kargs, st);
    return launch_persistent(bwd_strip_kernel<E, kWsWarps>, kWsWarps * 32,
                             WsStage<E, 4, true, kWsWarps>::kSmem, units, kargs, st);
  }
  const long long lbt = g.ntiles > g.ftiles ? g.ntiles : g.ftiles;
  MGS_CUDA_OK(cudaMemsetAsync(ws, 0, lookback_zero_bytes(lbt), st));
  p.lb = lookback_view(ws, lbt, nf_max(g));
  if (fwd) {
    p.nchunks = g.fchunks;
    p.ntiles = g.ftiles;
    if (g.algo == kDirectVec)
      fwd_direct_kernel<E, kVecCpt, kVecFwdS, kVecFwdNW>
          <<<(unsigned)g.ftiles, kVecFwdNW * 32, 0, st>>>(p);
    else
      fwd_direct_kernel<E, 1, kSclFwdS, kSclFwdNW><<<(unsigned)g.ftiles, kSclFwdNW * 32, 0, st>>>(p);
  } else {
    p.nchunks = g.nchunks;
    p.ntiles = g.ntiles;
    if (g.algo == kDirectVec)
      bwd_direct_kernel<E, kVecCpt, kBwdS, kBwdNW><<<(unsigned)g.ntiles, kBwdNW * 32, 0, st>>>(p);
    else
      bwd_direct_kernel<E, 1, kBwdS, kBwdNW><<<(unsigned)g.ntiles, kBwdNW * 32, 0, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

int dispatch(bool fwd, const void* a, const void* b, void* A, void* Bc, const void* gA,
             const void* gB, void* da, void* db, void* carries, long long B, long long T,
             long long D, int dtype, void* ws, size_t ws_bytes, cudaStream_t st,
             const float* cin = nullptr) {
  if (B < 0 || T < 0 || D < 0) return MGS_BAD_SHAPE;
  if (cin != nullptr && !aligned(cin, 4)) return MGS_BAD_ALIGNMENT;
  switch (dtype) {
    case MGS_F32:
      return run<float>(fwd, a, b, A, Bc, gA, gB, da, db, carries, B, T, D, dtype, ws, ws_bytes, st,
                        cin);
    case MGS_BF16:
      return run<__nv_bfloat16>(fwd, a, b, A, Bc, gA, gB, da, db, carries, B, T, D, dtype, ws,
                                ws_bytes, st, cin);
    case MGS_F16:
      return run<__half>(fwd, a, b, A, Bc, gA, gB, da, db, carries, B, T, D, dtype, ws, ws_bytes,
                         st, cin);
    default:
      return MGS_BAD_DTYPE;
  }
}

}  // namespace linear

unsigned take_error_linear(cudaStream_t s) { return take_sticky_error(s); }

// ------------------------------------------------------ time-out test hooks --
//
// Both hooks make a bounded wait run out on purpose, with a small poll bound,
// so a test can check the whole time-out path (error words set, launch
// completes, the host sees MGS_LOOKBACK_TIMEOUT, the context stays usable)
// without anything that could hang: every wait involved is bounded.

namespace linear {

// The forward direct path with the tile counter started at 1: no CTA takes
// tile 0, so the look-back of the tile after it in strip 0 waits on a flag
// that nothing sets. The tickets run 1..ntiles; the CTA that draws ntiles
// returns at once.
int run_lookback_stall(const float* a, const float* b, float* A, float* Bc, long long B,
                       long long T, long long D, void* ws, size_t ws_bytes, long long spin,
                       cudaStream_t st) {
  const Geometry g = geometry(B, T, D, MGS_F32);
  if (g.algo != kDirectVec || g.fchunks < 2) return MGS_UNSUPPORTED;  // needs a look-back
  if (spin < 1) return MGS_BAD_SHAPE;
  if (ws == nullptr || ws_bytes < workspace_bytes(g)) return MGS_WORKSPACE_TOO_SMALL;
  const void* ptrs[4] = {a, b, A, Bc};
  for (const void* q : ptrs)
    if (q == nullptr || !aligned(q, 16)) return MGS_BAD_ALIGNMENT;
  if (!aligned(ws, 256)) return MGS_BAD_ALIGNMENT;
  Args<float> p{};
  p.a = a;
  p.b = b;
  p.A = A;
  p.Bc = Bc;
  p.carries = nullptr;
  p.T_ = T;
  p.D = D;
  p.sper = g.sper;
  p.nstrips = g.nstrips;
  p.nchunks = g.fchunks;
  p.ntiles = g.ftiles;
  const long long lbt = g.ntiles > g.ftiles ? g.ntiles : g.ftiles;
  MGS_CUDA_OK(cudaMemsetAsync(ws, 0, lookback_zero_bytes(lbt), st));
  MGS_CUDA_OK(cudaMemsetAsync(ws, 1, 1, st));  // counter = 1 (little-endian u32)
  p.lb = lookback_view(ws, lbt, nf_max(g));
  p.lb.spin = spin;
  fwd_direct_kernel<float, kVecCpt, kVecFwdS, kVecFwdNW>
      <<<(unsigned)g.ftiles, kVecFwdNW * 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

// One CTA waits on an mbarrier that nothing arrives on.
__global__ void mbarrier_stall_kernel(unsigned* err, long long spin) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait(&bar, 0u, err, spin);
}

}  // namespace linear

// ------------------------------------------------ allocation-free variant --
//
// Scratch for mgs_linear_scan_fwd_noalloc: one fixed array per device, part
// of the library's device image, so the entry point needs no allocation.
// Host code cannot use `g_noalloc_scratch` as a device address (on the host
// the name is only a stand-in); the device address comes from
// cudaGetSymbolAddress, resolved once per device with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MGS_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;

// The array's address is resolved once per device and remembered together
// with the CUDA context it was resolved in: a device whose primary context
// was torn down and created again (cudaDeviceReset) gets a fresh address
// instead of a stale one.
struct ScratchSlot {
  CUcontext ctx;
  void* addr;
};
ScratchSlot g_scratch_slot[kMaxDevices] = {};
std::mutex g_scratch_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(ptr);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

void* noalloc_scratch_address() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    (void)cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch_slot[dev];
  const CUcontext ctx = current_context();
  if (slot.addr != nullptr && ctx != nullptr && slot.ctx == ctx) return slot.addr;
  // first call on this device, or its context changed: resolve the address
  // (this also makes the device's primary context current) and remember the
  // context it belongs to
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  slot.ctx = current_context();
  slot.addr = addr;
  return addr;
}
}  // namespace

}  // namespace mgs

extern "C" {

size_t mgs_linear_scan_workspace_size(int64_t B, int64_t T, int64_t D, int dtype) {
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || D < 0) return 0;
  const auto g = mgs::linear::geometry(B, T, D, dtype);
  return mgs::linear::workspace_bytes(g);
}

size_t mgs_linear_scan_carry_size(int64_t B, int64_t T, int64_t D, int dtype) {
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || D < 0) return 0;
  const auto g = mgs::linear::geometry(B, T, D, dtype);
  return (size_t)g.ntiles * 2 * g.cpt * 32 * sizeof(float);
}

int mgs_linear_scan_fwd(const void* a, const void* b, void* A, void* Bc, void* carries, int64_t B,
                        int64_t T, int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                        void* stream) {
  return mgs::linear::dispatch(true, a, b, A, Bc, nullptr, nullptr, nullptr, nullptr, carries, B, T,
                               D, dtype, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream));
}

int mgs_linear_scan_bwd(const void* a, const void* b, const void* gA, const void* gBc,
                        const void* carries, void* da, void* db, int64_t B, int64_t T, int64_t D,
                        int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return mgs::linear::dispatch(false, a, b, nullptr, nullptr, gA, gBc, da, db,
                               const_cast<void*>(carries), B, T, D, dtype, workspace,
                               workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mgs_linear_scan_fwd_fixup(const void* a, const void* b, const float* carry_in, void* A,
                              void* Bc, void* carries, int64_t B, int64_t T, int64_t D, int dtype,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (carry_in == nullptr) return MGS_BAD_SHAPE;
  return mgs::linear::dispatch(true, a, b, A, Bc, nullptr, nullptr, nullptr, nullptr, carries, B, T,
                               D, dtype, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream), carry_in);
}

int mgs_linear_scan_bwd_fixup(const void* a, const void* b, const void* gA, const void* gBc,
                              const void* carries, const float* adjoint_in, void* da, void* db,
                              int64_t B, int64_t T, int64_t D, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (adjoint_in == nullptr) return MGS_BAD_SHAPE;
  return mgs::linear::dispatch(false, a, b, nullptr, nullptr, gA, gBc, da, db,
                               const_cast<void*>(carries), B, T, D, dtype, workspace,
                               workspace_bytes, static_cast<cudaStream_t>(stream), adjoint_in);
}

int mgs_test_lookback_timeout(const void* a, const void* b, void* A, void* Bc, int64_t B,
                              int64_t T, int64_t D, void* workspace, size_t workspace_bytes,
                              int64_t spin_limit, void* stream) {
  if (B < 0 || T < 0 || D < 0) return MGS_BAD_SHAPE;
  return mgs::linear::run_lookback_stall(
      static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(A),
      static_cast<float*>(Bc), B, T, D, workspace, workspace_bytes, spin_limit,
      static_cast<cudaStream_t>(stream));
}

int mgs_test_mbarrier_timeout(void* err_word, int64_t spin_limit, void* stream) {
  if (err_word == nullptr || !mgs::aligned(err_word, 4)) return MGS_BAD_ALIGNMENT;
  if (spin_limit < 1) return MGS_BAD_SHAPE;
  mgs::linear::mbarrier_stall_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned*>(err_word), spin_limit);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

int mgs_linear_scan_fwd_noalloc(const void* a, const void* b, void* A, void* Bc, void* carries,
                                int64_t B, int64_t T, int64_t D, int dtype, void* stream) {
  if (mgs::dtype_size(dtype) == 0) return MGS_BAD_DTYPE;
  if (B < 0 || T < 0 || D < 0) return MGS_BAD_SHAPE;
  const auto g = mgs::linear::geometry(B, T, D, dtype);
  if (mgs::linear::workspace_bytes(g) > (size_t)MGS_NOALLOC_SCRATCH_BYTES)
    return MGS_WORKSPACE_TOO_SMALL;  // shape too large for the fixed scratch: use mgs_linear_scan_fwd
  void* scratch = mgs::noalloc_scratch_address();
  if (scratch == nullptr) return MGS_LAUNCH_FAILED;
  return mgs::linear::dispatch(true, a, b, A, Bc, nullptr, nullptr, nullptr, nullptr, carries, B,
                               T, D, dtype, scratch, (size_t)MGS_NOALLOC_SCRATCH_BYTES,
                               static_cast<cudaStream_t>(stream));
}

}  // extern "C"
