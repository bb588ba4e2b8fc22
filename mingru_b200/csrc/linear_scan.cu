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
// Design. A tile is L = S*NW time steps x 32*CPT channels: warp w owns steps
// [w*S, (w+1)*S) of the tile, lane l owns CPT adjacent channels (one 16-byte
// vector access per step), so every warp access is a fully coalesced row
// segment. Each thread reduces its S steps serially in registers; the NW warp
// aggregates are composed through shared memory; warp 0 runs the decoupled
// look-back across the strip's earlier tiles; every thread then replays its
// S steps from its exact carry and streams the outputs. The forward also
// writes each tile's chunk-start state ("carries", fp32), which lets the
// backward recompute A_{t-1}, Bc_{t-1} in registers instead of reading the
// saved outputs: the backward reads a, b, gA, gBc and writes da, db -- the
// algorithmic minimum -- and runs its own reverse look-back for G.
#include "common.cuh"

namespace mgs {
namespace linear {

// Tile geometry, shared by forward, backward, size queries and carries.
constexpr int kFwdS = 8, kFwdNW = 4;   // L = 32
constexpr int kBwdS = 4, kBwdNW = 8;   // L = 32
constexpr int kL = kFwdS * kFwdNW;
static_assert(kBwdS * kBwdNW == kL, "forward and backward tiles must match");

struct Geometry {
  int cpt;             // channels per lane
  long long sper;      // strips per batch row
  long long nstrips;   // B * sper
  long long nchunks;   // ceil(T / L)
  long long ntiles;
};

inline int vec_cpt(int dtype) { return 16 / dtype_size(dtype); }

inline Geometry geometry(long long B, long long T, long long D, int dtype) {
  Geometry g;
  const int vec = vec_cpt(dtype);
  g.cpt = (D % vec == 0) ? vec : 1;
  const long long w = 32LL * g.cpt;
  g.sper = (D + w - 1) / w;
  g.nstrips = B * g.sper;
  g.nchunks = (T + kL - 1) / kL;
  g.ntiles = g.nstrips * g.nchunks;
  return g;
}

// Forward monoid over (A, B) pairs, CPT channels per lane: x = [A0..A_{C-1}, B0..B_{C-1}].
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
  long long T_, D, sper, nstrips, nchunks;
  Lookback lb;
};

template <typename E, int C, int S, int NW>
__global__ void __launch_bounds__(NW * 32) fwd_kernel(Args<E> p) {
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
  M::identity(agg);
#pragma unroll
  for (int s = 0; s < S; ++s)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      agg[C + c] = fmaf(av[s][c], agg[C + c], bv[s][c]);
      agg[c] *= av[s][c];
    }
#pragma unroll
  for (int f = 0; f < NF; ++f) s_agg[warp][f][lane] = agg[f];
  __syncthreads();

  if (warp == 0) {
    float tot[NF], tmp[NF], w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) tot[f] = s_agg[0][f][lane];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
      M::combine(tot, w_, tmp);
#pragma unroll
      for (int f = 0; f < NF; ++f) tot[f] = tmp[f];
    }
    float ex[NF];
    warp_lookback<M, NF>(p.lb, tile, p.nstrips, chunk, tot, ex);
#pragma unroll
    for (int f = 0; f < NF; ++f) s_ex[f][lane] = ex[f];
    if (p.carries != nullptr) {
      float* dst = p.carries + (size_t)tile * NF * 32;
#pragma unroll
      for (int f = 0; f < NF; ++f) __stcs(dst + f * 32 + lane, ex[f]);
    }
  }
  __syncthreads();

  float cur[NF], tmp[NF], w_[NF];
#pragma unroll
  for (int f = 0; f < NF; ++f) cur[f] = s_ex[f][lane];
  for (int w = 0; w < warp; ++w) {
#pragma unroll
    for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
    M::combine(cur, w_, tmp);
#pragma unroll
    for (int f = 0; f < NF; ++f) cur[f] = tmp[f];
  }
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

template <typename E, int C, int S, int NW>
__global__ void __launch_bounds__(NW * 32) bwd_kernel(Args<E> p) {
  using FM = FwdMonoid<C>;
  using RM = RevMonoid<C>;
  constexpr int NFF = FM::NF, NFR = RM::NF;
  constexpr int L = S * NW;
  __shared__ unsigned s_tile;
  __shared__ float s_fagg[NW][NFF][32];
  __shared__ float s_ragg[NW][NFR][32];
  __shared__ float s_fex[NFF][32];
  __shared__ float s_rex[NFR][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long tile = s_tile;                 // position in reverse processing order
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
  // Local forward aggregate (for this warp's chunk-start state) and local
  // reverse aggregate (for the adjoint entering from later steps).
  float fagg[NFF], ragg[NFR];
  FM::identity(fagg);
  RM::identity(ragg);
#pragma unroll
  for (int s = 0; s < S; ++s)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      fagg[C + c] = fmaf(av[s][c], fagg[C + c], bv[s][c]);
      fagg[c] *= av[s][c];
    }
#pragma unroll
  for (int s = S - 1; s >= 0; --s)
#pragma unroll
    for (int c = 0; c < C; ++c) {
      ragg[C + c] = av[s][c] * (ga[s][c] + ragg[C + c]);
      ragg[2 * C + c] = av[s][c] * (gb[s][c] + ragg[2 * C + c]);
      ragg[c] *= av[s][c];
    }
#pragma unroll
  for (int f = 0; f < NFF; ++f) s_fagg[warp][f][lane] = fagg[f];
#pragma unroll
  for (int f = 0; f < NFR; ++f) s_ragg[warp][f][lane] = ragg[f];
  __syncthreads();

  if (warp == 0) {
    float tot[NFR], tmp[NFR], w_[NFR];
#pragma unroll
    for (int f = 0; f < NFR; ++f) tot[f] = s_ragg[NW - 1][f][lane];
#pragma unroll
    for (int w = NW - 2; w >= 0; --w) {
#pragma unroll
      for (int f = 0; f < NFR; ++f) w_[f] = s_ragg[w][f][lane];
      RM::combine(tot, w_, tmp);
#pragma unroll
      for (int f = 0; f < NFR; ++f) tot[f] = tmp[f];
    }
    float ex[NFR];
    warp_lookback<RM, NFR>(p.lb, tile, p.nstrips, rchunk, tot, ex);
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
    float tmp[NFF], w_[NFF];
#pragma unroll
    for (int f = 0; f < NFF; ++f) fcur[f] = s_fex[f][lane];
    for (int w = 0; w < warp; ++w) {
#pragma unroll
      for (int f = 0; f < NFF; ++f) w_[f] = s_fagg[w][f][lane];
      FM::combine(fcur, w_, tmp);
#pragma unroll
      for (int f = 0; f < NFF; ++f) fcur[f] = tmp[f];
    }
  }
  {
    float tmp[NFR], w_[NFR];
#pragma unroll
    for (int f = 0; f < NFR; ++f) rcur[f] = s_rex[f][lane];
    for (int w = NW - 1; w > warp; --w) {
#pragma unroll
      for (int f = 0; f < NFR; ++f) w_[f] = s_ragg[w][f][lane];
      RM::combine(rcur, w_, tmp);
#pragma unroll
      for (int f = 0; f < NFR; ++f) rcur[f] = tmp[f];
    }
  }
  // States before each step: A_{t-1}, Bc_{t-1} (bv is dead afterwards).
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
  float ya[C], yb[C];
#pragma unroll
  for (int c = 0; c < C; ++c) { ya[c] = rcur[C + c]; yb[c] = rcur[2 * C + c]; }
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

template <typename E, int C>
int launch_fwd(Args<E> p, const Geometry& g, cudaStream_t st) {
  fwd_kernel<E, C, kFwdS, kFwdNW><<<(unsigned)g.ntiles, kFwdNW * 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

template <typename E, int C>
int launch_bwd(Args<E> p, const Geometry& g, cudaStream_t st) {
  bwd_kernel<E, C, kBwdS, kBwdNW><<<(unsigned)g.ntiles, kBwdNW * 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

inline int nf_max(const Geometry& g) { return 3 * g.cpt; }

template <typename E>
int run(bool fwd, const void* a, const void* b, void* A, void* Bc, const void* gA,
        const void* gB, void* da, void* db, void* carries, long long B, long long T,
        long long D, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  const Geometry g = geometry(B, T, D, dtype);
  if (g.ntiles == 0) return MGS_OK;
  if (g.ntiles > 0x7fffffffLL) return MGS_UNSUPPORTED;
  if (ws == nullptr || ws_bytes < lookback_bytes(g.ntiles, nf_max(g)))
    return MGS_WORKSPACE_TOO_SMALL;
  const size_t va = (size_t)g.cpt * sizeof(E);
  const void* ptrs[8] = {a, b, fwd ? A : gA, fwd ? Bc : gB, fwd ? nullptr : da,
                         fwd ? nullptr : db, nullptr, nullptr};
  for (const void* q : ptrs)
    if (q != nullptr && !aligned(q, va)) return MGS_BAD_ALIGNMENT;
  if (!aligned(ws, 256) || (carries != nullptr && !aligned(carries, 16))) return MGS_BAD_ALIGNMENT;
  if (!fwd && carries == nullptr) return MGS_BAD_SHAPE;
  MGS_CUDA_OK(cudaMemsetAsync(ws, 0, lookback_zero_bytes(g.ntiles), st));
  Args<E> p;
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
  p.nchunks = g.nchunks;
  p.lb = lookback_view(ws, g.ntiles, nf_max(g));
  constexpr int V = 16 / sizeof(E);
  if (g.cpt == V) return fwd ? launch_fwd<E, V>(p, g, st) : launch_bwd<E, V>(p, g, st);
  return fwd ? launch_fwd<E, 1>(p, g, st) : launch_bwd<E, 1>(p, g, st);
}

int dispatch(bool fwd, const void* a, const void* b, void* A, void* Bc, const void* gA,
             const void* gB, void* da, void* db, void* carries, long long B, long long T,
             long long D, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (B < 0 || T < 0 || D < 0) return MGS_BAD_SHAPE;
  switch (dtype) {
    case MGS_F32:
      return run<float>(fwd, a, b, A, Bc, gA, gB, da, db, carries, B, T, D, dtype, ws, ws_bytes, st);
    case MGS_BF16:
      return run<__nv_bfloat16>(fwd, a, b, A, Bc, gA, gB, da, db, carries, B, T, D, dtype, ws,
                                ws_bytes, st);
    case MGS_F16:
      return run<__half>(fwd, a, b, A, Bc, gA, gB, da, db, carries, B, T, D, dtype, ws, ws_bytes,
                         st);
    default:
      return MGS_BAD_DTYPE;
  }
}

}  // namespace linear

unsigned take_error_linear(cudaStream_t s) { return take_sticky_error(s); }

}  // namespace mgs

extern "C" {

size_t mgs_linear_scan_workspace_size(int64_t B, int64_t T, int64_t D, int dtype) {
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || D < 0) return 0;
  const auto g = mgs::linear::geometry(B, T, D, dtype);
  return mgs::lookback_bytes(g.ntiles, mgs::linear::nf_max(g));
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

}  // extern "C"
