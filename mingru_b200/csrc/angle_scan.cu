// angle_scan.cu -- angle-fused Givens / rotation scan (the GivensMinGRU and
// RotationMinGRU recurrence) forward and backward, fp32 / bf16 / fp16
// storage, fp32 math.
//
// Reference behaviour: triton_scans.py:1038-1291 (`_angle_scan_fwd_kernel`,
// `_angle_scan_bwd_kernel`, op angle_scan_fwd / angle_scan_bwd at
// triton_scans.py:1579-1704, entry angle_scan_impl triton_scans.py:1743-1812).
// Per (b, block) lane with state v (k-vector), step t:
//   [v[1] *= scale_t]                                  (has_scale; rotation, k = 2)
//   R rounds: v'[p] = cos(a) v[p] + sgn[r,p] sin(a) v[perm[r,p]],
//             a = theta[b,t,blk,r,p2p[r,p]]
//   [v *= gamma_t]                                     (has_decay)
//   v += b_t;  h_t = v.
// This equals GivensMinGRU's eager M_t = gamma R_{R-1}..R_0 (min_gru.py:
// 2583-2599) and RotationMinGRU's M_t = gamma R(theta) diag(1, tanh u)
// (min_gru.py:2137-2150) applied to h_{t-1}. Backward (exact, per step):
//   gbar_t = grad_h_t + ghat_t; db_t = gbar_t; dgamma_t = <gbar_t, rot_t>;
//   rounds in reverse: dtheta(plane i,j) = a_i (-s v_i - c v_j) + a_j (c v_i - s v_j),
//   a <- R_r^T a; [dscale_t = a[1] h_{t-1}[1]; a[1] *= scale_t]; ghat_{t-1} = a.
//
// Design. One lane owns one (b, block); the state is a k-vector in registers
// and each step applies the rotations directly (never a k x k matrix). For
// chunk parallelism the aggregate of a run of steps is the affine map
// [P | q] (k x (k+1)), obtained by pushing the k+1 columns of [I | 0]
// through the same rotations; aggregates compose as [P2 P1 | P2 q1 + q2],
// the initial state enters as the element [0 | h0]. Warp aggregates compose
// in shared memory and the windowed decoupled look-back links tiles. The
// backward carries the adjoint with M_t^T through the same affine monoid,
// rebuilds h_{t-1} from the forward's chunk carries (the state at each tile
// start, k floats per lane) instead of reading the stored outputs, and
// recomputes cos/sin once per angle. The fast kernels derive the planes of
// round r from (k, r) -- the brick-wall layout both mixers build
// (min_gru.py:2544-2549, 2202-2219): planes (i, i+1 mod k) for
// i = r%2, r%2+2, ... -- and are used when the caller vouches for that
// metadata; any other metadata, k or R runs a sequential per-lane kernel
// that reads perm/sgn/p2p (backward from the stored outputs, like the
// reference).
#include "common.cuh"

namespace mgs {
namespace angle {

constexpr int kMaxK = 64, kMaxR = 16;  // sequential-kernel limits

template <typename E>
struct Args {
  const E* theta;   // (B, T, n, R, K/2)
  const E* scale;   // (B, T, n)
  const E* gamma;   // (B, T, n)
  const E* b;       // (B, T, n, K)
  const E* h0;      // (B, n, K)
  const int* perm;  // (R, K)  (sequential kernels only)
  const float* sgn; // (R, K)
  const int* p2p;   // (R, K)
  E* out;           // (B, T, n, K)   forward output / stored states for the sequential backward
  const E* gout;    // (B, T, n, K)
  E* dtheta;
  E* dscale;
  E* dgamma;
  E* db;
  E* dh0;
  float* carries;   // (tiles, K, 32) state at each tile start
  long long T_, n, sper, nstrips, nchunks, ntiles;
  int R, K, has_scale, has_decay;
  Lookback lb;
};

// Affine monoid on k x (k+1) maps x -> P x + q, stored row-major [P | q].
template <int K>
struct AffMonoid {
  static constexpr int W = K + 1;
  static constexpr int NF = K * W;
  __device__ static void identity(float (&x)[NF]) {
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < W; ++j) x[i * W + j] = (i == j) ? 1.f : 0.f;
  }
  // earlier e then later l: [Pl Pe | Pl qe + ql]; column by column, so o may alias e.
  __device__ static void combine(const float (&e)[NF], const float (&l)[NF], float (&o)[NF]) {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      float col[K];
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float s = j == K ? l[i * W + K] : 0.f;
#pragma unroll
        for (int q = 0; q < K; ++q) s = fmaf(l[i * W + q], e[q * W + j], s);
        col[i] = s;
      }
#pragma unroll
      for (int i = 0; i < K; ++i) o[i * W + j] = col[i];
    }
  }
};

// acc <- acc then later (the monoids' combine may write over its earlier operand).
template <class M, int NF>
__device__ __forceinline__ void combine_into(float (&acc)[NF], const float (&later)[NF]) {
  M::combine(acc, later, acc);
}

// Per-step coefficients of one lane: cos/sin of its R*K/2 angles, gamma, scale.
template <int K, int R>
struct StepCoef {
  float c[R * (K / 2)], s[R * (K / 2)];
  float gamma, scale;
};

template <typename E, int K, int R>
__device__ __forceinline__ void load_coef(const Args<E>& p, size_t st, StepCoef<K, R>& cf) {
  constexpr int NA = R * (K / 2);
  float th[NA];
  const E* tp = p.theta + st * NA;
#pragma unroll
  for (int i = 0; i < NA; ++i) th[i] = to_f32<E>(__ldcs(tp + i));
#pragma unroll
  for (int i = 0; i < NA; ++i) sincosf(th[i], &cf.s[i], &cf.c[i]);
  cf.gamma = p.has_decay ? to_f32<E>(__ldcs(p.gamma + st)) : 1.f;
  cf.scale = p.has_scale ? to_f32<E>(__ldcs(p.scale + st)) : 1.f;
}

// Plane m of round r: (i, j) = ((r%2 + 2m) % K, (i + 1) % K).
template <int K>
__device__ __forceinline__ void rotate(float (&v)[K], const float* c, const float* s, int r) {
  const int st = r & 1;
#pragma unroll
  for (int m = 0; m < K / 2; ++m) {
    // both parities unrolled; the branch is uniform
    const int i = st ? ((1 + 2 * m) % K) : (2 * m);
    const int j = (i + 1) % K;
    const float vi = v[i], vj = v[j];
    v[i] = fmaf(c[m], vi, -s[m] * vj);
    v[j] = fmaf(s[m], vi, c[m] * vj);
  }
}

template <int K>
__device__ __forceinline__ void rotate_t(float (&a)[K], const float* c, const float* s, int r) {
  const int st = r & 1;
#pragma unroll
  for (int m = 0; m < K / 2; ++m) {
    const int i = st ? ((1 + 2 * m) % K) : (2 * m);
    const int j = (i + 1) % K;
    const float ai = a[i], aj = a[j];
    a[i] = fmaf(c[m], ai, s[m] * aj);
    a[j] = fmaf(-s[m], ai, c[m] * aj);
  }
}

// v <- M v  (scale, rounds, decay; no injection)
template <int K, int R>
__device__ __forceinline__ void apply_M(float (&v)[K], const StepCoef<K, R>& cf, bool hs, bool hd) {
  if (hs) v[1] *= cf.scale;
#pragma unroll
  for (int r = 0; r < R; ++r) rotate<K>(v, cf.c + r * (K / 2), cf.s + r * (K / 2), r);
  if (hd)
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] *= cf.gamma;
}

// a <- M^T a
template <int K, int R>
__device__ __forceinline__ void apply_Mt(float (&a)[K], const StepCoef<K, R>& cf, bool hs, bool hd) {
  if (hd)
#pragma unroll
    for (int i = 0; i < K; ++i) a[i] *= cf.gamma;
#pragma unroll
  for (int r = R - 1; r >= 0; --r) rotate_t<K>(a, cf.c + r * (K / 2), cf.s + r * (K / 2), r);
  if (hs) a[1] *= cf.scale;
}

// X <- M X + [0 | bvec] on all K+1 columns of the aggregate. Without a scale
// M = gamma R (R a product of rotations), so the P columns can take R alone
// (pd = false) and the caller multiplies them by the product of the gammas
// once per tile: the decay then costs K multiplies per step instead of K^2 + K.
template <int K, int R>
__device__ __forceinline__ void agg_step(float (&X)[K * (K + 1)], const StepCoef<K, R>& cf,
                                         const float (&bv)[K], bool hs, bool hd, bool pd) {
#pragma unroll
  for (int j = 0; j <= K; ++j) {
    float col[K];
#pragma unroll
    for (int i = 0; i < K; ++i) col[i] = X[i * (K + 1) + j];
    apply_M<K, R>(col, cf, hs, j == K ? hd : pd);
#pragma unroll
    for (int i = 0; i < K; ++i) X[i * (K + 1) + j] = col[i] + (j == K ? bv[i] : 0.f);
  }
}

// Reverse aggregate step: Q <- M^T (g + Q), P <- M^T P (columns 0..K-1 = P,
// K = Q); pd as in agg_step.
template <int K, int R>
__device__ __forceinline__ void ragg_step(float (&X)[K * (K + 1)], const StepCoef<K, R>& cf,
                                          const float (&g)[K], bool hs, bool hd, bool pd) {
#pragma unroll
  for (int j = 0; j <= K; ++j) {
    float col[K];
#pragma unroll
    for (int i = 0; i < K; ++i) col[i] = X[i * (K + 1) + j] + (j == K ? g[i] : 0.f);
    apply_Mt<K, R>(col, cf, hs, j == K ? hd : pd);
#pragma unroll
    for (int i = 0; i < K; ++i) X[i * (K + 1) + j] = col[i];
  }
}

template <int K>
__device__ __forceinline__ void fold_state(float (&X)[K * (K + 1)], const float (&h)[K]) {
#pragma unroll
  for (int i = 0; i < K; ++i) {
#pragma unroll
    for (int j = 0; j < K; ++j) X[i * (K + 1) + j] = 0.f;
    X[i * (K + 1) + K] = h[i];
  }
}

template <typename E, int K>
__device__ __forceinline__ void load_k(const E* src, float (&o)[K]) {
#pragma unroll
  for (int i = 0; i < K; ++i) o[i] = to_f32<E>(__ldcs(src + i));
}

template <typename E, int K>
__device__ __forceinline__ void store_k(E* dst, const float (&o)[K]) {
#pragma unroll
  for (int i = 0; i < K; ++i) __stcs(dst + i, from_f32<E>(o[i]));
}

// ----------------------------------------------------------- fast kernels --
//
// One thread owns one (b, block) lane over a time tile of L steps; a CTA is
// 128 consecutive lanes of one tile (a work item, handed out in order by an
// atomic counter: all lanes' tile 0 first). Per item:
//   1. aggregate: push the k+1 columns of [I | 0] through the tile's steps
//      (forward: M_t, backward: M_t^T with the upstream gradient injected);
//   2. publish it, then look back along the lane's own chain for the nearest
//      earlier tile whose carried vector (state, or adjoint) is published,
//      and apply the aggregates in between to it (k x (k+1) times a vector:
//      no k x k compositions); publish this tile's outgoing vector;
//   3. replay the tile from its incoming vector, writing the outputs.
// Per lane and tile the workspace holds a flag, the aggregate and the
// outgoing vector, 128 lanes interleaved so a warp's accesses coalesce.

template <int W>
struct VecWord;  // the vector type moving W bytes
template <> struct VecWord<16> { using T = uint4; };
template <> struct VecWord<8> { using T = uint2; };
template <> struct VecWord<4> { using T = unsigned; };
template <> struct VecWord<2> { using T = unsigned short; };

template <typename E, int N>
struct Vec {  // N elements of E as the widest aligned vector chunks
  static constexpr int kBytes = N * (int)sizeof(E);
  static constexpr int kW = (kBytes % 16 == 0) ? 16 : (kBytes % 8 == 0) ? 8 : (kBytes % 4 == 0) ? 4 : 2;
  static constexpr int kPer = kW / (int)sizeof(E);
  using W = typename VecWord<kW>::T;
  union U {
    W w;
    E e[kPer];
  };
  __device__ static void load(const E* src, float (&o)[N]) {
#pragma unroll
    for (int c = 0; c < N / kPer; ++c) {
      U u;
      u.w = __ldcs(reinterpret_cast<const W*>(src) + c);
#pragma unroll
      for (int i = 0; i < kPer; ++i) o[c * kPer + i] = to_f32<E>(u.e[i]);
    }
  }
  __device__ static void store(E* dst, const float (&v)[N]) {
#pragma unroll
    for (int c = 0; c < N / kPer; ++c) {
      U u;
#pragma unroll
      for (int i = 0; i < kPer; ++i) u.e[i] = from_f32<E>(v[c * kPer + i]);
      __stcs(reinterpret_cast<W*>(dst) + c, u.w);
    }
  }
};

template <typename E, int K, int R>
__device__ __forceinline__ void load_coef_v(const Args<E>& p, size_t st, StepCoef<K, R>& cf) {
  constexpr int NA = R * (K / 2);
  float th[NA];
  Vec<E, NA>::load(p.theta + st * NA, th);
#pragma unroll
  for (int i = 0; i < NA; ++i) sincosf(th[i], &cf.s[i], &cf.c[i]);
  cf.gamma = p.has_decay ? to_f32<E>(__ldcs(p.gamma + st)) : 1.f;
  cf.scale = p.has_scale ? to_f32<E>(__ldcs(p.scale + st)) : 1.f;
}

// Loaded-but-unconverted inputs of one step, so the loads of later steps can
// be issued before the current step is computed (software prefetch).
template <typename E, int N>
struct Raw {
  using V = Vec<E, N>;
  typename V::W w[N / V::kPer];
  __device__ __forceinline__ void load(const E* src) {
#pragma unroll
    for (int c = 0; c < N / V::kPer; ++c)
      w[c] = __ldcs(reinterpret_cast<const typename V::W*>(src) + c);
  }
  __device__ __forceinline__ void get(float (&o)[N]) const {
#pragma unroll
    for (int c = 0; c < N / V::kPer; ++c) {
      typename V::U u;
      u.w = w[c];
#pragma unroll
      for (int i = 0; i < V::kPer; ++i) o[c * V::kPer + i] = to_f32<E>(u.e[i]);
    }
  }
};

template <typename E, int K, int R, bool TWO>
struct StepIn {
  Raw<E, R*(K / 2)> th;
  E gam, sc;
  Raw<E, K> x;  // b (forward) or grad_h (backward)
  Raw<E, K> y;  // h_{t-1} (backward replay)
  __device__ __forceinline__ void load(const Args<E>& p, size_t st, const E* xs, const E* ys,
                                       bool hs, bool hd) {
    th.load(p.theta + st * (R * (K / 2)));
    if (hd) gam = __ldcs(p.gamma + st);
    if (hs) sc = __ldcs(p.scale + st);
    x.load(xs);
    if (TWO) y.load(ys);
  }
  __device__ __forceinline__ void coef(StepCoef<K, R>& cf, bool hs, bool hd) const {
    float a[R * (K / 2)];
    th.get(a);
#pragma unroll
    for (int i = 0; i < R * (K / 2); ++i) sincosf(a[i], &cf.s[i], &cf.c[i]);
    cf.gamma = hd ? to_f32<E>(gam) : 1.f;
    cf.scale = hs ? to_f32<E>(sc) : 1.f;
  }
};

// body(step_in, t) for t = first, first + dir, ... (n steps), with the
// inputs of the next D steps already in flight.
template <int D, class SI, class LoadF, class BodyF>
__device__ __forceinline__ void stream_steps(long long first, long long n, int dir, LoadF load,
                                             BodyF body) {
  SI ring[D];
#pragma unroll
  for (int d = 0; d < D; ++d)
    if (d < n) load(ring[d], first + dir * d);
  for (long long i = 0; i < n; ++i) {
    SI cur = ring[0];
#pragma unroll
    for (int d = 0; d + 1 < D; ++d) ring[d] = ring[d + 1];
    if (i + D < n) load(ring[D - 1], first + dir * (i + D));
    body(cur, first + dir * i);
  }
}

constexpr int kLanes = 128;  // lanes (threads) per work item

struct TileRec {  // one work item's records in the workspace
  unsigned* flag;  // [128]
  float* agg;      // [NF][128]
  float* vec;      // [K][128]
};

// Workspace: 256-byte header (counter, error word), then the flags of every
// item (zeroed per launch), then the aggregates, then the carried vectors.
template <int K>
__device__ __forceinline__ TileRec rec_of(unsigned char* ws, long long items, long long item) {
  constexpr int NF = K * (K + 1);
  unsigned char* flags = ws + 256;
  float* aggs = reinterpret_cast<float*>(flags + (size_t)items * kLanes * 4);
  float* vecs = aggs + (size_t)items * NF * kLanes;
  TileRec r;
  r.flag = reinterpret_cast<unsigned*>(flags) + (size_t)item * kLanes;
  r.agg = aggs + (size_t)item * NF * kLanes;
  r.vec = vecs + (size_t)item * K * kLanes;
  return r;
}

// Bounded wait on one lane's flag; on time-out the error words are set and
// the caller proceeds with what is there (the host raises).
__device__ __forceinline__ unsigned wait_flag(const unsigned* f, unsigned* err) {
  unsigned v = ld_acquire_u32(f);
  long long it = 0;
  while (v == 0u) {
    if (++it > kSpinLimit) {
      atomicOr(err, kErrTimeout);
      atomicOr(&g_sticky_err, kErrTimeout);
      return 2u;
    }
    __nanosleep(32);
    v = ld_acquire_u32(f);
  }
  return v;
}

// Carried vector entering `item`: walk back along the lane's chain (stride
// `G` items) to the nearest published vector, then apply the aggregates of
// the items in between, oldest first: v <- P v + q.
template <int K>
__device__ __forceinline__ void look_back(unsigned char* ws, long long items, unsigned* err,
                                          long long item, long long G, float (&v)[K]) {
  constexpr int W = K + 1;
  const int t = threadIdx.x;
  long long j = item - G;
  int nagg = 0;
  while (true) {
    const TileRec r = rec_of<K>(ws, items, j);
    const unsigned f = wait_flag(r.flag + t, err);
    if (f == 2u || j < G) {
#pragma unroll
      for (int i = 0; i < K; ++i) v[i] = f == 2u ? r.vec[i * kLanes + t] : 0.f;
      break;
    }
    ++nagg;
    j -= G;
  }
  for (int q = nagg; q >= 1; --q) {
    const TileRec r = rec_of<K>(ws, items, item - q * G);
    float o[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      float s = r.agg[(i * W + K) * kLanes + t];
#pragma unroll
      for (int c = 0; c < K; ++c) s = fmaf(r.agg[(i * W + c) * kLanes + t], v[c], s);
      o[i] = s;
    }
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] = o[i];
  }
}

template <int K>
__device__ __forceinline__ void publish_agg(const TileRec& r, const float (&X)[K * (K + 1)]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int f = 0; f < K * (K + 1); ++f) r.agg[f * kLanes + t] = X[f];
  st_release_u32(r.flag + t, 1u);
}

template <int K>
__device__ __forceinline__ void publish_vec(const TileRec& r, const float (&v)[K]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < K; ++i) r.vec[i * kLanes + t] = v[i];
  st_release_u32(r.flag + t, 2u);
}

// v_out = P v_in + q for the aggregate X = [P | q].
template <int K>
__device__ __forceinline__ void apply_agg(const float (&X)[K * (K + 1)], const float (&vi)[K],
                                          float (&vo)[K]) {
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float s = X[i * (K + 1) + K];
#pragma unroll
    for (int c = 0; c < K; ++c) s = fmaf(X[i * (K + 1) + c], vi[c], s);
    vo[i] = s;
  }
}

template <typename E, int K, int R>
__global__ void __launch_bounds__(kLanes) fwd_tile_kernel(Args<E> p) {
  constexpr int NF = K * (K + 1);
  __shared__ unsigned s_item;
  const bool hs = p.has_scale != 0, hd = p.has_decay != 0;
  if (threadIdx.x == 0) s_item = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long item = s_item;
  const long long G = p.nstrips;  // lane groups
  const long long tile = item / G, grp = item - tile * G;
  const long long lane = grp * kLanes + threadIdx.x;
  const bool ok = lane < p.sper;  // sper = B * n lanes
  if (!ok) return;                // nobody reads this lane's records
  const long long bi = lane / p.n, blk = lane - bi * p.n;
  const long long t0 = tile * p.nchunks, t1 = min(p.T_, t0 + p.nchunks);  // nchunks = L
  const size_t lane0 = (size_t)bi * p.T_ * p.n + blk;
  unsigned char* ws = reinterpret_cast<unsigned char*>(p.lb.counter);
  const long long items = p.ntiles * G;
  const TileRec me = rec_of<K>(ws, items, item);

  using SI = StepIn<E, K, R, false>;
  auto load = [&](SI& q, long long t) {
    const size_t st = lane0 + t * p.n;
    q.load(p, st, p.b + st * K, nullptr, hs, hd);
  };
  float X[NF];
  AffMonoid<K>::identity(X);
  const bool pd = hd && hs;  // decay inside the P columns only when a scale is present
  float gprod = 1.f;
  stream_steps<1, SI>(t0, t1 - t0, 1, load, [&](const SI& q, long long) {
    StepCoef<K, R> cf;
    q.coef(cf, hs, hd);
    float bv[K];
    q.x.get(bv);
    agg_step<K, R>(X, cf, bv, hs, hd, pd);
    gprod *= cf.gamma;
  });
  if (hd && !pd)
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < K; ++j) X[i * (K + 1) + j] *= gprod;
  float v[K];
  if (tile == 0) {
    Vec<E, K>::load(p.h0 + ((size_t)bi * p.n + blk) * K, v);
  } else {
    publish_agg<K>(me, X);
    look_back<K>(ws, items, p.lb.err, item, G, v);
  }
  {
    float vo[K];
    apply_agg<K>(X, v, vo);
    publish_vec<K>(me, vo);
  }
  stream_steps<2, SI>(t0, t1 - t0, 1, load, [&](const SI& q, long long t) {
    StepCoef<K, R> cf;
    q.coef(cf, hs, hd);
    float bv[K];
    q.x.get(bv);
    apply_M<K, R>(v, cf, hs, hd);
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] += bv[i];
    Vec<E, K>::store(p.out + (lane0 + t * p.n) * K, v);
  });
}

template <typename E, int K, int R>
__global__ void __launch_bounds__(kLanes) bwd_tile_kernel(Args<E> p) {
  constexpr int NF = K * (K + 1), H = K / 2;
  __shared__ unsigned s_item;
  const bool hs = p.has_scale != 0, hd = p.has_decay != 0;
  if (threadIdx.x == 0) s_item = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long item = s_item;
  const long long G = p.nstrips;
  const long long rtile = item / G, grp = item - rtile * G;
  const long long tile = p.ntiles - 1 - rtile;  // ntiles = tiles per lane here
  const long long lane = grp * kLanes + threadIdx.x;
  if (lane >= p.sper) return;
  const long long bi = lane / p.n, blk = lane - bi * p.n;
  const long long t0 = tile * p.nchunks, t1 = min(p.T_, t0 + p.nchunks);
  const size_t lane0 = (size_t)bi * p.T_ * p.n + blk;
  const size_t h0off = ((size_t)bi * p.n + blk) * K;
  unsigned char* ws = reinterpret_cast<unsigned char*>(p.lb.counter);
  const long long items = p.ntiles * G;
  const TileRec me = rec_of<K>(ws, items, item);

  using SA = StepIn<E, K, R, false>;
  auto load_a = [&](SA& q, long long t) {
    const size_t st = lane0 + t * p.n;
    q.load(p, st, p.gout + st * K, nullptr, hs, hd);
  };
  float X[NF];
  AffMonoid<K>::identity(X);
  const bool pd = hd && hs;  // decay inside the P columns only when a scale is present
  float gprod = 1.f;
  stream_steps<1, SA>(t1 - 1, t1 - t0, -1, load_a, [&](const SA& q, long long) {
    StepCoef<K, R> cf;
    q.coef(cf, hs, hd);
    float g[K];
    q.x.get(g);
    ragg_step<K, R>(X, cf, g, hs, hd, pd);
    gprod *= cf.gamma;
  });
  if (hd && !pd)
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < K; ++j) X[i * (K + 1) + j] *= gprod;
  float y[K];
  if (rtile == 0) {
#pragma unroll
    for (int i = 0; i < K; ++i) y[i] = 0.f;
  } else {
    publish_agg<K>(me, X);
    look_back<K>(ws, items, p.lb.err, item, G, y);
  }
  {
    float yo[K];
    apply_agg<K>(X, y, yo);
    publish_vec<K>(me, yo);
  }
  using SB = StepIn<E, K, R, true>;
  auto load_b = [&](SB& q, long long t) {
    const size_t st = lane0 + t * p.n;
    q.load(p, st, p.gout + st * K, t > 0 ? p.out + (st - p.n) * K : p.h0 + h0off, hs, hd);
  };
  stream_steps<2, SB>(t1 - 1, t1 - t0, -1, load_b, [&](const SB& q, long long t) {
    const size_t st = lane0 + t * p.n;
    StepCoef<K, R> cf;
    q.coef(cf, hs, hd);
    float a[K], hp[K];
    q.x.get(a);
    q.y.get(hp);
#pragma unroll
    for (int i = 0; i < K; ++i) a[i] += y[i];
    Vec<E, K>::store(p.db + st * K, a);
    // state entering each round
    float vv[R + 1][K];
#pragma unroll
    for (int i = 0; i < K; ++i) vv[0][i] = hp[i];
    if (hs) vv[0][1] *= cf.scale;
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int i = 0; i < K; ++i) vv[r + 1][i] = vv[r][i];
      rotate<K>(vv[r + 1], cf.c + r * H, cf.s + r * H, r);
    }
    if (hd) {
      float dg = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) dg = fmaf(a[i], vv[R][i], dg);
      p.dgamma[st] = from_f32<E>(dg);
#pragma unroll
      for (int i = 0; i < K; ++i) a[i] *= cf.gamma;
    }
    float dth[R * H];
#pragma unroll
    for (int r = R - 1; r >= 0; --r) {
      const int par = r & 1;
#pragma unroll
      for (int m = 0; m < H; ++m) {
        const int i = par ? ((1 + 2 * m) % K) : (2 * m);
        const int j = (i + 1) % K;
        const float c = cf.c[r * H + m], sn = cf.s[r * H + m];
        const float vi = vv[r][i], vj = vv[r][j];
        dth[r * H + m] = a[i] * (-sn * vi - c * vj) + a[j] * (c * vi - sn * vj);
      }
      rotate_t<K>(a, cf.c + r * H, cf.s + r * H, r);
    }
    Vec<E, R * H>::store(p.dtheta + st * (R * H), dth);
    if (hs) {
      p.dscale[st] = from_f32<E>(a[1] * hp[1]);
      a[1] *= cf.scale;
    }
#pragma unroll
    for (int i = 0; i < K; ++i) y[i] = a[i];
  });
  if (t0 == 0) Vec<E, K>::store(p.dh0 + h0off, y);
}

// ---------------------------------------------------- sequential kernels --
// One thread per (b, block), any k <= 64, R <= 16 and any plane metadata.

template <typename E>
__global__ void seq_fwd_kernel(Args<E> p) {
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= p.sper) return;  // sper = B * n lanes here
  const int K = p.K, R = p.R, H = K / 2;
  const long long bi = id / p.n, blk = id - bi * p.n;
  float v[kMaxK], w[kMaxK];
  for (int i = 0; i < K; ++i) v[i] = to_f32<E>(p.h0[((size_t)bi * p.n + blk) * K + i]);
  for (long long t = 0; t < p.T_; ++t) {
    const size_t st = ((size_t)bi * p.T_ + t) * p.n + blk;
    if (p.has_scale) v[1] *= to_f32<E>(p.scale[st]);
    for (int r = 0; r < R; ++r) {
      for (int q = 0; q < K; ++q) {
        float sn, c;
        sincosf(to_f32<E>(p.theta[(st * R + r) * H + p.p2p[r * K + q]]), &sn, &c);
        w[q] = c * v[q] + p.sgn[r * K + q] * sn * v[p.perm[r * K + q]];
      }
      for (int q = 0; q < K; ++q) v[q] = w[q];
    }
    const float g = p.has_decay ? to_f32<E>(p.gamma[st]) : 1.f;
    for (int q = 0; q < K; ++q) {
      v[q] = v[q] * g + to_f32<E>(p.b[st * K + q]);
      p.out[st * K + q] = from_f32<E>(v[q]);
    }
  }
}

template <typename E>
__global__ void seq_bwd_kernel(Args<E> p) {
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= p.sper) return;
  const int K = p.K, R = p.R, H = K / 2;
  const long long bi = id / p.n, blk = id - bi * p.n;
  float gh[kMaxK], a[kMaxK], tmp[kMaxK];
  float vv[kMaxR + 1][kMaxK];
  for (int i = 0; i < K; ++i) gh[i] = 0.f;
  for (long long t = p.T_ - 1; t >= 0; --t) {
    const size_t st = ((size_t)bi * p.T_ + t) * p.n + blk;
    const E* hp = t > 0 ? p.out + (st - p.n) * K : p.h0 + ((size_t)bi * p.n + blk) * K;
    const float d = p.has_scale ? to_f32<E>(p.scale[st]) : 1.f;
    for (int i = 0; i < K; ++i) vv[0][i] = to_f32<E>(hp[i]);
    if (p.has_scale) vv[0][1] *= d;
    for (int r = 0; r < R; ++r)
      for (int q = 0; q < K; ++q) {
        float sn, c;
        sincosf(to_f32<E>(p.theta[(st * R + r) * H + p.p2p[r * K + q]]), &sn, &c);
        vv[r + 1][q] = c * vv[r][q] + p.sgn[r * K + q] * sn * vv[r][p.perm[r * K + q]];
      }
    for (int i = 0; i < K; ++i) {
      a[i] = to_f32<E>(p.gout[st * K + i]) + gh[i];
      p.db[st * K + i] = from_f32<E>(a[i]);
    }
    if (p.has_decay) {
      float s = 0.f;
      for (int i = 0; i < K; ++i) s += a[i] * vv[R][i];
      p.dgamma[st] = from_f32<E>(s);
      const float g = to_f32<E>(p.gamma[st]);
      for (int i = 0; i < K; ++i) a[i] *= g;
    }
    for (int r = R - 1; r >= 0; --r) {
      for (int m = 0; m < H; ++m) tmp[m] = 0.f;
      for (int q = 0; q < K; ++q) {
        float sn, c;
        sincosf(to_f32<E>(p.theta[(st * R + r) * H + p.p2p[r * K + q]]), &sn, &c);
        tmp[p.p2p[r * K + q]] +=
            a[q] * (-sn * vv[r][q] + p.sgn[r * K + q] * c * vv[r][p.perm[r * K + q]]);
      }
      for (int m = 0; m < H; ++m) p.dtheta[(st * R + r) * H + m] = from_f32<E>(tmp[m]);
      float na[kMaxK];
      for (int q = 0; q < K; ++q) {
        float sn, c;
        sincosf(to_f32<E>(p.theta[(st * R + r) * H + p.p2p[r * K + q]]), &sn, &c);
        na[q] = c * a[q];
      }
      for (int q = 0; q < K; ++q) {
        float sn, c;
        sincosf(to_f32<E>(p.theta[(st * R + r) * H + p.p2p[r * K + q]]), &sn, &c);
        na[p.perm[r * K + q]] += p.sgn[r * K + q] * sn * a[q];
      }
      for (int q = 0; q < K; ++q) a[q] = na[q];
    }
    if (p.has_scale) {
      p.dscale[st] = from_f32<E>(a[1] * to_f32<E>(hp[1]));
      a[1] *= d;
    }
    for (int i = 0; i < K; ++i) gh[i] = a[i];
  }
  for (int i = 0; i < K; ++i) p.dh0[((size_t)bi * p.n + blk) * K + i] = from_f32<E>(gh[i]);
}

// ---------------------------------------------------------------- launch --

struct Geometry {
  bool fast;
  int nf;
  long long G, L, ntiles, items;  // fast path: lane groups, steps per tile, tiles per lane
};

template <class F>
inline bool with_kr(int k, int R, F&& f) {
#define MGS_KR(KK, RR) \
  if (k == KK && R == RR) { f.template operator()<KK, RR>(); return true; }
#define MGS_KROW(KK) MGS_KR(KK, 1) MGS_KR(KK, 2) MGS_KR(KK, 3) MGS_KR(KK, 4)
  MGS_KROW(2) MGS_KROW(4) MGS_KROW(8)
#undef MGS_KROW
#undef MGS_KR
  return false;
}

// Steps per tile: long enough to amortise the per-tile aggregate and records,
// short enough to leave several work items per SM.
inline long long tile_steps(long long lanes, long long T) {
  const long long G = (lanes + kLanes - 1) / kLanes;
  long long L = 64;
  while (L > 8 && G * ((T + L - 1) / L) < 4LL * 148) L >>= 1;
  return L;
}

inline bool geometry(long long B, long long T, long long n, int R, int k, int brickwall,
                     Geometry* g) {
  if (k < 2 || k % 2 != 0 || k > kMaxK || R < 1 || R > kMaxR) return false;
  g->fast = false;
  if (brickwall) with_kr(k, R, [&]<int K, int RR>() { g->fast = true; g->nf = K * (K + 1); });
  if (!g->fast) {
    g->nf = 0;
    g->G = g->L = g->ntiles = g->items = 0;
    return true;
  }
  const long long lanes = B * n;
  g->G = (lanes + kLanes - 1) / kLanes;
  g->L = tile_steps(lanes, T);
  g->ntiles = (T + g->L - 1) / g->L;
  g->items = g->G * g->ntiles;
  return true;
}

template <typename E, int K, int R>
int launch_fast(bool fwd, Args<E>& p, const Geometry& g, void* ws, cudaStream_t st) {
  MGS_CUDA_OK(cudaMemsetAsync(ws, 0, 256 + (size_t)g.items * kLanes * 4, st));
  p.lb.counter = static_cast<unsigned*>(ws);
  p.lb.err = static_cast<unsigned*>(ws) + 1;
  p.nstrips = g.G;
  p.nchunks = g.L;
  p.ntiles = g.ntiles;
  if (fwd)
    fwd_tile_kernel<E, K, R><<<(unsigned)g.items, kLanes, 0, st>>>(p);
  else
    bwd_tile_kernel<E, K, R><<<(unsigned)g.items, kLanes, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

inline size_t workspace_bytes(const Geometry& g, int k) {
  return g.fast ? 256 + (size_t)g.items * kLanes * 4 * (1 + g.nf + k) : 256;
}

// The fast backward reads the forward's stored states: no carries.
inline size_t carry_bytes(const Geometry&, int) { return 0; }

template <typename E>
int run(bool fwd, const Args<E>& a0, long long B, long long T, long long n, int R, int k,
        int brickwall, void* ws, size_t ws_bytes, cudaStream_t st) {
  Geometry g;
  if (!geometry(B, T, n, R, k, brickwall, &g)) return MGS_UNSUPPORTED;
  Args<E> p = a0;
  p.T_ = T;
  p.n = n;
  p.R = R;
  p.K = k;
  if (B * n == 0) return MGS_OK;
  if (T == 0) {
    if (!fwd) {  // dh0 = 0 (no step reads h0's gradient path)
      MGS_CUDA_OK(cudaMemsetAsync(p.dh0, 0, (size_t)(B * n * k) * sizeof(E), st));
    }
    return MGS_OK;
  }
  if (ws == nullptr || ws_bytes < workspace_bytes(g, k) || !aligned(ws, 256))
    return MGS_WORKSPACE_TOO_SMALL;
  if (g.fast) {
    if (g.items > 0x7fffffffLL) return MGS_UNSUPPORTED;
    if (!fwd && p.out == nullptr) return MGS_BAD_SHAPE;
    p.sper = B * n;
    int rc = MGS_UNSUPPORTED;
    with_kr(k, R, [&]<int K, int RR>() { rc = launch_fast<E, K, RR>(fwd, p, g, ws, st); });
    return rc;
  }
  if (p.perm == nullptr || p.sgn == nullptr || p.p2p == nullptr) return MGS_BAD_SHAPE;
  if (!fwd && p.out == nullptr) return MGS_BAD_SHAPE;
  p.sper = B * n;
  const unsigned threads = 64;
  const unsigned blocks = (unsigned)((B * n + threads - 1) / threads);
  if (fwd)
    seq_fwd_kernel<E><<<blocks, threads, 0, st>>>(p);
  else
    seq_bwd_kernel<E><<<blocks, threads, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

template <typename E>
int dispatch_t(bool fwd, const void* theta, const void* scale, const void* gamma, const void* b,
               const void* h0, const int* perm, const float* sgn, const int* p2p, void* out,
               const void* gout, void* dtheta, void* dscale, void* dgamma, void* db, void* dh0,
               void* carries, long long B, long long T, long long n, int R, int k, int has_scale,
               int has_decay, int brickwall, void* ws, size_t ws_bytes, cudaStream_t st) {
  Args<E> p{};
  p.theta = static_cast<const E*>(theta);
  p.scale = static_cast<const E*>(scale);
  p.gamma = static_cast<const E*>(gamma);
  p.b = static_cast<const E*>(b);
  p.h0 = static_cast<const E*>(h0);
  p.perm = perm;
  p.sgn = sgn;
  p.p2p = p2p;
  p.out = static_cast<E*>(out);
  p.gout = static_cast<const E*>(gout);
  p.dtheta = static_cast<E*>(dtheta);
  p.dscale = static_cast<E*>(dscale);
  p.dgamma = static_cast<E*>(dgamma);
  p.db = static_cast<E*>(db);
  p.dh0 = static_cast<E*>(dh0);
  p.carries = static_cast<float*>(carries);
  p.has_scale = has_scale ? 1 : 0;
  p.has_decay = has_decay ? 1 : 0;
  return run<E>(fwd, p, B, T, n, R, k, brickwall, ws, ws_bytes, st);
}

int dispatch(bool fwd, const void* theta, const void* scale, const void* gamma, const void* b,
             const void* h0, const int* perm, const float* sgn, const int* p2p, void* out,
             const void* gout, void* dtheta, void* dscale, void* dgamma, void* db, void* dh0,
             void* carries, long long B, long long T, long long n, int R, int k, int has_scale,
             int has_decay, int brickwall, int dtype, void* ws, size_t ws_bytes,
             cudaStream_t st) {
  if (B < 0 || T < 0 || n < 0) return MGS_BAD_SHAPE;
#define MGS_ANGLE_CALL(E)                                                                        \
  dispatch_t<E>(fwd, theta, scale, gamma, b, h0, perm, sgn, p2p, out, gout, dtheta, dscale,     \
                dgamma, db, dh0, carries, B, T, n, R, k, has_scale, has_decay, brickwall, ws,   \
                ws_bytes, st)
  switch (dtype) {
    case MGS_F32: return MGS_ANGLE_CALL(float);
    case MGS_BF16: return MGS_ANGLE_CALL(__nv_bfloat16);
    case MGS_F16: return MGS_ANGLE_CALL(__half);
    default: return MGS_BAD_DTYPE;
  }
#undef MGS_ANGLE_CALL
}

}  // namespace angle

unsigned take_error_angle(cudaStream_t s) { return take_sticky_error(s); }

}  // namespace mgs

extern "C" {

size_t mgs_angle_scan_workspace_size(int64_t B, int64_t T, int64_t n, int R, int k,
                                     int brickwall, int dtype) {
  mgs::angle::Geometry g;
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || n < 0 ||
      !mgs::angle::geometry(B, T, n, R, k, brickwall, &g))
    return 0;
  return mgs::angle::workspace_bytes(g, k);
}

size_t mgs_angle_scan_carry_size(int64_t B, int64_t T, int64_t n, int R, int k, int brickwall,
                                 int dtype) {
  mgs::angle::Geometry g;
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || n < 0 ||
      !mgs::angle::geometry(B, T, n, R, k, brickwall, &g))
    return 0;
  return mgs::angle::carry_bytes(g, k);
}

int mgs_angle_scan_fwd(const void* theta, const void* scale, const void* gamma, const void* b,
                       const void* h0, const int32_t* perm, const float* sgn, const int32_t* p2p,
                       void* h, void* carries, int64_t B, int64_t T, int64_t n, int R, int k,
                       int has_scale, int has_decay, int brickwall, int dtype, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return mgs::angle::dispatch(true, theta, scale, gamma, b, h0, perm, sgn, p2p, h, nullptr,
                              nullptr, nullptr, nullptr, nullptr, nullptr, carries, B, T, n, R, k,
                              has_scale, has_decay, brickwall, dtype, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream));
}

int mgs_angle_scan_bwd(const void* theta, const void* scale, const void* gamma, const void* b,
                       const void* h0, const int32_t* perm, const float* sgn, const int32_t* p2p,
                       const void* h, const void* grad_h, const void* carries, void* dtheta,
                       void* dscale, void* dgamma, void* db, void* dh0, int64_t B, int64_t T,
                       int64_t n, int R, int k, int has_scale, int has_decay, int brickwall,
                       int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return mgs::angle::dispatch(false, theta, scale, gamma, b, h0, perm, sgn, p2p,
                              const_cast<void*>(h), grad_h, dtheta, dscale, dgamma, db, dh0,
                              const_cast<void*>(carries), B, T, n, R, k, has_scale, has_decay,
                              brickwall, dtype, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
