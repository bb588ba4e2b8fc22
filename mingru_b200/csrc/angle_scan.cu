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

template <int K>
struct Shape {
  static constexpr int NF = K * (K + 1);
  static constexpr int S = K <= 2 ? 8 : (K <= 4 ? 4 : 2);
  static constexpr int NW = 4;
  static constexpr int L = S * NW;
};

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

// X <- M X + [0 | bvec] on all K+1 columns of the aggregate.
template <int K, int R>
__device__ __forceinline__ void agg_step(float (&X)[K * (K + 1)], const StepCoef<K, R>& cf,
                                         const float (&bv)[K], bool hs, bool hd) {
#pragma unroll
  for (int j = 0; j <= K; ++j) {
    float col[K];
#pragma unroll
    for (int i = 0; i < K; ++i) col[i] = X[i * (K + 1) + j];
    apply_M<K, R>(col, cf, hs, hd);
#pragma unroll
    for (int i = 0; i < K; ++i) X[i * (K + 1) + j] = col[i] + (j == K ? bv[i] : 0.f);
  }
}

// Reverse aggregate step: Q <- M^T (g + Q), P <- M^T P (columns 0..K-1 = P, K = Q).
template <int K, int R>
__device__ __forceinline__ void ragg_step(float (&X)[K * (K + 1)], const StepCoef<K, R>& cf,
                                          const float (&g)[K], bool hs, bool hd) {
#pragma unroll
  for (int j = 0; j <= K; ++j) {
    float col[K];
#pragma unroll
    for (int i = 0; i < K; ++i) col[i] = X[i * (K + 1) + j] + (j == K ? g[i] : 0.f);
    apply_Mt<K, R>(col, cf, hs, hd);
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

template <typename E, int K, int R>
__global__ void __launch_bounds__(Shape<K>::NW * 32, 1) fwd_kernel(Args<E> p) {
  using SH = Shape<K>;
  using M = AffMonoid<K>;
  constexpr int NF = M::NF, S = SH::S, NW = SH::NW, L = SH::L;
  extern __shared__ __align__(16) float smem[];
  float(*s_agg)[NF][32] = reinterpret_cast<float(*)[NF][32]>(smem);
  float(*s_ex)[32] = reinterpret_cast<float(*)[32]>(smem + NW * NF * 32);
  float(*s_tot)[32] = reinterpret_cast<float(*)[32]>(smem + (NW + 1) * NF * 32);
  __shared__ unsigned s_tile;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool hs = p.has_scale != 0, hd = p.has_decay != 0;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long tile = s_tile;
  const long long chunk = tile / p.nstrips;
  const long long strip = tile - chunk * p.nstrips;
  const long long bi = strip / p.sper;
  const long long blk = (strip - bi * p.sper) * 32 + lane;
  const bool ok = blk < p.n;
  const long long t0 = chunk * L + (long long)warp * S;
  const size_t lane0 = (size_t)bi * p.T_ * p.n + blk;  // (b, t, blk) = lane0 + t * n

  StepCoef<K, R> cf[S];
  float bv[S][K];
  bool live[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const long long t = t0 + s;
    live[s] = ok && t < p.T_;
    if (live[s]) {
      const size_t st = lane0 + t * p.n;
      load_coef<E, K, R>(p, st, cf[s]);
      load_k<E, K>(p.b + st * K, bv[s]);
    }
  }
  float h0v[K];
  if (ok && t0 == 0) load_k<E, K>(p.h0 + ((size_t)bi * p.n + blk) * K, h0v);
  float X[NF];
  M::identity(X);
  if (ok && t0 == 0) fold_state<K>(X, h0v);
#pragma unroll
  for (int s = 0; s < S; ++s)
    if (live[s]) agg_step<K, R>(X, cf[s], bv[s], hs, hd);
#pragma unroll
  for (int f = 0; f < NF; ++f) s_agg[warp][f][lane] = X[f];
  __syncthreads();
  if (warp == 0) {
    float tot[NF], w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) tot[f] = s_agg[0][f][lane];
#pragma unroll 1
    for (int w = 1; w < NW; ++w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
      combine_into<M, NF>(tot, w_);
    }
#pragma unroll
    for (int f = 0; f < NF; ++f) s_tot[f][lane] = tot[f];
    __syncwarp();
    warp_lookback_win_smem<M, NF>(p.lb, tile, p.nstrips, chunk, s_tot, s_ex);
  }
  __syncthreads();
  {
    float w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) X[f] = s_ex[f][lane];
#pragma unroll 1
    for (int w = 0; w < warp; ++w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
      combine_into<M, NF>(X, w_);
    }
  }
  float v[K];
#pragma unroll
  for (int i = 0; i < K; ++i) v[i] = (ok && t0 == 0) ? h0v[i] : X[i * (K + 1) + K];
  if (p.carries != nullptr && warp == 0 && t0 < p.T_) {
    float* dst = p.carries + (size_t)tile * K * 32;
#pragma unroll
    for (int i = 0; i < K; ++i) __stcs(dst + i * 32 + lane, v[i]);
  }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    if (live[s]) {
      apply_M<K, R>(v, cf[s], hs, hd);
#pragma unroll
      for (int i = 0; i < K; ++i) v[i] += bv[s][i];
      store_k<E, K>(p.out + (lane0 + (t0 + s) * p.n) * K, v);
    }
  }
}

template <typename E, int K, int R>
__global__ void __launch_bounds__(Shape<K>::NW * 32, 1) bwd_kernel(Args<E> p) {
  using SH = Shape<K>;
  using M = AffMonoid<K>;
  constexpr int NF = M::NF, S = SH::S, NW = SH::NW, L = SH::L;
  constexpr int H = K / 2;
  extern __shared__ __align__(16) float smem[];
  float(*s_fagg)[NF][32] = reinterpret_cast<float(*)[NF][32]>(smem);
  float(*s_ragg)[NF][32] = reinterpret_cast<float(*)[NF][32]>(smem + NW * NF * 32);
  float(*s_rex)[32] = reinterpret_cast<float(*)[32]>(smem + 2 * NW * NF * 32);
  float(*s_fex)[32] = reinterpret_cast<float(*)[32]>(smem + 2 * NW * NF * 32 + NF * 32);
  float(*s_tot)[32] = reinterpret_cast<float(*)[32]>(smem + 2 * NW * NF * 32 + 2 * NF * 32);
  __shared__ unsigned s_tile;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool hs = p.has_scale != 0, hd = p.has_decay != 0;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long tile = s_tile;
  const long long rchunk = tile / p.nstrips;
  const long long strip = tile - rchunk * p.nstrips;
  const long long chunk = p.nchunks - 1 - rchunk;
  const long long bi = strip / p.sper;
  const long long blk = (strip - bi * p.sper) * 32 + lane;
  const bool ok = blk < p.n;
  const long long t0 = chunk * L + (long long)warp * S;
  const size_t lane0 = (size_t)bi * p.T_ * p.n + blk;

  StepCoef<K, R> cf[S];
  float bv[S][K], gv[S][K];
  bool live[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const long long t = t0 + s;
    live[s] = ok && t < p.T_;
    if (live[s]) {
      const size_t st = lane0 + t * p.n;
      load_coef<E, K, R>(p, st, cf[s]);
      load_k<E, K>(p.b + st * K, bv[s]);
      load_k<E, K>(p.gout + st * K, gv[s]);
    }
  }
  float h0v[K];
  if (ok && t0 == 0) load_k<E, K>(p.h0 + ((size_t)bi * p.n + blk) * K, h0v);
  {
    float X[NF];
    M::identity(X);
    if (ok && t0 == 0) fold_state<K>(X, h0v);
#pragma unroll
    for (int s = 0; s < S; ++s)
      if (live[s]) agg_step<K, R>(X, cf[s], bv[s], hs, hd);
#pragma unroll
    for (int f = 0; f < NF; ++f) s_fagg[warp][f][lane] = X[f];
    M::identity(X);
#pragma unroll
    for (int s = S - 1; s >= 0; --s)
      if (live[s]) ragg_step<K, R>(X, cf[s], gv[s], hs, hd);
#pragma unroll
    for (int f = 0; f < NF; ++f) s_ragg[warp][f][lane] = X[f];
  }
  __syncthreads();
  if (warp == 0) {
    float tot[NF], w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) tot[f] = s_ragg[NW - 1][f][lane];
#pragma unroll 1
    for (int w = NW - 2; w >= 0; --w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_ragg[w][f][lane];
      combine_into<M, NF>(tot, w_);
    }
#pragma unroll
    for (int f = 0; f < NF; ++f) s_tot[f][lane] = tot[f];
    __syncwarp();
    warp_lookback_win_smem<M, NF>(p.lb, tile, p.nstrips, rchunk, s_tot, s_rex);
  } else if (warp == 1) {
    const float* src = p.carries + (size_t)(chunk * p.nstrips + strip) * K * 32;
#pragma unroll
    for (int f = 0; f < NF; ++f) s_fex[f][lane] = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) s_fex[i * (K + 1) + K][lane] = __ldcs(src + i * 32 + lane);
  }
  __syncthreads();
  // forward state entering this warp's steps
  float v[K];
  {
    float X[NF], w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) X[f] = s_fex[f][lane];
#pragma unroll 1
    for (int w = 0; w < warp; ++w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_fagg[w][f][lane];
      combine_into<M, NF>(X, w_);
    }
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] = (ok && t0 == 0) ? h0v[i] : X[i * (K + 1) + K];
  }
  // adjoint entering from later steps
  float y[K];
  {
    float X[NF], w_[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f) X[f] = s_rex[f][lane];
#pragma unroll 1
    for (int w = NW - 1; w > warp; --w) {
#pragma unroll
      for (int f = 0; f < NF; ++f) w_[f] = s_ragg[w][f][lane];
      combine_into<M, NF>(X, w_);
    }
#pragma unroll
    for (int i = 0; i < K; ++i) y[i] = X[i * (K + 1) + K];
  }
  float hp[S][K];
#pragma unroll
  for (int s = 0; s < S; ++s) {
#pragma unroll
    for (int i = 0; i < K; ++i) hp[s][i] = v[i];
    if (live[s]) {
      apply_M<K, R>(v, cf[s], hs, hd);
#pragma unroll
      for (int i = 0; i < K; ++i) v[i] += bv[s][i];
    }
  }
#pragma unroll
  for (int s = S - 1; s >= 0; --s) {
    if (!live[s]) continue;
    const size_t st = lane0 + (t0 + s) * p.n;
    float a[K];
#pragma unroll
    for (int i = 0; i < K; ++i) a[i] = gv[s][i] + y[i];
    store_k<E, K>(p.db + st * K, a);
    // per-round states vv[r] (state entering round r)
    float vv[R + 1][K];
#pragma unroll
    for (int i = 0; i < K; ++i) vv[0][i] = hp[s][i];
    if (hs) vv[0][1] *= cf[s].scale;
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int i = 0; i < K; ++i) vv[r + 1][i] = vv[r][i];
      rotate<K>(vv[r + 1], cf[s].c + r * H, cf[s].s + r * H, r);
    }
    if (hd) {
      float dg = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) dg = fmaf(a[i], vv[R][i], dg);
      p.dgamma[st] = from_f32<E>(dg);
#pragma unroll
      for (int i = 0; i < K; ++i) a[i] *= cf[s].gamma;
    }
    float dth[R * H];
#pragma unroll
    for (int r = R - 1; r >= 0; --r) {
      const int par = r & 1;
#pragma unroll
      for (int m = 0; m < H; ++m) {
        const int i = par ? ((1 + 2 * m) % K) : (2 * m);
        const int j = (i + 1) % K;
        const float c = cf[s].c[r * H + m], sn = cf[s].s[r * H + m];
        const float vi = vv[r][i], vj = vv[r][j];
        dth[r * H + m] = a[i] * (-sn * vi - c * vj) + a[j] * (c * vi - sn * vj);
      }
      rotate_t<K>(a, cf[s].c + r * H, cf[s].s + r * H, r);
    }
    {
      E* dp = p.dtheta + st * (R * H);
#pragma unroll
      for (int q = 0; q < R * H; ++q) __stcs(dp + q, from_f32<E>(dth[q]));
    }
    if (hs) {
      p.dscale[st] = from_f32<E>(a[1] * hp[s][1]);
      a[1] *= cf[s].scale;
    }
#pragma unroll
    for (int i = 0; i < K; ++i) y[i] = a[i];
  }
  if (ok && t0 == 0) store_k<E, K>(p.dh0 + ((size_t)bi * p.n + blk) * K, y);
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
  int nf, L;
  long long sper, nstrips, nchunks, ntiles;
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

inline bool geometry(long long B, long long T, long long n, int R, int k, int brickwall,
                     Geometry* g) {
  if (k < 2 || k % 2 != 0 || k > kMaxK || R < 1 || R > kMaxR) return false;
  g->fast = false;
  if (brickwall)
    with_kr(k, R, [&]<int K, int RR>() {
      g->fast = true;
      g->nf = AffMonoid<K>::NF;
      g->L = Shape<K>::L;
    });
  g->sper = (n + 31) / 32;
  g->nstrips = B * g->sper;
  g->nchunks = g->fast ? (T + g->L - 1) / g->L : 0;
  g->ntiles = g->nstrips * g->nchunks;
  if (!g->fast) g->nf = 0;
  return true;
}

template <typename E, int K, int R>
int launch_fast(bool fwd, Args<E>& p, const Geometry& g, void* ws, cudaStream_t st) {
  using SH = Shape<K>;
  constexpr int NF = AffMonoid<K>::NF;
  MGS_CUDA_OK(cudaMemsetAsync(ws, 0, lookback_zero_bytes(g.ntiles), st));
  p.lb = lookback_view(ws, g.ntiles, NF);
  p.nchunks = g.nchunks;
  p.ntiles = g.ntiles;
  if (fwd) {
    const size_t smem = (size_t)(SH::NW + 2) * NF * 32 * sizeof(float);
    MGS_CUDA_OK(cudaFuncSetAttribute(fwd_kernel<E, K, R>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    fwd_kernel<E, K, R><<<(unsigned)g.ntiles, SH::NW * 32, smem, st>>>(p);
  } else {
    const size_t smem = (size_t)(2 * SH::NW + 3) * NF * 32 * sizeof(float);
    MGS_CUDA_OK(cudaFuncSetAttribute(bwd_kernel<E, K, R>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    bwd_kernel<E, K, R><<<(unsigned)g.ntiles, SH::NW * 32, smem, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

inline size_t workspace_bytes(const Geometry& g) {
  return g.fast ? lookback_bytes(g.ntiles, g.nf) : 256;
}

inline size_t carry_bytes(const Geometry& g, int k) {
  return g.fast ? (size_t)g.ntiles * k * 32 * sizeof(float) : 0;
}

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
  if (ws == nullptr || ws_bytes < workspace_bytes(g) || !aligned(ws, 256))
    return MGS_WORKSPACE_TOO_SMALL;
  if (g.fast) {
    if (g.ntiles > 0x7fffffffLL) return MGS_UNSUPPORTED;
    if (!fwd && p.carries == nullptr) return MGS_BAD_SHAPE;
    p.sper = g.sper;
    p.nstrips = g.nstrips;
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
  return mgs::angle::workspace_bytes(g);
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
