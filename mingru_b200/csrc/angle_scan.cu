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
// chunk parallelism the aggregate of a tile of steps is the affine map
// [P | q] (k x (k+1)), obtained by pushing the k+1 columns of [I | 0]
// through the same rotations, and tiles are linked by a decoupled look-back
// along each lane's chain. The backward carries the adjoint with M_t^T: over
// the same tile its aggregate is [P^T | q'], so it reuses the forward's P
// (the carries) and pushes only q'; it reads h_{t-1} from the stored outputs
// and recomputes cos/sin once per angle. The fast kernels derive the planes of
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
  float* carries;   // fast kernels: (items, K*K, 128) linear part of each forward tile aggregate
  float* lin;       // where the forward's tile linear parts live (carries, or the workspace)
  long long lin_ld; // floats per work item in `lin`
  long long T_, n, sper, nstrips, nchunks, ntiles;
  int R, K, has_scale, has_decay;
  Lookback lb;
};

// Per-step coefficients of one lane: cos/sin of its R*K/2 angles, gamma, scale.
template <int K, int R>
struct StepCoef {
  float c[R * (K / 2)], s[R * (K / 2)];
  float gamma, scale;
};

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

// cos / sin of the fast kernels' angles. Method: Cody-Waite reduction by
// pi/2 (W. J. Cody and W. Waite, Software Manual for the Elementary
// Functions, 1980) with a two-part fp32 pi/2 in fused multiply-adds -- the
// first product is exact, so r = x - k pi/2 takes one rounding -- then
// near-minimax polynomials on |r| <= 1.0005 pi/4, fitted for this file by
// Lawson's iteratively reweighted least squares in fp64 and rounded to fp32:
//   sin r = r + r^3 (S1 + S2 r^2 + S3 r^4)
//   cos r = 1 + r^2 (C1 + C2 r^2 + C3 r^4 + C4 r^6)
// and the quadrant k mod 4 read from the low bits of the rounding sum
// x (2/pi) + 1.5 2^23. Two angles go through one chain of paired FP32
// instructions. Measured in an fp32 emulation over |x| <= 8192 against fp64:
// absolute error <= 1.3 2^-24 for both; larger |x|, inf and NaN take
// sincosf. About a third of the instructions of two sincosf calls.
constexpr float kTwoOverPi = 0x1.45f306p-1f, kRoundMagic = 0x1.8p23f;
constexpr float kPio2Hi = 0x1.921fb6p+0f, kPio2Lo = -0x1.777a5cp-25f;
constexpr float kSinP1 = -0x1.555546p-3f, kSinP2 = 0x1.110736p-7f, kSinP3 = -0x1.994226p-13f;
constexpr float kCosP1 = -0x1.0p-1f, kCosP2 = 0x1.55553ep-5f, kCosP3 = -0x1.6c0878p-10f,
                kCosP4 = 0x1.99327p-16f;
constexpr float kSinCosFastArg = 8192.f;

__device__ __noinline__ float2 sincos_wide(float x) {  // (sin, cos) of a large or non-finite x
  float s, c;
  sincosf(x, &s, &c);
  return make_float2(s, c);
}

// Polynomial values (s, c) at r, rotated into quadrant j mod 4.
__device__ __forceinline__ void sincos_quadrant(float s, float c, unsigned j, float& so,
                                                float& co) {
  const bool sw = (j & 1u) != 0u;
  so = __uint_as_float(__float_as_uint(sw ? c : s) ^ ((j & 2u) << 30));
  co = __uint_as_float(__float_as_uint(sw ? s : c) ^ (((j + 1u) & 2u) << 30));
}

__device__ __forceinline__ float2 dup2(float x) { return make_float2(x, x); }

__device__ __forceinline__ void sincos_pair(float xa, float xb, float& sa, float& ca, float& sb,
                                            float& cb) {
  const float2 x = make_float2(xa, xb);
  const float2 t = __ffma2_rn(x, dup2(kTwoOverPi), dup2(kRoundMagic));
  const float2 k = __fadd2_rn(t, dup2(-kRoundMagic));
  float2 r = __ffma2_rn(k, dup2(-kPio2Hi), x);
  r = __ffma2_rn(k, dup2(-kPio2Lo), r);
  const float2 r2 = __fmul2_rn(r, r);
  float2 ps = __ffma2_rn(dup2(kSinP3), r2, dup2(kSinP2));
  ps = __ffma2_rn(ps, r2, dup2(kSinP1));
  const float2 s = __ffma2_rn(__fmul2_rn(r2, r), ps, r);
  float2 pc = __ffma2_rn(dup2(kCosP4), r2, dup2(kCosP3));
  pc = __ffma2_rn(pc, r2, dup2(kCosP2));
  pc = __ffma2_rn(pc, r2, dup2(kCosP1));
  const float2 c = __ffma2_rn(r2, pc, dup2(1.f));
  sincos_quadrant(s.x, c.x, __float_as_uint(t.x), sa, ca);
  sincos_quadrant(s.y, c.y, __float_as_uint(t.y), sb, cb);
  if (!(fabsf(xa) <= kSinCosFastArg)) {
    const float2 w = sincos_wide(xa);
    sa = w.x;
    ca = w.y;
  }
  if (!(fabsf(xb) <= kSinCosFastArg)) {
    const float2 w = sincos_wide(xb);
    sb = w.x;
    cb = w.y;
  }
}

__device__ __forceinline__ void sincos_one(float x, float& so, float& co) {
  const float t = fmaf(x, kTwoOverPi, kRoundMagic);
  const float k = t - kRoundMagic;
  float r = fmaf(k, -kPio2Hi, x);
  r = fmaf(k, -kPio2Lo, r);
  const float r2 = r * r;
  const float ps = fmaf(fmaf(kSinP3, r2, kSinP2), r2, kSinP1);
  const float s = fmaf(r2 * r, ps, r);
  const float pc = fmaf(fmaf(fmaf(kCosP4, r2, kCosP3), r2, kCosP2), r2, kCosP1);
  const float c = fmaf(r2, pc, 1.f);
  sincos_quadrant(s, c, __float_as_uint(t), so, co);
  if (!(fabsf(x) <= kSinCosFastArg)) {
    const float2 w = sincos_wide(x);
    so = w.x;
    co = w.y;
  }
}

// (sin, cos) of n angles.
template <int N>
__device__ __forceinline__ void sincos_n(const float (&a)[N], float* s, float* c) {
#pragma unroll
  for (int i = 0; i + 1 < N; i += 2) sincos_pair(a[i], a[i + 1], s[i], c[i], s[i + 1], c[i + 1]);
  if (N & 1) sincos_one(a[N - 1], s[N - 1], c[N - 1]);
}

// A forward tile aggregate x -> P x + q keeps its linear part P (K x K) as
// K/2 pairs of columns, Pp[i][m] = (P[i][2m], P[i][2m+1]): one sm_100 paired
// FP32 instruction (__ffma2_rn / __fmul2_rn, per component the same rounding
// as fmaf / a product) then advances two columns, so the per-step push of the
// K columns of P issues half the instructions of a column-by-column push and
// gives the same bits.
// Plane rotations of round r on a pair of columns (rotate() on each column).
template <int K>
__device__ __forceinline__ void rotate2(float2 (&v)[K], const float* c, const float* s, int r) {
  const int st = r & 1;
#pragma unroll
  for (int m = 0; m < K / 2; ++m) {
    const int i = st ? ((1 + 2 * m) % K) : (2 * m);
    const int j = (i + 1) % K;
    const float2 C = dup2(c[m]), S = dup2(s[m]), NS = dup2(-s[m]);
    const float2 vi = v[i], vj = v[j];
    v[i] = __ffma2_rn(C, vi, __fmul2_rn(NS, vj));
    v[j] = __ffma2_rn(S, vi, __fmul2_rn(C, vj));
  }
}

template <int K>
__device__ __forceinline__ void lin_identity(float2 (&Pp)[K][K / 2]) {
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int m = 0; m < K / 2; ++m)
      Pp[i][m] = make_float2(i == 2 * m ? 1.f : 0.f, i == 2 * m + 1 ? 1.f : 0.f);
}

// P <- M P. Without a scale M = gamma R (R a product of rotations), so the P
// columns take R alone (pd = false) and the caller multiplies them by the
// product of the gammas once per tile: the decay then costs nothing per step.
template <int K, int R>
__device__ __forceinline__ void lin_step(float2 (&Pp)[K][K / 2], const StepCoef<K, R>& cf,
                                         bool hs, bool pd) {
#pragma unroll
  for (int m = 0; m < K / 2; ++m) {
    float2 col[K];
#pragma unroll
    for (int i = 0; i < K; ++i) col[i] = Pp[i][m];
    if (hs) col[1] = __fmul2_rn(col[1], dup2(cf.scale));
#pragma unroll
    for (int r = 0; r < R; ++r) rotate2<K>(col, cf.c + r * (K / 2), cf.s + r * (K / 2), r);
    if (pd)
#pragma unroll
      for (int i = 0; i < K; ++i) col[i] = __fmul2_rn(col[i], dup2(cf.gamma));
#pragma unroll
    for (int i = 0; i < K; ++i) Pp[i][m] = col[i];
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
//   1. aggregate: the forward pushes the k columns of I (in pairs, see
//      lin_step) and the column 0 through the tile's steps M_t, giving
//      x -> P x + q; the backward's aggregate over the same tile is
//      a -> P^T a + q', so it takes P from the forward (saved as the
//      carries, one K x K matrix per lane and tile) and pushes only the
//      adjoint column q' (M_t^T with the upstream gradient injected);
//   2. publish it, then look back along the lane's own chain for the nearest
//      earlier tile whose carried vector (state, or adjoint) is published,
//      and apply the aggregates in between to it (k x (k+1) times a vector:
//      no k x k compositions); publish this tile's outgoing vector;
//   3. replay the tile from its incoming vector, writing the outputs.
// Per lane and tile the workspace holds a flag, q and the outgoing vector
// (and P when no carries are kept), 128 lanes interleaved so a warp's
// accesses coalesce.

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
    sincos_n<R * (K / 2)>(a, cf.s, cf.c);
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
  float* agg;      // [NF][128]: P row-major (f = i*K + c < K*K, when kept here), then q
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

// One look-back hop's payload: the linear part L of the forward tile behind
// the item (row-major, from `lin`) and the item's published column q.
template <int K>
__device__ __forceinline__ void hop_load(const float* P, const float* agg, float (&h)[K * K + K]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int f = 0; f < K * K; ++f) h[f] = __ldcg(P + f * kLanes + t);
#pragma unroll
  for (int i = 0; i < K; ++i) h[K * K + i] = __ldcg(agg + (K * K + i) * kLanes + t);
}

// v <- L v + q with L = P (forward) or P^T (TR, backward).
template <int K, bool TR>
__device__ __forceinline__ void hop_apply(const float (&h)[K * K + K], float (&v)[K]) {
  float o[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float s = h[K * K + i];
#pragma unroll
    for (int c = 0; c < K; ++c) s = fmaf(h[TR ? c * K + i : i * K + c], v[c], s);
    o[i] = s;
  }
#pragma unroll
  for (int i = 0; i < K; ++i) v[i] = o[i];
}

// Carried vector entering `item`: walk back along the lane's chain (stride
// `G` items) to the nearest published vector, then apply the aggregates of
// the items in between, oldest first: v <- L v + q, where L is P (forward) or
// P^T (TR, backward) of the forward tile behind that item (`lin_at(j)`, row-
// major, 128 lanes interleaved) and q is the item's published column.
// The walk reads the flags of 8 predecessors per round trip (relaxed loads,
// then one acquire fence), not one flag per round trip; each hop's payload
// (72 loads) then costs about one memory latency.
template <int K, bool TR, class LinAt>
__device__ __forceinline__ void look_back(unsigned char* ws, long long items, unsigned* err,
                                          long long item, long long G, LinAt lin_at,
                                          float (&v)[K]) {
  constexpr int kBatch = 8;
  const int t = threadIdx.x;
  long long j = item - G;  // nearest predecessor not examined yet
  int nagg = 0;
  unsigned fv = 0u;        // flag of the item where the walk stops
  while (true) {
    unsigned f[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const long long jj = j - i * G;
      f[i] = jj >= 0 ? ld_relaxed_u32(rec_of<K>(ws, items, jj).flag + t) : 2u;
    }
    int i = 0;
    bool stop = false;
    for (; i < kBatch; ++i) {
      const long long jj = j - i * G;
      if (f[i] == 0u) f[i] = wait_flag(rec_of<K>(ws, items, jj).flag + t, err);
      if (f[i] == 2u || jj < G) {
        stop = true;
        fv = f[i];
        break;
      }
    }
    nagg += i;
    j -= (long long)i * G;
    if (stop) break;
  }
  asm volatile("fence.acq_rel.gpu;" ::: "memory");  // the flags read above -> their payloads
  {
    const TileRec r = rec_of<K>(ws, items, j);
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] = fv == 2u ? __ldcg(r.vec + i * kLanes + t) : 0.f;
  }
  for (long long q = nagg; q >= 1; --q) {
    float h[K * K + K];
    hop_load<K>(lin_at(item - q * G), rec_of<K>(ws, items, item - q * G).agg, h);
    hop_apply<K, TR>(h, v);
  }
}

template <int K>
__device__ __forceinline__ void store_lin(float* P, const float2 (&Pp)[K][K / 2]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int m = 0; m < K / 2; ++m) {
      P[(i * K + 2 * m) * kLanes + t] = Pp[i][m].x;
      P[(i * K + 2 * m + 1) * kLanes + t] = Pp[i][m].y;
    }
}

// The item's q column, then flag 1 (its P is already in place).
template <int K>
__device__ __forceinline__ void publish_agg(const TileRec& r, const float (&q)[K]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < K; ++i) r.agg[(K * K + i) * kLanes + t] = q[i];
  st_release_u32(r.flag + t, 1u);
}

template <int K>
__device__ __forceinline__ void publish_vec(const TileRec& r, const float (&v)[K]) {
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < K; ++i) r.vec[i * kLanes + t] = v[i];
  st_release_u32(r.flag + t, 2u);
}

template <typename E, int K, int R>
__global__ void __launch_bounds__(kLanes, 3) fwd_tile_kernel(Args<E> p) {
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
  float2 Pp[K][K / 2];
  lin_identity<K>(Pp);
  float qv[K];
#pragma unroll
  for (int i = 0; i < K; ++i) qv[i] = 0.f;
  const bool pd = hd && hs;  // decay inside the P columns only when a scale is present
  float gprod = 1.f;
  stream_steps<1, SI>(t0, t1 - t0, 1, load, [&](const SI& q, long long) {
    StepCoef<K, R> cf;
    q.coef(cf, hs, hd);
    float bv[K];
    q.x.get(bv);
    lin_step<K, R>(Pp, cf, hs, pd);
    apply_M<K, R>(qv, cf, hs, hd);
#pragma unroll
    for (int i = 0; i < K; ++i) qv[i] += bv[i];
    gprod *= cf.gamma;
  });
  if (hd && !pd)
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int m = 0; m < K / 2; ++m) Pp[i][m] = __fmul2_rn(Pp[i][m], dup2(gprod));
  float* Pme = p.lin + item * p.lin_ld;
  store_lin<K>(Pme, Pp);
  float v[K];
  if (tile == 0) {
    Vec<E, K>::load(p.h0 + ((size_t)bi * p.n + blk) * K, v);
  } else {
    publish_agg<K>(me, qv);
    look_back<K, false>(ws, items, p.lb.err, item, G,
                        [&](long long j) { return p.lin + j * p.lin_ld; }, v);
  }
  {
    // own P read back (this thread's stores), so it holds no registers during the look-back
    float vo[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      float s = qv[i];
#pragma unroll
      for (int c = 0; c < K; ++c) s = fmaf(Pme[(i * K + c) * kLanes + threadIdx.x], v[c], s);
      vo[i] = s;
    }
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
  constexpr int H = K / 2;
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
  // Adjoint column of this tile's aggregate; its linear part is P^T of the
  // forward tile (saved by the forward in `lin`).
  float qv[K];
#pragma unroll
  for (int i = 0; i < K; ++i) qv[i] = 0.f;
  stream_steps<1, SA>(t1 - 1, t1 - t0, -1, load_a, [&](const SA& q, long long) {
    StepCoef<K, R> cf;
    q.coef(cf, hs, hd);
    float g[K];
    q.x.get(g);
#pragma unroll
    for (int i = 0; i < K; ++i) qv[i] += g[i];
    apply_Mt<K, R>(qv, cf, hs, hd);
  });
  auto lin_at = [&](long long j) {  // backward item j -> the forward item of its tile
    const long long rt = j / G;
    return p.lin + ((p.ntiles - 1 - rt) * G + (j - rt * G)) * p.lin_ld;
  };
  float y[K];
  if (rtile == 0) {
#pragma unroll
    for (int i = 0; i < K; ++i) y[i] = 0.f;
  } else {
    publish_agg<K>(me, qv);
    look_back<K, true>(ws, items, p.lb.err, item, G, lin_at, y);
  }
  {
    const float* P = lin_at(item);
    const int t = threadIdx.x;
    float yo[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      float s = qv[i];
#pragma unroll
      for (int c = 0; c < K; ++c) s = fmaf(P[(c * K + i) * kLanes + t], y[c], s);
      yo[i] = s;
    }
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

inline int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Steps per tile. Work items run in waves of `slots` CTAs (three per SM,
// less a sixteenth of headroom); an item costs its two passes (2L steps) plus
// a look-back whose length grows with the tiles of one lane in flight at
// once (about 0.2 step per such tile, measured at config 4). L in [8, 128]
// minimises (waves, rounded up) x (2L + look-back), the longer L on ties.
// Config 4 (1024 lanes, T = 4096, 148 SMs): L = 79, 416 items in one wave
// (measured: 445 us per fwd + bwd against 463 us for L = 40 in two waves,
// 497 us for L = 128, 479 us for L = 32 in 2.3 waves).
inline long long tile_steps(long long lanes, long long T) {
  const long long G = (lanes + kLanes - 1) / kLanes;
  const long long slots = 3LL * sm_count(), eff = slots - slots / 16;
  long long best = 8;
  double best_cost = 1e300;
  for (long long L = 8; L <= 128; ++L) {
    const long long tiles = (T + L - 1) / L, items = G * tiles;
    const long long waves = (items + eff - 1) / eff;
    const double in_flight = (double)(items < slots ? items : slots) / (double)G;
    const double cost = (double)waves * (2.0 * (double)(L < T ? L : T) + 0.2 * in_flight);
    if (cost <= best_cost) {
      best_cost = cost;
      best = L;
    }
  }
  return best;
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
  if (p.carries != nullptr) {  // the forward keeps each tile's P for the backward
    p.lin = p.carries;
    p.lin_ld = (long long)K * K * kLanes;
  } else {  // forward without a backward to follow: P only for the look-back
    p.lin = reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + 256 +
                                     (size_t)g.items * kLanes * 4);
    p.lin_ld = (long long)K * (K + 1) * kLanes;
  }
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

// The fast kernels' carries: the linear part P (k x k) of every forward tile
// aggregate, which the backward's tile aggregates use transposed.
inline size_t carry_bytes(const Geometry& g, int k) {
  return g.fast ? (size_t)g.items * kLanes * k * k * 4 : 0;
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
  if (ws == nullptr || ws_bytes < workspace_bytes(g, k) || !aligned(ws, 256))
    return MGS_WORKSPACE_TOO_SMALL;
  if (g.fast) {
    if (g.items > 0x7fffffffLL) return MGS_UNSUPPORTED;
    if (!fwd && (p.out == nullptr || p.carries == nullptr)) return MGS_BAD_SHAPE;
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
