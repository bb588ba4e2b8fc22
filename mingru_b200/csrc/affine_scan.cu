// affine_scan.cu -- block affine scan H_t = A_t H_{t-1} + B_t with k x k
// transitions and k x v injections (matrix_affine_scan; matrix_scan is the
// k = 2, v = 1 case), forward and backward, fp32 / bf16 / fp16 storage, fp32
// math.
//
// Reference behaviour: min_gru.py:1584-1655 `matrix_affine_scan(A, Bm)`
// returns (Abar_t = A_t Abar_{t-1}, Bbar_t = A_t Bbar_{t-1} + B_t) with
// Abar_0 = I, Bbar_0 = 0 for A (B, T, n, k, k), Bm (B, T, n, k, v); matrix_scan
// (min_gru.py:1513-1581) is the k = 2, v = 1 case with b (B, T, n, 2). The
// Triton kernels (triton_scans.py:629-700 forward, 823-959 backward) walk T
// per (b, block); the adjoint (triton_scans.py:900-947):
//   GA_t = gA_t + A_{t+1}^T GA_{t+1},  GB_t = gB_t + A_{t+1}^T GB_{t+1},
//   dA_t = GA_t Abar_{t-1}^T + GB_t Bbar_{t-1}^T,  dB_t = GB_t.
//
// Design. The state of one (b, block) lane is X = [Abar | Bbar], a
// k x (k+v) matrix, and so is the aggregate of any run of steps (from the
// identity [I | 0]); aggregates compose as [P2 P1 | P2 Q1 + Q2]. One lane of
// a warp owns one block, so 32 consecutive blocks of a batch row form a
// strip; a tile is S steps per warp x NW warps of one strip. Each thread
// reduces its S steps in registers, warp aggregates compose through shared
// memory, warp 0 runs the windowed decoupled look-back across the strip's
// earlier tiles, and every thread replays its steps from its exact start
// state (re-reading its inputs, which are L1/L2 resident by then). The
// backward carries Y_t = A_t^T (G_t + Y_{t+1}) in reverse (its aggregate is
// (P = A^T..A^T, Q)), rebuilds X_{t-1} from the forward's chunk carries, and
// writes dA_t = G_t X_{t-1}^T, dB_t = G_t[:, k:].
// Shapes with k (k + v) > 72 floats do not fit a thread's registers; they use
// a sequential per-lane kernel (one thread per (b, block), like the
// reference) and a backward that reads the saved forward outputs.
#include "common.cuh"

namespace mgs {
namespace affine {

inline int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Tile shape per (k, v): S steps per warp, NW warps, tile length L = S * NW.
template <int K, int V>
struct Shape {
  static constexpr int NF = K * (K + V);
  static constexpr int S = NF <= 6 ? 8 : (NF <= 20 ? 4 : (NF <= 40 ? 2 : 1));
  static constexpr int NW = (NF <= 6 || NF > 40) ? 4 : 8;  // k = 8: 4 warps keep smem < 227 KB
  static constexpr int L = S * NW;
  static constexpr bool kRegister = NF <= 72;
};

template <typename E>
struct Args {
  const E* A;     // (B, T, n, k, k)
  const E* Bm;    // (B, T, n, k, v)
  E* Abar;        // (B, T, n, k, k)  forward output / backward saved output
  E* Bbar;        // (B, T, n, k, v)
  const E* gA;    // (B, T, n, k, k)
  const E* gB;    // (B, T, n, k, v)
  E* dA;
  E* dB;
  float* carries;
  long long T_, n, sper, nstrips, nchunks, ntiles;
  Lookback lb;
};

template <typename E, int N>
__device__ __forceinline__ void load_n(const E* src, float (&out)[N]) {
  constexpr int VEC = (N * sizeof(E)) % 16 == 0 ? 16 / sizeof(E)
                      : ((N * sizeof(E)) % 8 == 0 ? 8 / sizeof(E) : 1);
#pragma unroll
  for (int i = 0; i < N; i += VEC) {
    float tmp[VEC];
    load_vec<E, VEC>(src + i, tmp);
#pragma unroll
    for (int j = 0; j < VEC; ++j) out[i + j] = tmp[j];
  }
}

template <typename E, int N>
__device__ __forceinline__ void store_n(E* dst, const float (&in)[N]) {
  constexpr int VEC = (N * sizeof(E)) % 16 == 0 ? 16 / sizeof(E)
                      : ((N * sizeof(E)) % 8 == 0 ? 8 / sizeof(E) : 1);
#pragma unroll
  for (int i = 0; i < N; i += VEC) {
    float tmp[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) tmp[j] = in[i + j];
    store_vec<E, VEC>(dst + i, tmp);
  }
}

// Cached (L1-allocating) variant for the replay pass, which re-reads data the
// first pass of the same thread has just loaded.
template <typename E, int N>
__device__ __forceinline__ void reload_n(const E* src, float (&out)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = to_f32<E>(src[i]);
}

// X <- A X + [0 | B] for X k x (k+v) row-major, A k x k, B k x v.
template <int K, int V>
__device__ __forceinline__ void step_fwd(float (&X)[K * (K + V)], const float (&A)[K * K],
                                         const float (&Bv)[K * V]) {
  constexpr int W = K + V;
  float R[K * W];
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < W; ++j) {
      float s = j >= K ? Bv[i * V + (j - K)] : 0.f;
#pragma unroll
      for (int q = 0; q < K; ++q) s = fmaf(A[i * K + q], X[q * W + j], s);
      R[i * W + j] = s;
    }
#pragma unroll
  for (int i = 0; i < K * W; ++i) X[i] = R[i];
}

template <int K, int V>
struct FwdMonoid {
  static constexpr int W = K + V;
  static constexpr int NF = K * W;
  __device__ static void identity(float (&x)[NF]) {
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < W; ++j) x[i * W + j] = (i == j) ? 1.f : 0.f;
  }
  // earlier e then later l: [Pl Pe | Pl Qe + Ql]; column by column, so o may alias e.
  __device__ static void combine(const float (&e)[NF], const float (&l)[NF], float (&o)[NF]) {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      float col[K];
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float s = j >= K ? l[i * W + j] : 0.f;
#pragma unroll
        for (int q = 0; q < K; ++q) s = fmaf(l[i * W + q], e[q * W + j], s);
        col[i] = s;
      }
#pragma unroll
      for (int i = 0; i < K; ++i) o[i * W + j] = col[i];
    }
  }
};

// Reverse adjoint aggregate: Y_out = P Y_in + Q with P k x k, Q k x (k+v);
// x = [P (k*k) | Q (k*W)].
template <int K, int V>
struct RevMonoid {
  static constexpr int W = K + V;
  static constexpr int NF = K * K + K * W;
  __device__ static void identity(float (&x)[NF]) {
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < K; ++j) x[i * K + j] = (i == j) ? 1.f : 0.f;
#pragma unroll
    for (int i = 0; i < K * W; ++i) x[K * K + i] = 0.f;
  }
  // earlier e then later l: (Pl Pe, Pl Qe + Ql); column by column, so o may alias e.
  __device__ static void combine(const float (&e)[NF], const float (&l)[NF], float (&o)[NF]) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float col[K];
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < K; ++q) s = fmaf(l[i * K + q], e[q * K + j], s);
        col[i] = s;
      }
#pragma unroll
      for (int i = 0; i < K; ++i) o[i * K + j] = col[i];
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
      float col[K];
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float s = l[K * K + i * W + j];
#pragma unroll
        for (int q = 0; q < K; ++q) s = fmaf(l[i * K + q], e[K * K + q * W + j], s);
        col[i] = s;
      }
#pragma unroll
      for (int i = 0; i < K; ++i) o[K * K + i * W + j] = col[i];
    }
  }
};

// acc <- acc then later (the monoids' combine may write over its earlier operand).
template <class M, int NF>
__device__ __forceinline__ void combine_into(float (&acc)[NF], const float (&later)[NF]) {
  M::combine(acc, later, acc);
}

// Reverse step on the adjoint aggregate: Q <- A^T (g + Q), P <- A^T P.
template <int K, int V>
__device__ __forceinline__ void step_rev(float (&x)[K * K + K * (K + V)], const float (&A)[K * K],
                                         const float (&g)[K * (K + V)]) {
  constexpr int W = K + V;
  float R[K * K + K * W];
#pragma unroll
  for (int p = 0; p < K; ++p) {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) s = fmaf(A[i * K + p], x[i * K + j], s);
      R[p * K + j] = s;
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) s = fmaf(A[i * K + p], g[i * W + j] + x[K * K + i * W + j], s);
      R[K * K + p * W + j] = s;
    }
  }
#pragma unroll
  for (int i = 0; i < K * K + K * W; ++i) x[i] = R[i];
}

template <typename E, int K, int V>
__device__ __forceinline__ void load_step(const Args<E>& p, size_t off, float (&A)[K * K],
                                          float (&Bv)[K * V], bool cached) {
  if (cached) {
    reload_n<E, K * K>(p.A + off * K * K, A);
    reload_n<E, K * V>(p.Bm + off * K * V, Bv);
  } else {
    load_n<E, K * K>(p.A + off * K * K, A);
    load_n<E, K * V>(p.Bm + off * K * V, Bv);
  }
}

// ------------------------------------------------------ register kernels --

template <typename E, int K, int V>
__global__ void __launch_bounds__(Shape<K, V>::NW * 32, 1) fwd_kernel(Args<E> p) {
  using SH = Shape<K, V>;
  using M = FwdMonoid<K, V>;
  constexpr int NF = M::NF, S = SH::S, NW = SH::NW, L = SH::L;
  extern __shared__ __align__(16) float smem[];
  float(*s_agg)[NF][32] = reinterpret_cast<float(*)[NF][32]>(smem);  // [NW][NF][32]
  float(*s_ex)[32] = reinterpret_cast<float(*)[32]>(smem + NW * NF * 32);
  __shared__ unsigned s_tile;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.lb.counter, 1u);
  __syncthreads();
  const long long tile = s_tile;
  const long long chunk = tile / p.nstrips;
  const long long strip = tile - chunk * p.nstrips;
  const long long bi = strip / p.sper;
  const long long blk = (strip - bi * p.sper) * 32 + lane;
  const bool ok = blk < p.n;
  const long long t0 = chunk * L + (long long)warp * S;
  const size_t lane0 = (size_t)bi * p.T_ * p.n + blk;  // step t of this lane: lane0 + t*n

  float X[NF];
  M::identity(X);
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    const long long t = t0 + s;
    if (ok && t < p.T_) {
      float A[K * K], Bv[K * V];
      load_step<E, K, V>(p, lane0 + t * p.n, A, Bv, false);
      step_fwd<K, V>(X, A, Bv);
    }
  }
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
    float ex[NF];
    warp_lookback_win<M, NF>(p.lb, tile, p.nstrips, chunk, tot, ex);
#pragma unroll
    for (int f = 0; f < NF; ++f) s_ex[f][lane] = ex[f];
    if (p.carries != nullptr) {
      float* dst = p.carries + (size_t)tile * NF * 32;
#pragma unroll
      for (int f = 0; f < NF; ++f) __stcs(dst + f * 32 + lane, ex[f]);
    }
  }
  __syncthreads();
  float w_[NF];
#pragma unroll
  for (int f = 0; f < NF; ++f) X[f] = s_ex[f][lane];
#pragma unroll 1
  for (int w = 0; w < warp; ++w) {
#pragma unroll
    for (int f = 0; f < NF; ++f) w_[f] = s_agg[w][f][lane];
    combine_into<M, NF>(X, w_);
  }
#pragma unroll 1
  for (int s = 0; s < S; ++s) {
    const long long t = t0 + s;
    if (ok && t < p.T_) {
      const size_t off = lane0 + t * p.n;
      float A[K * K], Bv[K * V];
      load_step<E, K, V>(p, off, A, Bv, true);
      step_fwd<K, V>(X, A, Bv);
      float oa[K * K], ob[K * V];
#pragma unroll
      for (int i = 0; i < K; ++i) {
#pragma unroll
        for (int j = 0; j < K; ++j) oa[i * K + j] = X[i * (K + V) + j];
#pragma unroll
        for (int j = 0; j < V; ++j) ob[i * V + j] = X[i * (K + V) + K + j];
      }
      store_n<E, K * K>(p.Abar + off * K * K, oa);
      store_n<E, K * V>(p.Bbar + off * K * V, ob);
    }
  }
}

template <typename E, int K, int V>
__global__ void __launch_bounds__(Shape<K, V>::NW * 32, 1) bwd_kernel(Args<E> p) {
  using SH = Shape<K, V>;
  using FM = FwdMonoid<K, V>;
  using RM = RevMonoid<K, V>;
  constexpr int W = K + V;
  constexpr int NFF = FM::NF, NFR = RM::NF, S = SH::S, NW = SH::NW, L = SH::L;
  extern __shared__ __align__(16) float smem[];
  float(*s_fagg)[NFF][32] = reinterpret_cast<float(*)[NFF][32]>(smem);
  float(*s_ragg)[NFR][32] = reinterpret_cast<float(*)[NFR][32]>(smem + NW * NFF * 32);
  float(*s_fex)[32] = reinterpret_cast<float(*)[32]>(smem + NW * (NFF + NFR) * 32);
  float(*s_rex)[32] = reinterpret_cast<float(*)[32]>(smem + NW * (NFF + NFR) * 32 + NFF * 32);
  __shared__ unsigned s_tile;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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

  {
    float X[NFF];
    FM::identity(X);
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
      const long long t = t0 + s;
      if (ok && t < p.T_) {
        float A[K * K], Bv[K * V];
        load_step<E, K, V>(p, lane0 + t * p.n, A, Bv, false);
        step_fwd<K, V>(X, A, Bv);
      }
    }
#pragma unroll
    for (int f = 0; f < NFF; ++f) s_fagg[warp][f][lane] = X[f];
  }
  {
    float Y[NFR];
    RM::identity(Y);
#pragma unroll 1
    for (int s = S - 1; s >= 0; --s) {
      const long long t = t0 + s;
      if (ok && t < p.T_) {
        const size_t off = lane0 + t * p.n;
        float A[K * K], g[K * W];
        reload_n<E, K * K>(p.A + off * K * K, A);
        {
          float ga[K * K], gb[K * V];
          load_n<E, K * K>(p.gA + off * K * K, ga);
          load_n<E, K * V>(p.gB + off * K * V, gb);
#pragma unroll
          for (int i = 0; i < K; ++i) {
#pragma unroll
            for (int j = 0; j < K; ++j) g[i * W + j] = ga[i * K + j];
#pragma unroll
            for (int j = 0; j < V; ++j) g[i * W + K + j] = gb[i * V + j];
          }
        }
        step_rev<K, V>(Y, A, g);
      }
    }
#pragma unroll
    for (int f = 0; f < NFR; ++f) s_ragg[warp][f][lane] = Y[f];
  }
  __syncthreads();
  if (warp == 0) {
    float tot[NFR], w_[NFR];
#pragma unroll
    for (int f = 0; f < NFR; ++f) tot[f] = s_ragg[NW - 1][f][lane];
#pragma unroll 1
    for (int w = NW - 2; w >= 0; --w) {
#pragma unroll
      for (int f = 0; f < NFR; ++f) w_[f] = s_ragg[w][f][lane];
      combine_into<RM, NFR>(tot, w_);
    }
    float ex[NFR];
    warp_lookback_win<RM, NFR>(p.lb, tile, p.nstrips, rchunk, tot, ex);
#pragma unroll
    for (int f = 0; f < NFR; ++f) s_rex[f][lane] = ex[f];
  } else if (warp == 1) {
    const float* src = p.carries + (size_t)(chunk * p.nstrips + strip) * NFF * 32;
#pragma unroll
    for (int f = 0; f < NFF; ++f) s_fex[f][lane] = __ldcs(src + f * 32 + lane);
  }
  __syncthreads();

  // Forward start state of this warp's steps.
  float Xs[S][NFF];
  {
    float X[NFF], w_[NFF];
#pragma unroll
    for (int f = 0; f < NFF; ++f) X[f] = s_fex[f][lane];
#pragma unroll 1
    for (int w = 0; w < warp; ++w) {
#pragma unroll
      for (int f = 0; f < NFF; ++f) w_[f] = s_fagg[w][f][lane];
      combine_into<FM, NFF>(X, w_);
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
#pragma unroll
      for (int f = 0; f < NFF; ++f) Xs[s][f] = X[f];
      const long long t = t0 + s;
      if (s + 1 < S && ok && t < p.T_) {
        float A[K * K], Bv[K * V];
        load_step<E, K, V>(p, lane0 + t * p.n, A, Bv, true);
        step_fwd<K, V>(X, A, Bv);
      }
    }
  }
  // Adjoint entering from later steps: Y = Q of the composed later aggregates.
  float Y[K * W];
  {
    float R[NFR], w_[NFR];
#pragma unroll
    for (int f = 0; f < NFR; ++f) R[f] = s_rex[f][lane];
#pragma unroll 1
    for (int w = NW - 1; w > warp; --w) {
#pragma unroll
      for (int f = 0; f < NFR; ++f) w_[f] = s_ragg[w][f][lane];
      combine_into<RM, NFR>(R, w_);
    }
#pragma unroll
    for (int f = 0; f < K * W; ++f) Y[f] = R[K * K + f];
  }
#pragma unroll
  for (int s = S - 1; s >= 0; --s) {
    const long long t = t0 + s;
    if (ok && t < p.T_) {
      const size_t off = lane0 + t * p.n;
      float A[K * K];
      reload_n<E, K * K>(p.A + off * K * K, A);
      {
        float ga[K * K], gb[K * V];
        reload_n<E, K * K>(p.gA + off * K * K, ga);
        reload_n<E, K * V>(p.gB + off * K * V, gb);
#pragma unroll
        for (int i = 0; i < K; ++i) {
#pragma unroll
          for (int j = 0; j < K; ++j) Y[i * W + j] += ga[i * K + j];
#pragma unroll
          for (int j = 0; j < V; ++j) Y[i * W + K + j] += gb[i * V + j];
        }
      }
      // Y now holds G_t = [GA | GB]; dA = G X_{t-1}^T, dB = G[:, K:].
      float oa[K * K], ob[K * V];
#pragma unroll
      for (int i = 0; i < K; ++i) {
#pragma unroll
        for (int q = 0; q < K; ++q) {
          float s2 = 0.f;
#pragma unroll
          for (int j = 0; j < W; ++j) s2 = fmaf(Y[i * W + j], Xs[s][q * W + j], s2);
          oa[i * K + q] = s2;
        }
#pragma unroll
        for (int j = 0; j < V; ++j) ob[i * V + j] = Y[i * W + K + j];
      }
      store_n<E, K * K>(p.dA + off * K * K, oa);
      store_n<E, K * V>(p.dB + off * K * V, ob);
      // Y <- A^T G (column by column, in place)
#pragma unroll
      for (int j = 0; j < W; ++j) {
        float col[K];
#pragma unroll
        for (int q = 0; q < K; ++q) {
          float s2 = 0.f;
#pragma unroll
          for (int i = 0; i < K; ++i) s2 = fmaf(A[i * K + q], Y[i * W + j], s2);
          col[q] = s2;
        }
#pragma unroll
        for (int q = 0; q < K; ++q) Y[q * W + j] = col[q];
      }
    }
  }
}

// ------------------------------------------------------------ strip path --
//
// Small elements (32 k^2 and 32 k v elements per time row fit one TMA box:
// k <= 2, k v <= 8 -- matrix_scan is k = 2, v = 1): persistent CTAs of
// kStripNW consumer warps + 1 producer warp, each CTA walking 32-block strips
// through all of T. The producer streams 32-step chunks of A and Bm (backward:
// also gA, gB and the chunk's forward carry) into a shared-memory ring with
// TMA; consumer warp w takes steps w*S .. w*S+S-1 (S = 4) of each chunk with its lane's
// inputs in registers, warp aggregates combine through shared memory and the
// strip state is carried on chip from chunk to chunk: no look-back, every
// input read once. The forward writes each chunk's start state (the carries);
// the backward walks the chunks in reverse, rebuilds X_{t-1} from them and
// carries the adjoint like the register kernels.

constexpr int kLc = 32;          // steps per chunk (= carry granularity of the strip path)
constexpr int kStripNW = 8;      // consumer warps
constexpr int kStripS = kLc / kStripNW;
constexpr int kMaxStages = 16;

template <int K, int V>
struct StripOK {
  static constexpr bool value = 32 * K * K <= 256 && 32 * K * V <= 256 && K * (K + V) <= 8;
};

template <typename E, int K, int V, bool BWD>
struct AStage {
  static constexpr int kA = 32 * K * K, kB = 32 * K * V;  // elements per time row
  static constexpr int NF = K * (K + V);
  static constexpr size_t kABytes = (size_t)kLc * kA * sizeof(E);
  static constexpr size_t kBBytes = (size_t)kLc * kB * sizeof(E);
  static constexpr size_t kCarryBytes = BWD ? (size_t)NF * 32 * sizeof(float) : 0;
  static constexpr size_t kBytes =
      ((BWD ? 2 : 1) * (kABytes + kBBytes) + kCarryBytes + 127) / 128 * 128;
};

struct AStripMaps {
  CUtensorMap m[4];  // A, Bm, gA, gB
};

struct StripArgs {
  long long T_, n, sper, nstrips, nchunks;
  int nstage;
  float* carries;  // (nchunks, nstrips, NF, 32) chunk-start states
  unsigned* err;
};

template <typename E, int K, int V, bool BWD>
__device__ __forceinline__ void astrip_produce(const StripArgs& a, const AStripMaps& maps,
                                               unsigned char* ring, uint64_t* full,
                                               uint64_t* empty) {
  using SS = AStage<E, K, V, BWD>;
  constexpr int NIN = BWD ? 4 : 2;
  const int lane = threadIdx.x & 31;
  if (lane == 0)
    for (int i = 0; i < NIN; ++i) tma_prefetch_desc(&maps.m[i]);
  int s = 0;
  unsigned ph = 0, pending = 0u, pend_ph = 0u;
  for (long long strip = blockIdx.x; strip < a.nstrips; strip += gridDim.x) {
    const long long bi = strip / a.sper;
    const int g0 = (int)(strip - bi * a.sper);
    for (long long q = 0; q < a.nchunks; ++q) {
      const long long chunk = BWD ? a.nchunks - 1 - q : q;
      if (!mbar_wait(&empty[s], ph ^ 1u, a.err)) goto drain;
      pending &= ~(1u << s);
      if (lane == 0) {
        unsigned char* st = ring + (size_t)s * SS::kBytes;
        mbar_arrive_expect_tx(&full[s], (unsigned)((BWD ? 2 : 1) * (SS::kABytes + SS::kBBytes) +
                                                   SS::kCarryBytes));
        const int y = (int)(chunk * kLc);
        tma_load_3d(st, &maps.m[0], g0 * SS::kA, y, (int)bi, &full[s]);
        tma_load_3d(st + SS::kABytes, &maps.m[1], g0 * SS::kB, y, (int)bi, &full[s]);
        if (BWD) {
          tma_load_3d(st + SS::kABytes + SS::kBBytes, &maps.m[2], g0 * SS::kA, y, (int)bi,
                      &full[s]);
          tma_load_3d(st + 2 * SS::kABytes + SS::kBBytes, &maps.m[3], g0 * SS::kB, y, (int)bi,
                      &full[s]);
          bulk_g2s(st + 2 * (SS::kABytes + SS::kBBytes),
                   a.carries + (size_t)(chunk * a.nstrips + strip) * SS::NF * 32,
                   (unsigned)SS::kCarryBytes, &full[s]);
        }
      }
      __syncwarp();
      pending |= 1u << s;
      pend_ph = (pend_ph & ~(1u << s)) | (ph << s);
      if (++s == a.nstage) {
        s = 0;
        ph ^= 1u;
      }
    }
  }
drain:
  for (int i = 0; i < a.nstage; ++i)
    if (pending & (1u << i)) mbar_wait(&full[i], (pend_ph >> i) & 1u, a.err);
}

// Lane `lane`'s N elements of time row `row` of a staged (rows x 32 N) block,
// read as the widest vectors their alignment allows (N is a power of two, the
// block 128-byte aligned).
template <typename E, int N>
__device__ __forceinline__ void stage_get(const unsigned char* base, int row, float (&o)[N]) {
  constexpr int kBytes = N * (int)sizeof(E) < 16 ? N * (int)sizeof(E) : 16;
  constexpr int kPer = kBytes / (int)sizeof(E);
  using Vt = typename VecOf<kBytes>::type;
  const E* p = reinterpret_cast<const E*>(base) + (size_t)row * 32 * N + (threadIdx.x & 31) * N;
#pragma unroll
  for (int c = 0; c < N / kPer; ++c) {
    const Vt w = reinterpret_cast<const Vt*>(p)[c];
    const E* e = reinterpret_cast<const E*>(&w);
#pragma unroll
    for (int i = 0; i < kPer; ++i) o[c * kPer + i] = to_f32<E>(e[i]);
  }
}

template <typename E, int K, int V>
__global__ void __launch_bounds__((kStripNW + 1) * 32, 1)
    fwd_strip_kernel(Args<E> p, StripArgs a, const __grid_constant__ AStripMaps maps) {
  using SS = AStage<E, K, V, false>;
  using M = FwdMonoid<K, V>;
  constexpr int NF = M::NF, NW = kStripNW, S = kStripS, W = K + V;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ float s_agg[2][NW][NF][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nstage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == NW) {
    astrip_produce<E, K, V, false>(a, maps, ring, full, empty);
    return;
  }
  int s = 0, buf = 0;
  unsigned ph = 0;
  for (long long strip = blockIdx.x; strip < a.nstrips; strip += gridDim.x) {
    const long long bi = strip / a.sper;
    const long long blk = (strip - bi * a.sper) * 32 + lane;
    const bool ok = blk < a.n;
    const size_t lane0 = (size_t)bi * a.T_ * a.n + blk;
    float carry[NF];
    M::identity(carry);
    for (long long chunk = 0; chunk < a.nchunks; ++chunk) {
      const bool okw = mbar_wait(&full[s], ph, a.err);
      if (bar_any(1, NW * 32, !okw)) return;
      const unsigned char* st = ring + (size_t)s * SS::kBytes;
      float Av[S][K * K], Bv[S][K * V];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        stage_get<E, K * K>(st, warp * S + i, Av[i]);
        stage_get<E, K * V>(st + SS::kABytes, warp * S + i, Bv[i]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == a.nstage) {
        s = 0;
        ph ^= 1u;
      }
      const long long t0 = chunk * kLc + (long long)warp * S;
      float agg[NF];
      M::identity(agg);
#pragma unroll
      for (int i = 0; i < S; ++i)
        if (t0 + i < a.T_) step_fwd<K, V>(agg, Av[i], Bv[i]);
#pragma unroll
      for (int f = 0; f < NF; ++f) s_agg[buf][warp][f][lane] = agg[f];
      named_bar(2, NW * 32);
      if (warp == 0 && a.carries != nullptr) {
        float* dst = a.carries + (size_t)(chunk * a.nstrips + strip) * NF * 32;
#pragma unroll
        for (int f = 0; f < NF; ++f) __stcs(dst + f * 32 + lane, carry[f]);
      }
      float X[NF];
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        float e[NF];
#pragma unroll
        for (int f = 0; f < NF; ++f) e[f] = s_agg[buf][w][f][lane];
        if (w == warp)
#pragma unroll
          for (int f = 0; f < NF; ++f) X[f] = carry[f];
        combine_into<M, NF>(carry, e);
      }
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const long long t = t0 + i;
        if (t < a.T_) {
          step_fwd<K, V>(X, Av[i], Bv[i]);
          if (ok) {
            const size_t off = lane0 + t * a.n;
            float oa[K * K], ob[K * V];
#pragma unroll
            for (int r = 0; r < K; ++r) {
#pragma unroll
              for (int c = 0; c < K; ++c) oa[r * K + c] = X[r * W + c];
#pragma unroll
              for (int c = 0; c < V; ++c) ob[r * V + c] = X[r * W + K + c];
            }
            store_n<E, K * K>(p.Abar + off * K * K, oa);
            store_n<E, K * V>(p.Bbar + off * K * V, ob);
          }
        }
      }
      buf ^= 1;
    }
  }
}

template <typename E, int K, int V>
__global__ void __launch_bounds__((kStripNW + 1) * 32, 1)
    bwd_strip_kernel(Args<E> p, StripArgs a, const __grid_constant__ AStripMaps maps) {
  using SS = AStage<E, K, V, true>;
  using FM = FwdMonoid<K, V>;
  using RM = RevMonoid<K, V>;
  constexpr int NFF = FM::NF, NFR = RM::NF, NW = kStripNW, S = kStripS, W = K + V;
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ float s_fagg[2][NW][NFF][32];
  __shared__ float s_ragg[2][NW][NFR][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.nstage; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == NW) {
    astrip_produce<E, K, V, true>(a, maps, ring, full, empty);
    return;
  }
  int s = 0, buf = 0;
  unsigned ph = 0;
  for (long long strip = blockIdx.x; strip < a.nstrips; strip += gridDim.x) {
    const long long bi = strip / a.sper;
    const long long blk = (strip - bi * a.sper) * 32 + lane;
    const bool ok = blk < a.n;
    const size_t lane0 = (size_t)bi * a.T_ * a.n + blk;
    float rcarry[NFR];
    RM::identity(rcarry);
    for (long long q = 0; q < a.nchunks; ++q) {
      const long long chunk = a.nchunks - 1 - q;
      const bool okw = mbar_wait(&full[s], ph, a.err);
      if (bar_any(1, NW * 32, !okw)) return;
      const unsigned char* st = ring + (size_t)s * SS::kBytes;
      float Av[S][K * K], Bv[S][K * V], Ga[S][K * W];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        stage_get<E, K * K>(st, warp * S + i, Av[i]);
        stage_get<E, K * V>(st + SS::kABytes, warp * S + i, Bv[i]);
        float ga[K * K], gb[K * V];
        stage_get<E, K * K>(st + SS::kABytes + SS::kBBytes, warp * S + i, ga);
        stage_get<E, K * V>(st + 2 * SS::kABytes + SS::kBBytes, warp * S + i, gb);
#pragma unroll
        for (int r = 0; r < K; ++r) {
#pragma unroll
          for (int c = 0; c < K; ++c) Ga[i][r * W + c] = ga[r * K + c];
#pragma unroll
          for (int c = 0; c < V; ++c) Ga[i][r * W + K + c] = gb[r * V + c];
        }
      }
      float fcur[NFF];
      {
        const float* fc = reinterpret_cast<const float*>(st + 2 * (SS::kABytes + SS::kBBytes));
#pragma unroll
        for (int f = 0; f < NFF; ++f) fcur[f] = fc[f * 32 + lane];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == a.nstage) {
        s = 0;
        ph ^= 1u;
      }
      const long long t0 = chunk * kLc + (long long)warp * S;
      {
        float fagg[NFF], ragg[NFR];
        FM::identity(fagg);
        RM::identity(ragg);
#pragma unroll
        for (int i = 0; i < S; ++i)
          if (t0 + i < a.T_) step_fwd<K, V>(fagg, Av[i], Bv[i]);
#pragma unroll
        for (int i = S - 1; i >= 0; --i)
          if (t0 + i < a.T_) step_rev<K, V>(ragg, Av[i], Ga[i]);
#pragma unroll
        for (int f = 0; f < NFF; ++f) s_fagg[buf][warp][f][lane] = fagg[f];
#pragma unroll
        for (int f = 0; f < NFR; ++f) s_ragg[buf][warp][f][lane] = ragg[f];
      }
      named_bar(2, NW * 32);
      for (int w = 0; w < warp; ++w) {
        float e[NFF];
#pragma unroll
        for (int f = 0; f < NFF; ++f) e[f] = s_fagg[buf][w][f][lane];
        combine_into<FM, NFF>(fcur, e);
      }
      float rcur[NFR];
#pragma unroll
      for (int w = NW - 1; w >= 0; --w) {
        if (w == warp)
#pragma unroll
          for (int f = 0; f < NFR; ++f) rcur[f] = rcarry[f];
        float e[NFR];
#pragma unroll
        for (int f = 0; f < NFR; ++f) e[f] = s_ragg[buf][w][f][lane];
        combine_into<RM, NFR>(rcarry, e);
      }
      // forward states entering each step, then the reverse sweep
      float Xs[S][NFF];
#pragma unroll
      for (int i = 0; i < S; ++i) {
#pragma unroll
        for (int f = 0; f < NFF; ++f) Xs[i][f] = fcur[f];
        if (i + 1 < S) step_fwd<K, V>(fcur, Av[i], Bv[i]);
      }
      float Y[K * W];
#pragma unroll
      for (int f = 0; f < K * W; ++f) Y[f] = rcur[K * K + f];
#pragma unroll
      for (int i = S - 1; i >= 0; --i) {
        const long long t = t0 + i;
        if (t >= a.T_) continue;
#pragma unroll
        for (int f = 0; f < K * W; ++f) Y[f] += Ga[i][f];
        if (ok) {
          const size_t off = lane0 + t * a.n;
          float oa[K * K], ob[K * V];
#pragma unroll
          for (int r = 0; r < K; ++r) {
#pragma unroll
            for (int c = 0; c < K; ++c) {
              float s2 = 0.f;
#pragma unroll
              for (int j = 0; j < W; ++j) s2 = fmaf(Y[r * W + j], Xs[i][c * W + j], s2);
              oa[r * K + c] = s2;
            }
#pragma unroll
            for (int c = 0; c < V; ++c) ob[r * V + c] = Y[r * W + K + c];
          }
          store_n<E, K * K>(p.dA + off * K * K, oa);
          store_n<E, K * V>(p.dB + off * K * V, ob);
        }
#pragma unroll
        for (int j = 0; j < W; ++j) {
          float col[K];
#pragma unroll
          for (int c = 0; c < K; ++c) {
            float s2 = 0.f;
#pragma unroll
            for (int r = 0; r < K; ++r) s2 = fmaf(Av[i][r * K + c], Y[r * W + j], s2);
            col[c] = s2;
          }
#pragma unroll
          for (int c = 0; c < K; ++c) Y[c * W + j] = col[c];
        }
      }
      buf ^= 1;
    }
  }
}

// ------------------------------------------------- sequential (large k) --

template <typename E>
__global__ void seq_fwd_kernel(Args<E> p, int K, int V, float* scratch) {
  const long long lanes = p.sper;  // here: B * n lanes
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= lanes) return;
  const int W = K + V;
  float* X = scratch + (size_t)id * 2 * K * W;  // per-lane state + temp in global scratch
  float* R = X + K * W;
  for (int i = 0; i < K; ++i)
    for (int j = 0; j < W; ++j) X[i * W + j] = (i == j) ? 1.f : 0.f;
  const long long bi = id / p.n, blk = id - bi * p.n;
  for (long long t = 0; t < p.T_; ++t) {
    const size_t off = ((size_t)bi * p.T_ + t) * p.n + blk;
    const E* A = p.A + off * K * K;
    const E* Bv = p.Bm + off * K * V;
    for (int i = 0; i < K; ++i)
      for (int j = 0; j < W; ++j) {
        float s = j >= K ? to_f32<E>(Bv[i * V + j - K]) : 0.f;
        for (int q = 0; q < K; ++q) s = fmaf(to_f32<E>(A[i * K + q]), X[q * W + j], s);
        R[i * W + j] = s;
      }
    for (int i = 0; i < K; ++i)
      for (int j = 0; j < W; ++j) {
        X[i * W + j] = R[i * W + j];
        if (j < K)
          p.Abar[off * K * K + i * K + j] = from_f32<E>(R[i * W + j]);
        else
          p.Bbar[off * K * V + i * V + j - K] = from_f32<E>(R[i * W + j]);
      }
  }
}

template <typename E>
__global__ void seq_bwd_kernel(Args<E> p, int K, int V, float* scratch) {
  const long long lanes = p.sper;
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= lanes) return;
  const int W = K + V;
  float* G = scratch + (size_t)id * 2 * K * W;
  float* R = G + K * W;
  for (int i = 0; i < K * W; ++i) G[i] = 0.f;  // holds Y_{t+1} = A_{t+1}^T G_{t+1}
  const long long bi = id / p.n, blk = id - bi * p.n;
  for (long long t = p.T_ - 1; t >= 0; --t) {
    const size_t off = ((size_t)bi * p.T_ + t) * p.n + blk;
    for (int i = 0; i < K; ++i)
      for (int j = 0; j < W; ++j)
        G[i * W + j] += j < K ? to_f32<E>(p.gA[off * K * K + i * K + j])
                              : to_f32<E>(p.gB[off * K * V + i * V + j - K]);
    // dA_t = G X_{t-1}^T with X_{t-1} from the saved outputs (I / 0 at t = 0)
    for (int i = 0; i < K; ++i) {
      for (int q = 0; q < K; ++q) {
        float s = 0.f;
        for (int j = 0; j < W; ++j) {
          float xv;
          if (t == 0)
            xv = (j == q) ? 1.f : 0.f;
          else if (j < K)
            xv = to_f32<E>(p.Abar[(off - p.n) * K * K + q * K + j]);
          else
            xv = to_f32<E>(p.Bbar[(off - p.n) * K * V + q * V + j - K]);
          s = fmaf(G[i * W + j], xv, s);
        }
        p.dA[off * K * K + i * K + q] = from_f32<E>(s);
      }
      for (int j = 0; j < V; ++j) p.dB[off * K * V + i * V + j] = from_f32<E>(G[i * W + K + j]);
    }
    for (int q = 0; q < K; ++q)
      for (int j = 0; j < W; ++j) {
        float s = 0.f;
        for (int i = 0; i < K; ++i) s = fmaf(to_f32<E>(p.A[off * K * K + i * K + q]), G[i * W + j], s);
        R[q * W + j] = s;
      }
    for (int i = 0; i < K * W; ++i) G[i] = R[i];
  }
}

// ---------------------------------------------------------------- launch --

struct Geometry {
  bool reg, strip;
  int nff, nfr, L;
  long long sper, nstrips, nchunks, ntiles;
};

template <int K, int V>
inline Geometry geometry_kv(long long B, long long T, long long n, int dtype) {
  Geometry g;
  using SH = Shape<K, V>;
  g.reg = SH::kRegister;
  // Strip-serial walk (no look-back, inputs read once) when the strips fill
  // most SMs and the TMA row strides are 16-byte multiples.
  const long long strips = B * ((n + 31) / 32);
  const size_t es = (size_t)dtype_size(dtype);
  g.strip = StripOK<K, V>::value && (n * K * K * es) % 16 == 0 && (n * K * V * es) % 16 == 0 &&
            strips * 4 >= 3LL * sm_count() && T >= 2 * kLc;
  if (g.strip) {
    g.reg = false;
    g.nff = FwdMonoid<K, V>::NF;
    g.nfr = RevMonoid<K, V>::NF;
    g.L = kLc;
    g.sper = (n + 31) / 32;
    g.nstrips = B * g.sper;
    g.nchunks = (T + kLc - 1) / kLc;
    g.ntiles = g.nstrips * g.nchunks;
    return g;
  }
  g.nff = FwdMonoid<K, V>::NF;
  g.nfr = RevMonoid<K, V>::NF;
  g.L = SH::L;
  g.sper = (n + 31) / 32;
  g.nstrips = B * g.sper;
  g.nchunks = (T + g.L - 1) / g.L;
  g.ntiles = g.nstrips * g.nchunks;
  return g;
}

// Calls f.template operator()<K, V>() for the runtime (k, v); false if out of envelope.
template <class F>
inline bool with_kv(int k, int v, F&& f) {
#define MGS_KV(KK, VV) \
  if (k == KK && v == VV) { f.template operator()<KK, VV>(); return true; }
#define MGS_KROW(KK) MGS_KV(KK, 1) MGS_KV(KK, 2) MGS_KV(KK, 4) MGS_KV(KK, 8) MGS_KV(KK, 16)
  MGS_KROW(1) MGS_KROW(2) MGS_KROW(4) MGS_KROW(8) MGS_KROW(16)
#undef MGS_KROW
#undef MGS_KV
  return false;
}

// Register kernels for the reference envelope k, v in {1, 2, 4, 8, 16} with
// k (k + v) <= 72; any other k, v >= 1 (up to 64) runs the sequential kernels.
constexpr int kMaxSeqKV = 64;

inline bool geometry(long long B, long long T, long long n, int k, int v, int dtype,
                     Geometry* g) {
  if (k < 1 || v < 1 || k > kMaxSeqKV || v > kMaxSeqKV) return false;
  if (with_kv(k, v, [&]<int K, int V>() { *g = geometry_kv<K, V>(B, T, n, dtype); }) &&
      (g->reg || g->strip))
    return true;
  g->reg = false;
  g->strip = false;
  g->nff = k * (k + v);
  g->nfr = k * k + k * (k + v);
  g->L = 0;
  g->sper = (n + 31) / 32;
  g->nstrips = B * g->sper;
  g->nchunks = 0;
  g->ntiles = 0;
  return true;
}

inline size_t workspace_bytes(const Geometry& g, long long B, long long n, int k, int v) {
  if (g.strip) return 256;  // error word only: no look-back
  if (!g.reg) return 256 + align_up((size_t)(B * n) * 2 * k * (k + v) * sizeof(float), 256);
  return lookback_bytes(g.ntiles, g.nfr > g.nff ? g.nfr : g.nff);
}

inline size_t carry_bytes(const Geometry& g) {
  return (g.reg || g.strip) ? (size_t)g.ntiles * g.nff * 32 * sizeof(float) : 0;
}

template <typename E, int K, int V>
int launch_strip(bool fwd, Args<E>& p, const Geometry& g, void* ws, long long B, long long T,
                 cudaStream_t st) {
  if constexpr (!StripOK<K, V>::value) {
    return MGS_UNSUPPORTED;
  } else {
    MGS_CUDA_OK(cudaMemsetAsync(ws, 0, 256, st));  // error word
    StripArgs a;
    a.T_ = T;
    a.n = p.n;
    a.sper = g.sper;
    a.nstrips = g.nstrips;
    a.nchunks = g.nchunks;
    a.carries = p.carries;
    a.err = static_cast<unsigned*>(ws) + 1;
    AStripMaps maps;
    const long long n = p.n;
    if (!make_tmap_3d<E>(&maps.m[0], p.A, n * K * K, T, B, 32u * K * K, (unsigned)kLc) ||
        !make_tmap_3d<E>(&maps.m[1], p.Bm, n * K * V, T, B, 32u * K * V, (unsigned)kLc))
      return MGS_LAUNCH_FAILED;
    if (!fwd && (!make_tmap_3d<E>(&maps.m[2], p.gA, n * K * K, T, B, 32u * K * K, (unsigned)kLc) ||
                 !make_tmap_3d<E>(&maps.m[3], p.gB, n * K * V, T, B, 32u * K * V, (unsigned)kLc)))
      return MGS_LAUNCH_FAILED;
    // One CTA per SM gets a deep ring; two share an SM when strips outnumber SMs
    // (228 KB of shared memory per SM, 1 KB of it reserved per CTA).
    const void* fn = fwd ? (const void*)fwd_strip_kernel<E, K, V> : (const void*)bwd_strip_kernel<E, K, V>;
    cudaFuncAttributes fa;
    MGS_CUDA_OK(cudaFuncGetAttributes(&fa, fn));
    const int sms = sm_count();
    const size_t sbytes = fwd ? AStage<E, K, V, false>::kBytes : AStage<E, K, V, true>::kBytes;
    auto stages = [&](int ctas_per_sm) {
      const size_t per_cta = ctas_per_sm == 1 ? 227 * 1024 : 113 * 1024;
      const size_t budget = per_cta > fa.sharedSizeBytes ? per_cta - fa.sharedSizeBytes : 0;
      const int n = (int)(budget / sbytes);
      return n > kMaxStages ? kMaxStages : n;
    };
    int per_sm = g.nstrips > sms ? 2 : 1;
    int nst = stages(per_sm);
    if (nst < 2 && per_sm == 2) nst = stages(per_sm = 1);
    if (nst < 2) return MGS_UNSUPPORTED;
    a.nstage = nst;
    const size_t smem = (size_t)nst * sbytes;
    long long grid = (long long)per_sm * sms;
    if (grid > g.nstrips) grid = g.nstrips;
    void* kargs[] = {&p, &a, &maps};
    MGS_CUDA_OK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    MGS_CUDA_OK(cudaLaunchKernel(fn, dim3((unsigned)grid), dim3((kStripNW + 1) * 32), kargs, smem, st));
    return MGS_OK;
  }
}

template <typename E, int K, int V>
int launch_reg(bool fwd, Args<E>& p, const Geometry& g, void* ws, cudaStream_t st) {
  using SH = Shape<K, V>;
  if constexpr (!SH::kRegister) {
    return MGS_UNSUPPORTED;
  } else {
    MGS_CUDA_OK(cudaMemsetAsync(ws, 0, lookback_zero_bytes(g.ntiles), st));
    p.lb = lookback_view(ws, g.ntiles, g.nfr > g.nff ? g.nfr : g.nff);
    p.nchunks = g.nchunks;
    p.ntiles = g.ntiles;
    if (fwd) {
      const size_t smem = (size_t)(SH::NW + 1) * g.nff * 32 * sizeof(float);
      MGS_CUDA_OK(cudaFuncSetAttribute(fwd_kernel<E, K, V>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      fwd_kernel<E, K, V><<<(unsigned)g.ntiles, SH::NW * 32, smem, st>>>(p);
    } else {
      const size_t smem = (size_t)(SH::NW + 1) * (g.nff + g.nfr) * 32 * sizeof(float);
      MGS_CUDA_OK(cudaFuncSetAttribute(bwd_kernel<E, K, V>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      bwd_kernel<E, K, V><<<(unsigned)g.ntiles, SH::NW * 32, smem, st>>>(p);
    }
    return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
  }
}

template <typename E>
int run(bool fwd, const void* A, const void* Bm, void* Abar, void* Bbar, const void* gA,
        const void* gB, void* dA, void* dB, void* carries, long long B, long long T, long long n,
        int k, int v, void* ws, size_t ws_bytes, cudaStream_t st) {
  Geometry g;
  if (!geometry(B, T, n, k, v, dtype_of<E>(), &g)) return MGS_UNSUPPORTED;
  if (B * T * n == 0) return MGS_OK;
  if (g.ntiles > 0x7fffffffLL) return MGS_UNSUPPORTED;
  if (ws == nullptr || ws_bytes < workspace_bytes(g, B, n, k, v) || !aligned(ws, 256))
    return MGS_WORKSPACE_TOO_SMALL;
  const void* ptrs[8] = {A, Bm, fwd ? Abar : gA, fwd ? Bbar : gB, dA, dB, nullptr, nullptr};
  for (const void* q : ptrs)
    if (q != nullptr && !aligned(q, 16)) return MGS_BAD_ALIGNMENT;
  Args<E> p;
  p.A = static_cast<const E*>(A);
  p.Bm = static_cast<const E*>(Bm);
  p.Abar = static_cast<E*>(Abar);
  p.Bbar = static_cast<E*>(Bbar);
  p.gA = static_cast<const E*>(gA);
  p.gB = static_cast<const E*>(gB);
  p.dA = static_cast<E*>(dA);
  p.dB = static_cast<E*>(dB);
  p.carries = static_cast<float*>(carries);
  p.T_ = T;
  p.n = n;
  if (g.strip) {
    if (!fwd && carries == nullptr) return MGS_BAD_SHAPE;
    if (carries != nullptr && !aligned(carries, 16)) return MGS_BAD_ALIGNMENT;
    int rc = MGS_UNSUPPORTED;
    with_kv(k, v, [&]<int K, int V>() { rc = launch_strip<E, K, V>(fwd, p, g, ws, B, T, st); });
    return rc;
  }
  if (g.reg) {
    if (!fwd && carries == nullptr) return MGS_BAD_SHAPE;
    if (carries != nullptr && !aligned(carries, 16)) return MGS_BAD_ALIGNMENT;
    p.sper = g.sper;
    p.nstrips = g.nstrips;
    int rc = MGS_UNSUPPORTED;
    with_kv(k, v, [&]<int K, int V>() { rc = launch_reg<E, K, V>(fwd, p, g, ws, st); });
    return rc;
  }
  // Sequential path: the backward needs the saved forward outputs.
  if (!fwd && (Abar == nullptr || Bbar == nullptr)) return MGS_BAD_SHAPE;
  p.sper = B * n;  // lanes
  float* scratch = reinterpret_cast<float*>(static_cast<char*>(ws) + 256);
  const unsigned threads = 128;
  const unsigned blocks = (unsigned)((B * n + threads - 1) / threads);
  if (fwd)
    seq_fwd_kernel<E><<<blocks, threads, 0, st>>>(p, k, v, scratch);
  else
    seq_bwd_kernel<E><<<blocks, threads, 0, st>>>(p, k, v, scratch);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

int dispatch(bool fwd, const void* A, const void* Bm, void* Abar, void* Bbar, const void* gA,
             const void* gB, void* dA, void* dB, void* carries, long long B, long long T,
             long long n, int k, int v, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (B < 0 || T < 0 || n < 0) return MGS_BAD_SHAPE;
  switch (dtype) {
    case MGS_F32:
      return run<float>(fwd, A, Bm, Abar, Bbar, gA, gB, dA, dB, carries, B, T, n, k, v, ws,
                        ws_bytes, st);
    case MGS_BF16:
      return run<__nv_bfloat16>(fwd, A, Bm, Abar, Bbar, gA, gB, dA, dB, carries, B, T, n, k, v, ws,
                                ws_bytes, st);
    case MGS_F16:
      return run<__half>(fwd, A, Bm, Abar, Bbar, gA, gB, dA, dB, carries, B, T, n, k, v, ws,
                         ws_bytes, st);
    default:
      return MGS_BAD_DTYPE;
  }
}

}  // namespace affine

unsigned take_error_affine(cudaStream_t s) { return take_sticky_error(s); }

}  // namespace mgs

extern "C" {

size_t mgs_affine_scan_workspace_size(int64_t B, int64_t T, int64_t n, int k, int v, int dtype) {
  mgs::affine::Geometry g;
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || n < 0 ||
      !mgs::affine::geometry(B, T, n, k, v, dtype, &g))
    return 0;
  return mgs::affine::workspace_bytes(g, B, n, k, v);
}

size_t mgs_affine_scan_carry_size(int64_t B, int64_t T, int64_t n, int k, int v, int dtype) {
  mgs::affine::Geometry g;
  if (mgs::dtype_size(dtype) == 0 || B < 0 || T < 0 || n < 0 ||
      !mgs::affine::geometry(B, T, n, k, v, dtype, &g))
    return 0;
  return mgs::affine::carry_bytes(g);
}

int mgs_affine_scan_fwd(const void* A, const void* Bm, void* Abar, void* Bbar, void* carries,
                        int64_t B, int64_t T, int64_t n, int k, int v, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return mgs::affine::dispatch(true, A, Bm, Abar, Bbar, nullptr, nullptr, nullptr, nullptr, carries,
                               B, T, n, k, v, dtype, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream));
}

int mgs_affine_scan_bwd(const void* A, const void* Bm, const void* Abar, const void* Bbar,
                        const void* gAbar, const void* gBbar, const void* carries, void* dA,
                        void* dBm, int64_t B, int64_t T, int64_t n, int k, int v, int dtype,
                        void* workspace, size_t workspace_bytes, void* stream) {
  return mgs::affine::dispatch(false, A, Bm, const_cast<void*>(Abar), const_cast<void*>(Bbar),
                               gAbar, gBbar, dA, dBm, const_cast<void*>(carries), B, T, n, k, v,
                               dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
