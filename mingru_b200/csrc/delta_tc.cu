// delta_tc.cu -- DeltaMinGRU chunked-WY delta rule on the tensor cores (bf16
// or fp32 inputs, fp32 state and accumulation).
//
// Same mathematics as delta.cu (reference: DeltaMinGRU._forward_chunked,
// min_gru.py:3152-3255; backward _delta_backward_torch, triton_scans.py:
// 473-605). Per chunk of C tokens (M = nh * C micro-steps), S the state
// entering it, Ti = T^{-1}, T = I + strict_lower(K K^T) diag(beta):
//   W = Ti K,  U' = Ti V,  U = U' - W S
//   y = Q S + P U,  P = (Q K^T) diag(beta) * read_mask
//   S' = S + K^T diag(beta) U
// and, for the backward with dS' the gradient of the chunk's output state:
//   dbU = K dS',  dU = P^T dy + diag(beta) dbU,  G = Ti^T dU  (= dV)
//   dS  = dS' + Q^T dy - K^T G
//   dQ  = dy S^T + dS_ K,            dS_ = (dy U^T) diag(beta) * read_mask
//   dK  = diag(beta) U dS'^T + dS_^T Q - G S^T + dKK K + dKK^T K,
//         dKK = (-G U^T) diag(beta) * strict_lower
//   dbeta = rowsum(U * dbU) + colsum((dy U^T) * QK^T * read) + colsum((-G U^T) * KK^T * strict)
//
// Each chunk is an affine map of the state, S' = S + Xn S + Bc with
// Xn = -K^T diag(beta) W and Bc = K^T diag(beta) U', read out as
// y = Qt S + Yp with Qt = Q - P W and Yp = P U'; the adjoint chain is
// dS = dS' + Xn^T dS' + Qt^T dy. So every product that does not involve the
// state runs in parallel over all chunks, and the two chunk-serial kernels do
// one state product per chunk.
//
// Operands. A bf16 input is exact in one bf16 tile. Every other operand (fp32
// values computed here, and fp32 inputs) is held as bf16 levels: hi and lo
// (x = hi + lo to 2^-16) when the inputs are bf16, hi, mid and lo (x = h + m
// + l to 2^-24) when they are fp32. A product takes every term down to 2^-16
// of its leading one -- three MMAs per k-step for two levels, six for three
// (umma::products) -- so fp32 inputs get results within fp32 rounding of an
// fp32 computation, at twice the MMA count of the bf16 path.
//
// Kernels (the 64 x 64 chunk products run on the tcgen05 tensor cores,
// umma.cuh; for bf16 inputs T^{-1} by blocked substitution with its 16 x 16
// blocks on mma.sync, mma_bf16.cuh, for fp32 inputs by substitution in fp32):
//   prep_kernel       one CTA per (b, h, chunk): T^{-1} (saved), Xn, Qt
//   prep_f32_kernel   (saved), Bc, Yp (forward workspace).
//   chain_fwd_kernel  one CTA per (b, h, value-column split): S in registers,
//                     one chunk per step; writes y, H_T and every chunk-start
//                     state (saved for the backward).
//   chain_bwd_kernel  one CTA per (b, h, split): dS in reverse; writes dS' of
//                     every chunk and dH0.
//   bwd_grads_kernel  one CTA per (b, h, chunk): every gradient of the chunk
//                     from its saved S, T^{-1} and dS'.
// Inputs are staged with cp.async (the next chunk prefetched during the
// current one in the chunk-serial kernels); out-of-range rows and columns are
// zero-filled, which makes every padded product exact (a zero K row gives an
// identity row of T, a zero U row and no state update).
#include "delta_args.cuh"
#include "mma_bf16.cuh"
#include "umma.cuh"

namespace mgs {
namespace delta {
namespace {

using bf16 = __nv_bfloat16;
using tc::kLd;
using tc::Op;

constexpr int kTcThreads = 256;
constexpr int kTile = 64 * kLd;            // bf16 elements of one 64 x 64 tile
constexpr int kTileBytes = kTile * 2;      // 9216
constexpr int kTdBytes = 4 * 16 * 17 * 4;  // T's four diagonal 16 x 16 blocks, fp32, padded rows
constexpr int kRing = 3;  // staging depth of the chunk-serial kernels

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(tc::smem_addr(dst)),
               "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

struct Ident {
  __device__ float operator()(int, int, float x) const { return x; }
};
struct Neg {
  __device__ float operator()(int, int, float x) const { return -x; }
};

// Ti = T^{-1} for the unit lower-triangular T = I + strict_lower(T) of a chunk,
// as split bf16 tiles (X). Inputs: the strictly-lower part of T as split tiles
// (TS) and its four diagonal 16 x 16 blocks in fp32 (Td: [block][16][17]).
//   1. diagonal blocks D_b^{-1} by forward substitution (one thread per column)
//   2. X_10 = -D_1^{-1} T_10 D_0^{-1} and X_32 = -D_3^{-1} T_32 D_2^{-1} (warps 0, 1)
//   3. X[32:64, 0:32] = -X[32:64, 32:64] (T[32:64, 0:32] X[0:32, 0:32])  (warps 0-3)
// with every block product on the tensor cores (split operands, fp32 accumulate).
// X's strictly-upper 16 x 16 blocks must be zero on entry (they are never
// written); Y is scratch (two tiles).
__device__ void tri_inv_tc(const float* Td, Op TS, bf16* XH, bf16* XL, bf16* YH, bf16* YL) {
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid < 64) {
    const int o = (tid >> 4) * 16, j = tid & 15;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < i; ++k) s = fmaf(Td[(o >> 4) * 272 + i * 17 + k], x[k], s);
      x[i] = i == j ? 1.f : (i > j ? -s : 0.f);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const bf16 h = __float2bfloat16_rn(x[i]);
      XH[(o + i) * kLd + o + j] = h;
      XL[(o + i) * kLd + o + j] = __float2bfloat16_rn(x[i] - __bfloat162float(h));
    }
  }
  __syncthreads();
  const Op X{XH, XL}, Y{YH, YL};
  if (warp < 2) {
    const int i = 1 + 2 * warp, j = i - 1;
    float y[2][4];
    tc::zero(y);
    tc::gemm<2, false, true>(y, TS, 16 * i, X, 16 * j, 16 * j, 16 * j + 16);
    tc::store_split(y, YH, YL, 16 * i, 16 * j, Ident());
    __syncwarp();
    float x[2][4];
    tc::zero(x);
    tc::gemm<2, false, true>(x, X, 16 * i, Y, 16 * j, 16 * i, 16 * i + 16);
    tc::store_split(x, XH, XL, 16 * i, 16 * j, Neg());
  }
  __syncthreads();
  const int m0 = 32 + 16 * ((warp >> 1) & 1), n0 = 16 * (warp & 1);
  if (warp < 4) {
    float y[2][4];
    tc::zero(y);
    tc::gemm<2, false, true>(y, TS, m0, X, n0, 0, 32);
    tc::store_split(y, YH, YL, m0, n0, Ident());
  }
  __syncthreads();
  if (warp < 4) {
    float x[2][4];
    tc::zero(x);
    tc::gemm<2, false, true>(x, X, m0, Y, n0, 32, 64);
    tc::store_split(x, XH, XL, m0, n0, Neg());
  }
  __syncthreads();
}

// Zero the strictly-upper 16 x 16 blocks of a split tile pair (once per kernel).
template <int NTHR = kTcThreads>
__device__ void zero_upper_blocks(bf16* H, bf16* L) {
  for (int i = threadIdx.x; i < 64 * 64; i += NTHR) {
    const int row = i >> 6, col = i & 63;
    if ((col >> 4) > (row >> 4)) {
      H[row * kLd + col] = __float2bfloat16_rn(0.f);
      L[row * kLd + col] = __float2bfloat16_rn(0.f);
    }
  }
}

template <typename E>
struct TcArgs {
  const E* Q;
  const E* K;
  const E* V;
  const E* beta;
  const float* H0;
  E* y;
  float* HT;
  const E* dy;
  const float* dHT;
  E* dQ;
  E* dK;
  E* dV;
  E* dbeta;
  float* dH0;
  float* Hs;    // (BH, nchunks, dk, dv) chunk-start states
  bf16* Ti;     // (BH, nchunks, L, 64, 64) T^{-1} of every chunk, L bf16 levels, blocked
  bf16* Xn;     // (BH, nchunks, L, 64, 64) -K^T diag(beta) W
  bf16* Qt;     // (BH, nchunks, L, 64, 64) Q - P W
  float* Bc;    // (BH, nchunks, 4096) K^T diag(beta) U' as [dk][dv] (forward workspace)
  float* Yp;    // (BH, nchunks, 4096) P U' as [C][dv] (forward workspace)
  float* dHs;   // (BH, nchunks, dk, dv) gradient of each chunk's output state
  const float* lg;  // (BH, T) per-token log decay <= 0 (fp32 inputs only), or null
  float* dlg;       // (BH, T) its gradient (backward with decay)
  long long T;
  int nh, dk, dv, C, nchunks, S, dvs;
};

template <typename E>
constexpr bool kF32 = std::is_same_v<E, float>;
// bf16 levels of an fp32 operand: 2 for bf16 inputs, 3 for fp32 inputs
template <typename E>
constexpr int kLevels = kF32<E> ? 3 : 2;
// bf16 elements of one saved matrix (T^{-1}, Xn, Qt): its levels, each a
// blocked 64 x 64 tile, contiguous, so one bulk copy stages all of them
template <typename E>
constexpr long long kSavedSet = kLevels<E> * 4096LL;

__device__ __forceinline__ float tof(float x) { return x; }
__device__ __forceinline__ float tof(bf16 x) { return __bfloat162float(x); }
template <typename E>
__device__ __forceinline__ E fromf(float x) {
  if constexpr (kF32<E>) return x; else return __float2bfloat16_rn(x);
}

// A matrix held as up to three bf16 levels, each a blocked 64-column tile in
// shared memory (null: the level is absent; level 0 is always present).
struct Lv {
  bf16* t[3];
};
__device__ __forceinline__ Lv lv(bf16* a, bf16* b = nullptr, bf16* c = nullptr) {
  return Lv{{a, b, c}};
}
// the first n levels of x
__device__ __forceinline__ Lv lv_first(const Lv& x, int n) {
  return Lv{{x.t[0], n > 1 ? x.t[1] : nullptr, n > 2 ? x.t[2] : nullptr}};
}
// levels 1.. of x, level 1 first
__device__ __forceinline__ Lv lv_rest(const Lv& x) { return Lv{{x.t[1], x.t[2], nullptr}}; }
__device__ __forceinline__ uint32_t lv_addr(const bf16* t) { return t ? umma::saddr(t) : 0u; }
__device__ __forceinline__ umma::Opnd op(const Lv& x, bool mn) {
  return umma::opnd3(lv_addr(x.t[0]), lv_addr(x.t[1]), lv_addr(x.t[2]), mn);
}
__device__ __forceinline__ umma::Opnd op_mn(const Lv& x, int cols) {
  return umma::opnd_mn3(lv_addr(x.t[0]), lv_addr(x.t[1]), lv_addr(x.t[2]), cols);
}
// 8 consecutive values -> the levels of x at element offset o (of a blocked tile)
__device__ __forceinline__ void store8(const Lv& x, int o, const float* v) {
  if (x.t[2]) {
    umma::store_split8_3(x.t[0], x.t[1], x.t[2], o, v);
    return;
  }
  uint32_t ph[4], pl[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) tc::split_pack(v[2 * i], v[2 * i + 1], ph[i], pl[i]);
  *reinterpret_cast<uint4*>(x.t[0] + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
  if (x.t[1]) *reinterpret_cast<uint4*>(x.t[1] + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
}
// 16 values of row r (columns c0.., c0 % 8 == 0) of a blocked 64-column matrix
__device__ __forceinline__ void store16(const Lv& x, int r, int c0, const float (&v)[16]) {
  store8(x, umma::boff(r, c0), v);
  store8(x, umma::boff(r, c0 + 8), v + 8);
}
// as store16 for a blocked tile of `cols` columns (8-column chunks starting
// below `valid` only)
__device__ __forceinline__ void store16_n(const Lv& x, int r, int c0, int cols, int valid,
                                          const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    if (c0 + 8 * h < valid) store8(x, umma::boff_n(r, c0 + 8 * h, cols), v + 8 * h);
}

// 16 fp32 values of row r (columns c0..) -> global row (columns < ncols).
__device__ __forceinline__ void row16_f32_to_global(float* g, int c0, int ncols, const float (&v)[16]) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (c0 + 4 * k < ncols)
      *reinterpret_cast<float4*>(g + c0 + 4 * k) = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

// Per-token time decay (DeltaMinGRU._forward_chunked_gated, min_gru.py:
// 3290-3448; span sums min_gru.py:3257-3288). With l_s the chunk's per-token
// log decay, every factor is exp of a span sum span[t][t'] = sum_{s=t'+1}^{t}
// l_s, accumulated from s = t down (as the reference's flipped cumulative sum),
// each span from its own terms -- never a difference of running sums, so a
// saturated gap zeroes exactly the spans that contain it:
//   F[t][t'] = exp(span[t][t']) (t' <= t; 64 x 64 table, rows kFLd apart), P_t = exp(span[t][-1]),
//   c_m = F[Ct-1][tau(m)] (tau(m) = m / nh, the token of micro-step m).
// The chunk's maps with decay:
//   T = I + strict(K K^T * E) diag(beta),  E[i][l] = F[tau(i)][tau(l)]
//   R = (Q K^T * D * read) diag(beta),     D[t][l] = F[t][tau(l)]
//   W' = T^{-1} diag(P^) K,  U' = T^{-1} V  (P^_m = P_{tau(m)})
//   S' = P_{C-1} S + K^T diag(c beta) (U' - W' S),  y = diag(P) Q S + R (U' - W' S)
constexpr int kFLd = 65;  // row stride of the factor table: lanes reading one column of many rows hit distinct banks

// tau(m) = m / nh (the token of micro-step m) for 0 <= m < 128 without an
// integer division: (m + 1/2) / nh lies at least 1 / (2 nh) >= 1/128 from an
// integer, far beyond the rounding of m * (1 / nh) in fp32.
__device__ __forceinline__ int tok_of(int m, float inv_nh) {
  return __float2int_rz(((float)m + 0.5f) * inv_nh);
}

// The factor table F, P_t and c_m of a chunk. Row t, one warp:
// span[t][t-1-j] = a_0 + ... + a_j with a_j = l_{t-j}, an inclusive warp scan
// per 32 terms plus the running total. Every l <= 0, so any summation order
// is well conditioned; each partial sum holds only its own span's terms (no
// differences). Ends with a barrier.
__device__ void decay_tables(const float* lg, int Ct, int nh, float* F, float* Pt, float* cm) {
  for (int i = threadIdx.x; i < 64 * kFLd; i += blockDim.x) F[i] = 0.f;  // padding factors are 0
  for (int i = threadIdx.x; i < 64; i += blockDim.x) Pt[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int t = threadIdx.x >> 5; t < Ct; t += nw) {
    float carry = 0.f;
    for (int j0 = 0; j0 < t; j0 += 32) {
      const int j = j0 + lane;
      float v = j < t ? lg[t - j] : 0.f;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += n;
      }
      v += carry;
      if (j < t) F[t * kFLd + t - 1 - j] = expf(v);
      carry = __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) {
      F[t * kFLd + t] = 1.f;
      Pt[t] = expf(carry + lg[0]);
    }
  }
  __syncthreads();
  const float inh = 1.f / (float)nh;
  for (int m = threadIdx.x; m < 64; m += blockDim.x)
    cm[m] = m < Ct * nh ? F[(Ct - 1) * kFLd + tok_of(m, inh)] : 0.f;
  __syncthreads();
}

// dst = diag(f[tau(row)]) x, x given by its three blocked levels in shared
// memory (rows >= nrows zero), re-split into three levels.
template <int NTHR>
__device__ __forceinline__ void scale_rows_levels(const Lv& dst, const Lv& x, int nrows, const float* f,
                                                  float inh) {
  for (int i = threadIdx.x; i < 64 * 8; i += NTHR) {
    const int row = i >> 3, ch = i & 7, o = umma::boff(row, ch * 8);
    const float sc = row < nrows ? f[tok_of(row, inh)] : 0.f;
    const uint4 h = *reinterpret_cast<const uint4*>(x.t[0] + o);
    const uint4 m = *reinterpret_cast<const uint4*>(x.t[1] + o);
    const uint4 l = *reinterpret_cast<const uint4*>(x.t[2] + o);
    const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, mw[4] = {m.x, m.y, m.z, m.w}, lw[4] = {l.x, l.y, l.z, l.w};
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hw[k]));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&mw[k]));
      const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&lw[k]));
      v[2 * k] = sc * (a.x + b.x + c.x);
      v[2 * k + 1] = sc * (a.y + b.y + c.y);
    }
    store8(dst, o, v);
  }
}

// ----------------------------------------------------- backward: grads --
// One CTA per (b, h, chunk), two CTAs per SM for bf16 inputs (one for fp32):
// every gradient of the chunk from its saved S, T^{-1} and dS', on the tcgen05
// tensor cores (umma.cuh). Two
// threads (lane 0 of warps 0 and 1) issue each level of products, split by
// accumulator, as batches of 64 x 64 x 64 split MMAs into TMEM and commit to
// one barrier of arrival count 2 (MMA issue, not the tensor pipe, bounds these
// shapes, so the second CTA on the SM fills the gaps); all 8 warps then read
// the accumulators (warp w: rows 16*(w%4).., columns 32*(w/4)..) and write the
// masked / scaled / split operands of the next level:
//   1. W = Ti K, U' = Ti V, dbU = K dS', Q K^T            [P = Q K^T beta * read]
//   2. U = U' + (-W) S (same accumulator), P^T dy         [dU = P^T dy + beta dbU]
//   3. G = Ti^T dU (two accumulators, -> dV), U dS'^T (held in registers)
//   4. dy U^T, Gn U^T (Gn = -G), K K^T, Q K^T             [-> dS_, dKK, dbeta columns]
//   5. dQ = dy S^T + dS_ K;  dK = beta * (U dS'^T) + dS_^T Q + dKK K + Gn S^T + dKK^T K
// TMEM: four 64-column accumulators A, B, C, D (256 columns per CTA), each
// reused once its previous contents have been read.
// Shared tiles (blocked, 8 KB), bf16 inputs: 0 K | 1 Q | 2 dY | 3, 4 S |
//   5, 6 dS' -> dKK | 7, 8 Ti -> Gn | 9 V -> -W hi -> U hi | 10, 11 P -> dU ->
//   dS_ | 12 -W lo -> U lo (two CTAs per SM); fp32 inputs, three levels each:
//   0-2 K | 3-5 Q | 6-8 dY | 9-11 S | 12-14 dS' -> dKK | 15-17 Ti -> Gn |
//   18-20 V -> -W -> U | 21-23 P -> dU -> dS_ (one CTA per SM).
constexpr int kGradThreads = 256;
template <typename E>
constexpr int kGradTiles = kF32<E> ? 24 : 13;
template <typename E>
constexpr size_t kGradSmem = 1024 + kGradTiles<E> * (size_t)umma::kTileBytes + 2048;
// decay: span factor table [64][65], P_t [64], c_m [64]; fp64: the d l difference
// array [80], column sums [4][2][32], row sums [2][64] x 2, carry terms [64], warp sums [16]
constexpr size_t kGradDecaySmem = 64 * 65 * 4 + (64 + 64) * 4 + (80 + 256 + 128 + 128 + 64 + 16) * 8;
constexpr int kGradTmemCols = 256;

// 64 rows x (8 * valid_ch) columns of a row-major global bf16 matrix into a
// blocked tile (cp.async); rows >= nrows and chunks >= valid_ch are zero.
template <int NTHR>
__device__ __forceinline__ void stage_blocked(bf16* tile, const bf16* g, long long ld, int nrows,
                                              int valid_ch) {
  for (int i = threadIdx.x; i < 64 * 8; i += NTHR) {
    const int row = i >> 3, ch = i & 7;
    const bool ok = row < nrows && ch < valid_ch;
    cp_async16(tile + umma::boff(row, ch * 8), ok ? g + row * ld + ch * 8 : g, ok ? 16 : 0);
  }
}

// An input matrix (64 rows x 8 * valid_ch columns of a row-major global
// matrix; other rows and chunks zero) into its blocked levels: bf16 by
// cp.async (the caller commits and waits), fp32 loaded and split into three
// levels here.
template <int NTHR, typename E>
__device__ __forceinline__ void stage_in(const Lv& x, const E* g, long long ld, int nrows,
                                         int valid_ch) {
  if constexpr (kF32<E>) {
    for (int i = threadIdx.x; i < 64 * 8; i += NTHR) {
      const int row = i >> 3, ch = i & 7;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (row < nrows && ch < valid_ch) {
        a = __ldg(reinterpret_cast<const float4*>(g + row * ld + ch * 8));
        b = __ldg(reinterpret_cast<const float4*>(g + row * ld + ch * 8 + 4));
      }
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      store8(x, umma::boff(row, ch * 8), v);
    }
  } else {
    stage_blocked<NTHR>(x.t[0], g, ld, nrows, valid_ch);
  }
}

// Several fp32 input matrices into their blocked levels with every load of
// every matrix issued before the first split (one memory round trip, as the
// bf16 path's cp.async copies are all in flight together).
struct InSrc {
  const float* g;
  long long ld;
  int nrows, valid_ch;
};
template <int NTHR, int N>
__device__ __forceinline__ void stage_in_f32(const Lv (&x)[N], const InSrc (&src)[N]) {
  constexpr int U = 64 * 8 / NTHR;  // 8-column units of a 64 x 64 matrix per thread
  float4 a[N][U][2];
#pragma unroll
  for (int m = 0; m < N; ++m)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = threadIdx.x + u * NTHR, row = i >> 3, ch = i & 7;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const bool ok = row < src[m].nrows && ch < src[m].valid_ch;
      const float4* q = reinterpret_cast<const float4*>(src[m].g + row * src[m].ld + ch * 8);
      a[m][u][0] = ok ? __ldg(q) : z;
      a[m][u][1] = ok ? __ldg(q + 1) : z;
    }
#pragma unroll
  for (int m = 0; m < N; ++m)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = threadIdx.x + u * NTHR, row = i >> 3, ch = i & 7;
      const float v[8] = {a[m][u][0].x, a[m][u][0].y, a[m][u][0].z, a[m][u][0].w,
                          a[m][u][1].x, a[m][u][1].y, a[m][u][1].z, a[m][u][1].w};
      store8(x[m], umma::boff(row, ch * 8), v);
    }
}


// Columns c0..c0+15 of an accumulator row -> bf16 global row (columns < ncols).
__device__ __forceinline__ void row16_to_global(bf16* g, int c0, int ncols, const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    if (c0 + 8 * h < ncols) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = tc::pack_bf16(v[8 * h + 2 * i], v[8 * h + 2 * i + 1]);
      *reinterpret_cast<uint4*>(g + c0 + 8 * h) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}
__device__ __forceinline__ void row16_to_global(float* g, int c0, int ncols, const float (&v)[16]) {
  row16_f32_to_global(g, c0, ncols, v);
}

// DEC (fp32 inputs, per-token decay p.lg; the maps of decay_tables): level 1
// takes K S instead of T^{-1} K and level 2 forms U = U' + T^{-1} (-P^ K S);
// level 3 adds dy S^T (diag(P) dy S^T is dQ's first term, kept in registers);
// the masks of levels 1 and 4 carry the span factors; dK's -G S^T rows take
// P^, its U dS'^T rows c; and every factor's gradient is gathered per token
// span (t', t] into `dl` as a difference array (+w at t' + 1, -w at t + 1:
// d l_s is the sum over the spans containing s, a prefix sum at the end), the
// entries of span-free factors (same token, factor 1) left out.
template <typename E, bool DEC = false>
__global__ void __launch_bounds__(kGradThreads, kF32<E> ? 1 : 2) bwd_grads_kernel(const TcArgs<E> p) {
  namespace um = umma;
  constexpr bool F = kF32<E>;
  constexpr int L = kLevels<E>;
  extern __shared__ __align__(1024) unsigned char gsmem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(gsmem);  // [0] MMA batches, [1] T^{-1} copy
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(gsmem + 64);
  bf16* tiles = reinterpret_cast<bf16*>(gsmem + 1024);
  auto T = [&](int i) { return tiles + i * (um::kTileBytes / 2); };
  const Lv K = F ? lv(T(0), T(1), T(2)) : lv(T(0));
  const Lv Q = F ? lv(T(3), T(4), T(5)) : lv(T(1));
  const Lv dY = F ? lv(T(6), T(7), T(8)) : lv(T(2));
  const Lv S = F ? lv(T(9), T(10), T(11)) : lv(T(3), T(4));
  const Lv Dp = F ? lv(T(12), T(13), T(14)) : lv(T(5), T(6));  // dS' -> dKK
  const Lv Ti = F ? lv(T(15), T(16), T(17)) : lv(T(7), T(8));  // T^{-1} -> Gn
  const Lv V = F ? lv(T(18), T(19), T(20)) : lv(T(9));
  const Lv W = F ? V : lv(T(9), T(12));                         // -W -> U
  const Lv P = F ? lv(T(21), T(22), T(23)) : lv(T(10), T(11));  // P -> dU -> dS_
  const Lv &dKK = Dp, &Gn = Ti, &U = W, &dU = P, &dS_ = P;
  float* bs = reinterpret_cast<float*>(T(kGradTiles<E>));
  float* rpart = bs + 64;      // [2 column halves][64 rows]: sum_col U * dbU
  float* cpart = rpart + 128;  // [8 warps][32 columns]: masked-product column sums
  float* Ft = bs + 512;        // decay: factor table [64][kFLd]
  float* Pt = Ft + 64 * kFLd;  // decay: P_t
  float* cm = Pt + 64;         // decay: c_m
  // decay: the d l difference array [Cc + 1] and the partial sums it is built
  // from, in fp64 (a prefix sum carries every entry's rounding into all later
  // tokens, and in fp32 that shared error adds up coherently in sums over tokens,
  // the gradient of lambda). Every partial has one writer: no atomics.
  double* dl = reinterpret_cast<double*>(cm + 64);
  double* colb = dl + 80;     // [q][hh][32]: column sums of the level-4 span terms (+ at tau(l) + 1)
  double* rowT = colb + 256;  // [hh][64]: token-row terms, negated (at t + 1)
  double* rowM = rowT + 128;  // [hh][64]: micro-step-row terms, negated (at tau(i) + 1)
  double* carS = rowM + 128;  // [64]: carry terms (+ at tau(m) + 1, - at Ct)
  double* wred = carS + 64;   // [2][8]: per-warp sums of the (-1, .] terms and of <S, dS'>
  double accT = 0.0, accM = 0.0, acc0 = 0.0, accS = 0.0;  // this thread's partials

  constexpr int NTH = kGradThreads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hh = warp >> 2, row = 16 * q + lane;
  const bool rv = lane < 16;  // this lane holds row `row` of the 64-row accumulators
  const float inh = 1.f / (float)p.nh;
  const int c = blockIdx.x % p.nchunks;
  const long long bh = blockIdx.x / p.nchunks;
  const long long t0 = (long long)c * p.C;
  const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
  const long long r0 = t0 * p.nh, rows = p.T * p.nh;
  const long long blk = bh * p.nchunks + c;
  const long long sofs = blk * (long long)p.dk * p.dv;

  // decay: two more accumulators (E, F: U dS'^T and dy S^T, read at the last
  // epilogue) -- one CTA per SM, so all 512 columns are free
  constexpr int kCols = DEC ? 2 * kGradTmemCols : kGradTmemCols;
  if (warp == 0) um::alloc(tbase_s, kCols);
  if (tid == 0) {
    mbar_init(bar, 2);  // MMA batches: one commit from each issuing thread
    mbar_init(bar + 1, 1);
    mbar_fence_init();
  }
  if constexpr (F) {
    const Lv xs[4] = {K, Q, dY, V};
    const InSrc ss[4] = {{p.K + (bh * rows + r0) * p.dk, p.dk, Mc, p.dk >> 3},
                         {p.Q + (bh * p.T + t0) * p.dk, p.dk, Cc, p.dk >> 3},
                         {p.dy + (bh * p.T + t0) * p.dv, p.dv, Cc, p.dv >> 3},
                         {p.V + (bh * rows + r0) * p.dv, p.dv, Mc, p.dv >> 3}};
    stage_in_f32<NTH>(xs, ss);
  } else {
    stage_in<NTH>(K, p.K + (bh * rows + r0) * p.dk, p.dk, Mc, p.dk >> 3);
    stage_in<NTH>(Q, p.Q + (bh * p.T + t0) * p.dk, p.dk, Cc, p.dk >> 3);
    stage_in<NTH>(dY, p.dy + (bh * p.T + t0) * p.dv, p.dv, Cc, p.dv >> 3);
    stage_in<NTH>(V, p.V + (bh * rows + r0) * p.dv, p.dv, Mc, p.dv >> 3);
  }
  cp_async_commit();
  um::fence_before();
  __syncthreads();  // barriers initialised, TMEM base written
  if (tid == 0) {  // T^{-1}: its levels are contiguous in `saved` and in shared memory
    mbar_arrive_expect_tx(bar + 1, L * um::kTileBytes);
    bulk_g2s(Ti.t[0], p.Ti + blk * kSavedSet<E>, L * um::kTileBytes, bar + 1);
  }
  {  // S (chunk-start state) and dS' (fp32 [dk][dv]) -> blocked levels
    float4 a[2][2], b[2][2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * NTH, r = i >> 3, cb = i & 7;
      const bool ok = r < p.dk && cb * 8 < p.dv;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4* sa = reinterpret_cast<const float4*>(p.Hs + sofs + r * p.dv + cb * 8);
      const float4* sb = reinterpret_cast<const float4*>(p.dHs + sofs + r * p.dv + cb * 8);
      a[k][0] = ok ? sa[0] : z;
      a[k][1] = ok ? sa[1] : z;
      b[k][0] = ok ? sb[0] : z;
      b[k][1] = ok ? sb[1] : z;
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * NTH, r = i >> 3, cb = i & 7;
      const float av[8] = {a[k][0].x, a[k][0].y, a[k][0].z, a[k][0].w,
                           a[k][1].x, a[k][1].y, a[k][1].z, a[k][1].w};
      const float bv[8] = {b[k][0].x, b[k][0].y, b[k][0].z, b[k][0].w,
                           b[k][1].x, b[k][1].y, b[k][1].z, b[k][1].w};
      const int o = um::boff(r, cb * 8);
      store8(S, o, av);
      store8(Dp, o, bv);
      if constexpr (DEC) {  // <S, dS'>: the gradient of P_{C-1} S
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) d = fmaf(av[j], bv[j], d);
        accS += d;
      }
    }
  }
  if (tid < 64) bs[tid] = tid < Mc ? tof(p.beta[bh * rows + r0 + tid]) : 0.f;
  if constexpr (DEC) decay_tables(p.lg + bh * p.T + t0, Cc, p.nh, Ft, Pt, cm);  // barriers inside
  cp_async_wait_all();
  // okw: every wait so far completed. A wait that runs out records the time-out
  // (sticky word) and from then on this CTA issues no MMA, waits on nothing and
  // writes no output; to_mma makes the flag the same in every thread.
  bool okw = mbar_wait(bar + 1, 0, &g_sticky_err);
  const uint32_t tb = *tbase_s;
  const uint32_t tA = tb, tB = tb + 64, tC = tb + 128, tD = tb + 192;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + 32 * hh;  // this warp's accumulator window

  unsigned phase = 0;
  // make this thread's shared-memory writes visible to the tensor cores and
  // order its TMEM reads before the next batch of MMAs
  auto to_mma = [&]() {
    fence_proxy_async_smem();
    um::fence_before();
    okw = !__syncthreads_or(!okw);
    um::fence_after();
  };
  auto wait_mma = [&]() {
    if (okw) okw = mbar_wait(bar, phase, &g_sticky_err);
    phase ^= 1u;
    um::fence_after();
  };

  // level 1
  to_mma();
  if (okw && tid == 0) {
    const um::Opnd oTi = op(Ti, false);
    const um::Prod ps[2] = {{tA, DEC ? op(K, false) : oTi, op(DEC ? S : K, true), false},
                            {tB, oTi, op(V, true), false}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {
    const um::Prod ps[2] = {{tC, op(K, false), op(Dp, true), false},
                            {tD, op(Q, false), op(K, false), false}};
    um::products(ps);
    um::commit(bar);
  }
  wait_mma();
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // P = Q K^T beta[col] * read (D);  -W (A)
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16];
    float v[16], w[16];
    um::ld16_async(lb + 192 + 16 * half, r1);
    um::ld16_async(lb + 0 + 16 * half, r2);
    um::ld_wait();
    um::ld_bind(r1, v);
    um::ld_bind(r2, w);
    if (rv) {
      // decay: -W <- -P^ (K S) (rhs of U = T^{-1} (V - P^ K S)), P's read factors D
      const float ph = DEC ? (row < Mc ? Pt[tok_of(row, inh)] : 0.f) : 1.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int cl = c0 + i;
        const bool rd = cl < (row + 1) * p.nh && cl < Mc;
        v[i] = rd ? v[i] * bs[cl] : 0.f;
        if constexpr (DEC) v[i] *= rd && row < Cc ? Ft[row * kFLd + tok_of(cl, inh)] : 0.f;
        w[i] = -ph * w[i];
      }
      store16(P, row, c0, v);
      store16(W, row, c0, w);
    }
  }
  // level 2
  to_mma();
  if (okw && tid == 0) {  // U = U' + (-W) S, decay U' + T^{-1} (-P^ K S)
    const um::Prod ps[1] = {{tB, op(DEC ? Ti : W, false), op(DEC ? W : S, true), true}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {
    const um::Prod ps[1] = {{tA, op(P, true), op(dY, true), false}};
    um::products(ps);
    um::commit(bar);
  }
  wait_mma();
  {  // U (B), beta U, dU = P^T dy (A) + beta dbU (C); row sums of U * dbU
    float rs = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c0 = 32 * hh + 16 * half;
      uint32_t r1[16], r2[16], r3[16];
      float u[16], db[16], pd[16];
      um::ld16_async(lb + 64 + 16 * half, r1);
      um::ld16_async(lb + 128 + 16 * half, r2);
      um::ld16_async(lb + 0 + 16 * half, r3);
      um::ld_wait();
      um::ld_bind(r1, u);
      um::ld_bind(r2, db);
      um::ld_bind(r3, pd);
      if (rv) {
        const float b = DEC ? bs[row] * cm[row] : bs[row];  // decay: carry factor c
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          rs += u[i] * db[i];
          pd[i] += b * db[i];
        }
        store16(U, row, c0, u);
        store16(dU, row, c0, pd);
      }
    }
    if (rv) rpart[hh * 64 + row] = rs;
  }
  // level 3
  to_mma();
  if (okw && tid == 0) {  // G = Ti^T dU, its terms in two accumulators: Ti^T dU_hi (C), the rest (D)
    const um::Prod ps[2] = {
        {tC, op(Ti, true), op(lv_first(dU, 1), true), false},
        {tD, op(lv_first(Ti, L - 1), true), op(lv_rest(dU), true), false}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {  // U dS'^T in A (decay: in E, and dy S^T in F)
    if constexpr (DEC) {
      const um::Prod ps[2] = {{tb + 256, op(U, false), op(Dp, false), false},
                              {tb + 320, op(dY, false), op(S, false), false}};
      um::products(ps);
    } else {
      const um::Prod ps[1] = {{tA, op(U, false), op(Dp, false), false}};
      um::products(ps);
    }
    um::commit(bar);
  }
  wait_mma();
  float uds[2][16];  // U dS'^T of this thread's row, held until the last epilogue (no decay)
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // dV = G; Gn = -G
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16], r3[16];
    float g[16], g2[16];
    um::ld16_async(lb + 128 + 16 * half, r1);
    um::ld16_async(lb + 192 + 16 * half, r2);
    if constexpr (!DEC) um::ld16_async(lb + 0 + 16 * half, r3);
    um::ld_wait();
    um::ld_bind(r1, g);
    um::ld_bind(r2, g2);
    if constexpr (!DEC) um::ld_bind(r3, uds[half]);
    if (rv) {
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] += g2[i];
      if (okw && row < Mc) row16_to_global(p.dV + (bh * rows + r0 + row) * p.dv, c0, p.dv, g);
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] = -g[i];
      store16(Gn, row, c0, g);
    }
  }
  // level 4
  to_mma();
  if (okw && tid == 0) {  // Gn U^T in B, K K^T in C
    const um::Prod ps[2] = {{tB, op(Gn, false), op(U, false), false},
                            {tC, op(K, false), op(K, false), false}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {  // dy U^T in A, Q K^T in D
    const um::Prod ps[2] = {{tA, op(dY, false), op(U, false), false},
                            {tD, op(Q, false), op(K, false), false}};
    um::products(ps);
    um::commit(bar);
  }
  wait_mma();
  {  // dS_ = (dy U^T) beta * read; dKK = (Gn U^T) beta * strict; dbeta column terms
    float cs = 0.f;  // after the reductions lane i < 32 holds column 32*hh + i
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c0 = 32 * hh + 16 * half;
      uint32_t r1[16], r2[16], r3[16], r4[16];
      float ds[16], dk[16], kk[16], qk[16];
      um::ld16_async(lb + 0 + 16 * half, r1);
      um::ld16_async(lb + 64 + 16 * half, r2);
      um::ld16_async(lb + 128 + 16 * half, r3);
      um::ld16_async(lb + 192 + 16 * half, r4);
      um::ld_wait();
      um::ld_bind(r1, ds);
      um::ld_bind(r2, dk);
      um::ld_bind(r3, kk);
      um::ld_bind(r4, qk);
      float e[16];  // this row's dbeta column terms
      // decay: the factor gradients of span-carrying entries (x beta), summed by
      // row and by column in fp64 so that the +w / -w entries they make in the
      // difference array cancel exactly outside each span
      double eg[16];
      double rsR = 0.0, rsT = 0.0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int cl = c0 + i;
        const float x = (rv && cl < (row + 1) * p.nh && cl < Mc) ? ds[i] : 0.f;
        const float y = (rv && cl < row && cl < Mc) ? dk[i] : 0.f;
        if constexpr (DEC) {
          const int tl = tok_of(cl, inh), tr = tok_of(row, inh);
          const float fd = rv && row < Cc ? Ft[row * kFLd + tl] : 0.f;     // D[t][l]
          const float fe = rv && row < Mc ? Ft[tr * kFLd + tl] : 0.f;      // E[i][l]
          const float xr = x * qk[i] * fd, yt = y * kk[i] * fe;
          e[i] = xr + yt;
          const double wr = tl < row ? (double)(xr * bs[cl]) : 0.0;  // span (tau(l), t]
          const double wt = tl < tr ? (double)(yt * bs[cl]) : 0.0;   // span (tau(l), tau(i)]
          rsR += wr;
          rsT += wt;
          eg[i] = wr + wt;
          ds[i] = x * bs[cl] * fd;
          dk[i] = y * bs[cl] * fe;
        } else {
          e[i] = rv ? x * qk[i] + y * kk[i] : 0.f;
          ds[i] = x * bs[cl];
          dk[i] = y * bs[cl];
        }
      }
      if constexpr (DEC) {
        accT -= rsR;  // zero on padded rows (their factors are 0)
        accM -= rsT;
        // column sums of eg (as for e below): + at tau(l) + 1
#pragma unroll
        for (int d = 8, n = 16; d >= 1; d >>= 1, n >>= 1) {
          const bool upper = (lane & d) != 0;
#pragma unroll
          for (int j = 0; j < n / 2; ++j) {
            const double keep = upper ? eg[j + n / 2] : eg[j];
            const double send = upper ? eg[j] : eg[j + n / 2];
            eg[j] = keep + __shfl_xor_sync(0xffffffffu, send, d);
          }
        }
        const double colg = __shfl_sync(0xffffffffu, eg[0], lane & 15);
        if (lane < 16) colb[(q * 2 + hh) * 32 + 16 * half + lane] = colg;
      }
      // column sums over the 16 rows of each half-warp by a transposing
      // butterfly: at distance d a lane keeps the half of its values selected
      // by lane bit d and adds its partner's copy of that half, so lane i ends
      // with column i (15 shuffles for 16 columns).
#pragma unroll
      for (int d = 8, n = 16; d >= 1; d >>= 1, n >>= 1) {
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int j = 0; j < n / 2; ++j) {
          const float keep = upper ? e[j + n / 2] : e[j];
          const float send = upper ? e[j] : e[j + n / 2];
          e[j] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
      }
      const float colsum = __shfl_sync(0xffffffffu, e[0], lane & 15);  // from the row lanes 0-15
      if ((lane >> 4) == half) cs = colsum;
      if (rv) {
        store16(dS_, row, c0, ds);
        store16(dKK, row, c0, dk);
      }
    }
    cpart[warp * 32 + lane] = cs;
  }
  // level 5
  to_mma();
  if (okw && tid == 0) {  // dQ in A (decay: its dy S^T term is in registers), Gn S^T in C
    const um::Opnd oS = op(S, false);
    if constexpr (DEC) {
      const um::Prod ps[2] = {{tC, op(Gn, false), oS, false}, {tA, op(dS_, false), op(K, true), false}};
      um::products(ps);
    } else {
      const um::Prod ps[3] = {{tA, op(dY, false), oS, false},
                              {tC, op(Gn, false), oS, false},
                              {tA, op(dS_, false), op(K, true), true}};
      um::products(ps);
    }
    um::commit(bar);
  } else if (okw && tid == 32) {  // dS_^T Q + dKK K in B, dKK^T K in D
    const um::Opnd oKmn = op(K, true);
    const um::Prod ps[3] = {{tB, op(dS_, true), op(Q, true), false},
                            {tD, op(dKK, true), oKmn, false},
                            {tB, op(dKK, false), oKmn, true}};
    um::products(ps);
    um::commit(bar);
  }
  wait_mma();
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // dQ (token rows), dK (micro-step rows)
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16], r3[16], r4[16];
    float v[16], v2[16], v3[16], v4[16];
    um::ld16_async(lb + 0 + 16 * half, r1);
    um::ld16_async(lb + 64 + 16 * half, r2);
    um::ld16_async(lb + 128 + 16 * half, r3);
    um::ld16_async(lb + 192 + 16 * half, r4);
    um::ld_wait();
    um::ld_bind(r1, v);
    um::ld_bind(r2, v2);
    um::ld_bind(r3, v3);
    um::ld_bind(r4, v4);
    if constexpr (DEC) {  // U dS'^T (E); dQ += P_t (dy S^T) (F), whose Q-weighted sum is dP_t
      uint32_t r5[16], r6[16];
      float dys[16];
      um::ld16_async(lb + 256 + 16 * half, r5);
      um::ld16_async(lb + 320 + 16 * half, r6);
      um::ld_wait();
      um::ld_bind(r5, uds[half]);
      um::ld_bind(r6, dys);
      const float pt = rv && row < Cc ? Pt[row] : 0.f;
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int o = um::boff(row, c0 + i);
        const float qv = __bfloat162float(Q.t[0][o]) + __bfloat162float(Q.t[1][o]) +
                         __bfloat162float(Q.t[2][o]);
        d = fmaf(qv, dys[i], d);
        v[i] += pt * dys[i];
      }
      if (rv && row < Cc) {  // G2[t][-1] += P_t dP_t
        acc0 += (double)(pt * d);
        accT -= (double)(pt * d);
      }
    }
    if (okw && rv && row < Cc) row16_to_global(p.dQ + (bh * p.T + t0 + row) * p.dk, c0, p.dk, v);
    if (okw && rv && row < Mc) {
      const float b = DEC ? bs[row] * cm[row] : bs[row];
      if constexpr (DEC) {  // -G S^T rows take P^; its K-weighted sum is the gradient of P^
        const float ph = Pt[tok_of(row, inh)];
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int o = um::boff(row, c0 + i);
          const float kv = __bfloat162float(K.t[0][o]) + __bfloat162float(K.t[1][o]) +
                           __bfloat162float(K.t[2][o]);
          d = fmaf(kv, v3[i], d);
          v3[i] *= ph;
        }
        acc0 += (double)(ph * d);  // G2[tau(m)][-1] += P^_m dP^_m
        accM -= (double)(ph * d);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) v2[i] += v3[i] + v4[i] + b * uds[half][i];
      row16_to_global(p.dK + (bh * rows + r0 + row) * p.dk, c0, p.dk, v2);
    }
  }
  um::fence_before();
  __syncthreads();
  if (okw && tid < Mc) {  // dbeta = row sums of U * dbU + column sums of the masked products
    const int h2 = tid >> 5, cl = tid & 31;
    const float ru = rpart[tid] + rpart[64 + tid];
    const float d = (DEC ? cm[tid] * ru : ru) +
                    (cpart[(4 * h2) * 32 + cl] + cpart[(4 * h2 + 1) * 32 + cl]) +
                    (cpart[(4 * h2 + 2) * 32 + cl] + cpart[(4 * h2 + 3) * 32 + cl]);
    p.dbeta[bh * rows + r0 + tid] = fromf<E>(d);
    if constexpr (DEC)  // carry factor c_m: span (tau(m), Ct - 1]
      carS[tid] = tok_of(tid, inh) < Cc - 1 ? (double)(bs[tid] * cm[tid] * ru) : 0.0;
  }
  if constexpr (DEC) {
    if (tid >= Mc && tid < 64) carS[tid] = 0.0;
    if (rv) {
      rowT[hh * 64 + row] = accT;
      rowM[hh * 64 + row] = accM;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
      accS += __shfl_xor_sync(0xffffffffu, accS, o);
    }
    if (lane == 0) {
      wred[warp] = acc0;
      wred[8 + warp] = accS;
    }
    __syncthreads();
    if (tid <= Cc) {  // difference-array entry u = tid: + terms starting at u, - terms ending at u
      const int u = tid;
      double sum = 0.0, car = 0.0;
      for (int m = 0; m < Mc; ++m) car += carS[m];
      if (u == 0) {
        double z = 0.0, sd = 0.0;
        for (int w = 0; w < 8; ++w) {
          z += wred[w];
          sd += wred[8 + w];
        }
        sum = z + (double)Pt[Cc - 1] * sd;  // (-1, t] terms and P_{C-1} S: span (-1, Ct - 1]
      }
      if (u >= 1) {
        for (int l = (u - 1) * p.nh; l < u * p.nh && l < Mc; ++l) {  // columns of token u - 1
          for (int qq = 0; qq < 4; ++qq) sum += colb[(qq * 2 + (l >> 5)) * 32 + (l & 31)];
          sum += carS[l];
          sum += rowM[l] + rowM[64 + l];  // micro-step rows of token u - 1 (hold -w)
        }
        if (u - 1 < Cc) sum += rowT[u - 1] + rowT[64 + u - 1];  // token row u - 1 (holds -w)
      }
      if (u == Cc) sum -= car + (double)Pt[Cc - 1] * [&] {
        double sd = 0.0;
        for (int w = 0; w < 8; ++w) sd += wred[8 + w];
        return sd;
      }();
      dl[u] = sum;
    }
    __syncthreads();
    if (okw && tid == 0) {  // d l_s = prefix sums of the difference array
      double acc = 0.0;
      for (int t = 0; t < Cc; ++t) {
        acc += dl[t];
        p.dlg[bh * p.T + t0 + t] = (float)acc;
      }
    }
  }
  if (warp == 0) {
    um::fence_after();
    um::dealloc(tb, kCols);
  }
}

constexpr int kF32Ld = 65;  // row stride of the fp32 64 x 64 matrices of the inverse

// X = T^{-1} for the unit lower-triangular T = I + Tf (Tf strictly lower,
// fp32 [64][kF32Ld]) in fp32: the four diagonal 16 x 16 blocks by forward
// substitution (a thread per column), then block row i = 1..3 from the rows
// above it, X_ij = -D_i^{-1} sum_{k=j}^{i-1} T_ik X_kj (Ys holds the sums).
// X's strictly-upper blocks are zeroed first, so every sum runs over a fixed
// range (unrolled; each thread carries 1-3 independent sums). 256 threads;
// ends with __syncthreads.
__device__ void tri_inv_f32(const float* Tf, float* Xf, float* Ys) {
  const int tid = threadIdx.x;
  for (int i = tid; i < 64 * 64; i += 256) {
    const int r = i >> 6, c = i & 63;
    if ((c >> 4) > (r >> 4)) Xf[r * kF32Ld + c] = 0.f;
  }
  if (tid < 64) {
    const int o = (tid >> 4) * 16, j = tid & 15;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < i; ++k) s = fmaf(Tf[(o + i) * kF32Ld + o + k], x[k], s);
      x[i] = i == j ? 1.f : (i > j ? -s : 0.f);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) Xf[(o + i) * kF32Ld + o + j] = x[i];
  }
  __syncthreads();
#pragma unroll
  for (int bi = 1; bi < 4; ++bi) {
    const int r0 = 16 * bi, ncol = 16 * bi;  // 16 x ncol outputs: bi per thread
    float y[3];
#pragma unroll
    for (int u = 0; u < bi; ++u) {
      const int e = tid + 256 * u, r = e / ncol, cc = e - r * ncol;
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < r0; ++k) acc = fmaf(Tf[(r0 + r) * kF32Ld + k], Xf[k * kF32Ld + cc], acc);
      y[u] = acc;
    }
#pragma unroll
    for (int u = 0; u < bi; ++u) {
      const int e = tid + 256 * u, r = e / ncol, cc = e - r * ncol;
      Ys[r * 48 + cc] = y[u];
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < bi; ++u) {
      const int e = tid + 256 * u, r = e / ncol, cc = e - r * ncol;
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) acc = fmaf(Xf[(r0 + r) * kF32Ld + r0 + k], Ys[k * 48 + cc], acc);
      y[u] = -acc;
    }
#pragma unroll
    for (int u = 0; u < bi; ++u) {
      const int e = tid + 256 * u, r = e / ncol, cc = e - r * ncol;
      Xf[(r0 + r) * kF32Ld + cc] = y[u];
    }
    __syncthreads();
  }
}

// DEC: per-token time decay (p.lg): the span factors enter T and P~ (level-1
// epilogue), W' is T^{-1} (P^ K) and the K^T products take c K (levels 3, 4),
// and Xn, Qt take P_{C-1} and P (last epilogue) -- the maps above. The tables
// live in Xf until the inverse, P^ K and then c K over Tf / Xf.
// ------------------------------------------------------- forward: prep --
// One CTA per (b, h, chunk), independent of the state, two CTAs per SM: T,
// T^{-1} (saved for the backward), and the chunk's affine state map and readout
//   S' = S + Xn S + Bc,   Xn = -K^T (beta W),  Bc = K^T (beta U')
//   y  = Qt S + Yp,       Qt = Q - P~ (beta W), Yp = P~ (beta U')
// with W = Ti K, U' = Ti V, P~ = (Q K^T) * read_mask (P = P~ diag(beta)).
// The products run on the tcgen05 tensor cores (umma.cuh):
//   1. [K; Q] K^T as one M = 128 product          -> T (strict lower, beta), P~
//   2. (T^{-1} by blocked substitution on mma.sync, tri_inv_tc)
//   3. Ti K, Ti V                                   -> beta W, beta U'
//   4. K^T (beta W), P~ (beta W), K^T (beta U'), P~ (beta U')
// Xn, Qt (split bf16) and T^{-1} (for the grads) go to `saved` in the blocked
// layout, Bc and Yp (fp32) to the forward workspace, all staged in shared
// memory and written by bulk copies.
// smem: header | K | Q | V | P~ h/l (blocked) | beta | Td | region R of six
// padded tiles: T h/l, X h/l, Y h/l for the inverse; afterwards beta W (over T),
// beta U' (over X) and the blocked T^{-1} (over Y).
constexpr int kPrepThreads = 256;
constexpr size_t kPrepSmem =
    1024 + 5 * (size_t)umma::kTileBytes + 256 + kTdBytes + 6 * (size_t)kTileBytes;

// 16 values of row r (columns c0..c0+15) -> split bf16 tiles in the padded layout.
__device__ __forceinline__ void store_split16_padded(bf16* hi, bf16* lo, int r, int c0,
                                                     const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t ph[4], pl[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) tc::split_pack(v[8 * h + 2 * i], v[8 * h + 2 * i + 1], ph[i], pl[i]);
    *reinterpret_cast<uint4*>(hi + r * kLd + c0 + 8 * h) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
    *reinterpret_cast<uint4*>(lo + r * kLd + c0 + 8 * h) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
  }
}

__global__ void __launch_bounds__(kPrepThreads, 2) prep_kernel(const TcArgs<bf16> p) {
  namespace um = umma;
  extern __shared__ __align__(1024) unsigned char psmem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(psmem);  // [0] level 1, [1] levels 3-4 (two issuers)
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(psmem + 64);
  bf16* bt = reinterpret_cast<bf16*>(psmem + 1024);
  bf16 *K = bt, *Q = bt + 4096, *V = bt + 2 * 4096, *PH = bt + 3 * 4096, *PL = bt + 4 * 4096;
  float* bs = reinterpret_cast<float*>(bt + 5 * 4096);
  float* Td = bs + 64;
  bf16* R = reinterpret_cast<bf16*>(reinterpret_cast<unsigned char*>(Td) + kTdBytes);
  bf16 *TH = R, *TL = R + kTile, *XH = R + 2 * kTile, *XL = R + 3 * kTile, *YH = R + 4 * kTile,
       *YL = R + 5 * kTile;
  bf16 *BWH = TH, *BWL = TH + 4096, *BUH = XH, *BUL = XH + 4096, *TiH = YH, *TiL = YH + 4096;

  constexpr int NTH = kPrepThreads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hh = warp >> 2;
  const int c = blockIdx.x % p.nchunks;
  const long long bh = blockIdx.x / p.nchunks;
  const long long t0 = (long long)c * p.C;
  const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
  const long long r0 = t0 * p.nh, rows = p.T * p.nh;
  const long long blk = bh * p.nchunks + c;

  if (warp == 0) um::alloc(tbase_s, 256);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 2);
    mbar_fence_init();
  }
  zero_upper_blocks<NTH>(XH, XL);
  stage_blocked<NTH>(K, p.K + (bh * rows + r0) * p.dk, p.dk, Mc, p.dk >> 3);
  stage_blocked<NTH>(Q, p.Q + (bh * p.T + t0) * p.dk, p.dk, Cc, p.dk >> 3);
  stage_blocked<NTH>(V, p.V + (bh * rows + r0) * p.dv, p.dv, Mc, p.dv >> 3);
  cp_async_commit();
  if (tid < 64) bs[tid] = tid < Mc ? __bfloat162float(p.beta[bh * rows + r0 + tid]) : 0.f;
  cp_async_wait_all();
  // okw: every wait so far completed. After a wait that runs out (recorded in
  // the sticky word) the CTA issues no MMA, waits on nothing and writes no
  // output; to_mma makes the flag the same in every thread.
  bool okw = true;
  auto to_mma = [&]() {
    fence_proxy_async_smem();
    um::fence_before();
    okw = !__syncthreads_or(!okw);
    um::fence_after();
  };
  to_mma();
  const uint32_t tb = *tbase_s;
  const uint32_t tA = tb, tB = tb + 64, tC = tb + 128, tD = tb + 192;
  auto S_ = [](const bf16* t) { return um::saddr(t); };

  // level 1: [K; Q] K^T (K and Q are consecutive blocked tiles: one M = 128 operand)
  if (tid == 0) {
    const um::Prod ps[1] = {{tA, um::opnd(S_(K), 0, false), um::opnd(S_(K), 0, false), false, true}};
    um::products(ps);
    um::commit(bar);
  }
  okw = mbar_wait(bar, 0, &g_sticky_err);
  um::fence_after();
  {  // row r = 32 q + lane of the M = 128 accumulator: T row r (r < 64) or P~ row r - 64
    const int r = 32 * q + lane;
    const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + 32 * hh;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c0 = 32 * hh + 16 * half;
      float v[16];
      um::ld16(lb + 16 * half, v);
      if (r < 64) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = c0 + i < r ? v[i] * bs[c0 + i] : 0.f;
        if ((c0 >> 4) == (r >> 4))
#pragma unroll
          for (int i = 0; i < 16; ++i) Td[(r >> 4) * 272 + (r & 15) * 17 + i] = v[i];
        store_split16_padded(TH, TL, r, c0, v);
      } else {
        const int ti = r - 64;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = (c0 + i < (ti + 1) * p.nh && c0 + i < Mc) ? v[i] : 0.f;
        um::store_split16(PH, PL, ti, c0, v);
      }
    }
  }
  um::fence_before();
  okw = !__syncthreads_or(!okw);
  tri_inv_tc(Td, Op{TH, TL}, XH, XL, YH, YL);  // ends with __syncthreads
  for (int i = tid; i < 64 * 8; i += NTH) {  // padded X -> blocked T^{-1} (over Y)
    const int row = i >> 3, ch = i & 7;
    *reinterpret_cast<uint4*>(TiH + um::boff(row, ch * 8)) =
        *reinterpret_cast<const uint4*>(XH + row * kLd + ch * 8);
    *reinterpret_cast<uint4*>(TiL + um::boff(row, ch * 8)) =
        *reinterpret_cast<const uint4*>(XL + row * kLd + ch * 8);
  }
  to_mma();
  if (okw && tid == 64) {  // T^{-1} (blocked) to `saved` by bulk copies; Y is not reused until the end
    bulk_s2g(p.Ti + blk * kSavedSet<bf16>, TiH, um::kTileBytes);
    bulk_s2g(p.Ti + blk * kSavedSet<bf16> + 4096, TiL, um::kTileBytes);
    bulk_commit();
  }
  // level 3: W = Ti K (B), U' = Ti V (C)
  if (okw && (tid == 0 || tid == 32)) {
    const um::Prod ps[1] = {{tid == 0 ? tB : tC, um::opnd(S_(TiH), S_(TiL), false),
                             um::opnd(S_(tid == 0 ? K : V), 0, true), false}};
    um::products(ps);
    um::commit(bar + 1);
  }
  if (okw) okw = mbar_wait(bar + 1, 0, &g_sticky_err);
  um::fence_after();
  const int row = 16 * q + lane;  // M = 64 accumulators: lanes 0-15 hold rows
  const bool rv = lane < 16;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + 32 * hh;
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // beta W (over T), beta U' (over X)
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16];
    float w[16], u[16];
    um::ld16_async(lb + 64 + 16 * half, r1);
    um::ld16_async(lb + 128 + 16 * half, r2);
    um::ld_wait();
    um::ld_bind(r1, w);
    um::ld_bind(r2, u);
    if (rv) {
      const float b = bs[row];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        w[i] *= b;
        u[i] *= b;
      }
      um::store_split16(BWH, BWL, row, c0, w);
      um::store_split16(BUH, BUL, row, c0, u);
    }
  }
  to_mma();
  // level 4: K^T (beta W) (A), P~ (beta W) (B), K^T (beta U') (C), P~ (beta U') (D)
  if (okw && tid == 0) {
    const um::Opnd oBW = um::opnd(S_(BWH), S_(BWL), true);
    const um::Prod ps[2] = {{tA, um::opnd(S_(K), 0, true), oBW, false},
                            {tB, um::opnd(S_(PH), S_(PL), false), oBW, false}};
    um::products(ps);
    um::commit(bar + 1);
  } else if (okw && tid == 32) {
    const um::Opnd oBU = um::opnd(S_(BUH), S_(BUL), true);
    const um::Prod ps[2] = {{tC, um::opnd(S_(K), 0, true), oBU, false},
                            {tD, um::opnd(S_(PH), S_(PL), false), oBU, false}};
    um::products(ps);
    um::commit(bar + 1);
  }
  if (okw) okw = mbar_wait(bar + 1, 1, &g_sticky_err);
  um::fence_after();
  // Outputs are staged in shared memory no longer read by the MMAs and leave
  // by bulk copies: Xn h/l over T, Qt h/l over X (blocked, as the chains'
  // MMAs read them), Bc [dk][dv] fp32 over Y, Yp [C][dv] fp32 over V and P~.
  if (tid == 64) bulk_wait_read();  // the T^{-1} copies out of Y have read it
  okw = !__syncthreads_or(!okw);
  bf16 *XsH = TH, *XsL = TH + 4096, *QsH = XH, *QsL = XH + 4096;  // blocked
  float* Bcs = reinterpret_cast<float*>(YH);
  float* Yps = reinterpret_cast<float*>(V);
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // Xn, Qt (saved, padded), Bc, Yp (workspace, fp32)
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16], r3[16], r4[16];
    float x[16], qt[16], bc[16], yp[16];
    um::ld16_async(lb + 0 + 16 * half, r1);
    um::ld16_async(lb + 64 + 16 * half, r2);
    um::ld16_async(lb + 128 + 16 * half, r3);
    um::ld16_async(lb + 192 + 16 * half, r4);
    um::ld_wait();
    um::ld_bind(r1, x);
    um::ld_bind(r2, qt);
    um::ld_bind(r3, bc);
    um::ld_bind(r4, yp);
    if (rv) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        x[i] = -x[i];
        qt[i] = __bfloat162float(Q[um::boff(row, c0 + i)]) - qt[i];
      }
      um::store_split16(XsH, XsL, row, c0, x);
      um::store_split16(QsH, QsL, row, c0, qt);
      if (row < p.dk) row16_f32_to_global(Bcs + row * p.dv, c0, p.dv, bc);
      if (row < Cc) row16_f32_to_global(Yps + row * p.dv, c0, p.dv, yp);
    }
  }
  fence_proxy_async_smem();
  um::fence_before();
  __syncthreads();
  if (okw && tid == 0) {
    bulk_s2g(p.Xn + blk * kSavedSet<bf16>, XsH, 2 * um::kTileBytes);  // hi, lo contiguous
    bulk_s2g(p.Qt + blk * kSavedSet<bf16>, QsH, 2 * um::kTileBytes);
    bulk_s2g(p.Bc + blk * 4096, Bcs, (unsigned)(p.dk * p.dv * 4));
    bulk_s2g(p.Yp + blk * 4096, Yps, (unsigned)(Cc * p.dv * 4));
    bulk_commit();
    bulk_wait_read();  // shared memory stays valid until the copies have read it
  }
  if (warp == 0) {
    um::fence_after();
    um::dealloc(tb, 256);
  }
}

// ------------------------------------------------ forward: prep (fp32) --
// prep_kernel for fp32 inputs: the same products with every operand in three
// bf16 levels, and T^{-1} by substitution in fp32 on the CUDA cores
// (tri_inv_f32). One CTA per SM.
// smem: header | 15 blocked tiles: 0-5 the levels of [K; Q] interleaved
// (Kh Qh Km Qm Kl Ql, so each level is one M = 128 operand) | 6-8 V | 9-11 P~ |
// 12-14 T^{-1} | beta | Tf, Xf fp32 [64][65] | Ys fp32 [16][48].
// beta W goes over Q's levels, beta U' over V's; the outputs (Xn, Qt as
// blocked levels, Bc, Yp fp32) go from registers straight to global memory.
constexpr size_t kPrepF32Smem =
    1024 + 15 * (size_t)umma::kTileBytes + 256 + 2 * 64 * kF32Ld * 4 + 16 * 48 * 4 + 512;

template <bool DEC>
__global__ void __launch_bounds__(kPrepThreads, 1) prep_f32_kernel(const TcArgs<float> p) {
  namespace um = umma;
  extern __shared__ __align__(1024) unsigned char psmem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(psmem);  // [0] level 1, [1] levels 3-4 (two issuers)
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(psmem + 64);
  bf16* bt = reinterpret_cast<bf16*>(psmem + 1024);
  auto T = [&](int i) { return bt + i * 4096; };
  const Lv K = lv(T(0), T(2), T(4)), Q = lv(T(1), T(3), T(5)), V = lv(T(6), T(7), T(8));
  const Lv P = lv(T(9), T(10), T(11)), Ti = lv(T(12), T(13), T(14));
  const Lv &BW = Q, &BU = V;
  float* bs = reinterpret_cast<float*>(T(15));
  float* Tf = bs + 64;
  float* Xf = Tf + 64 * kF32Ld;
  float* Ys = Xf + 64 * kF32Ld;
  float* Pt = Ys + 16 * 48;  // decay: P_t (64), c_m (64)
  float* cm = Pt + 64;
  float* Ft = Xf;            // decay: span factor table, until the inverse
  const Lv Ks = lv(reinterpret_cast<bf16*>(Tf), reinterpret_cast<bf16*>(Tf) + 4096,
                   reinterpret_cast<bf16*>(Tf) + 8192);  // decay: P^ K (level 3), c K (level 4)

  constexpr int NTH = kPrepThreads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hh = warp >> 2;
  const int c = blockIdx.x % p.nchunks;
  const long long bh = blockIdx.x / p.nchunks;
  const long long t0 = (long long)c * p.C;
  const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
  const long long r0 = t0 * p.nh, rows = p.T * p.nh;
  const long long blk = bh * p.nchunks + c;
  const float inh = 1.f / (float)p.nh;

  if (warp == 0) um::alloc(tbase_s, 256);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 2);
    mbar_fence_init();
  }
  {
    const Lv xs[3] = {K, Q, V};
    const InSrc ss[3] = {{p.K + (bh * rows + r0) * p.dk, p.dk, Mc, p.dk >> 3},
                         {p.Q + (bh * p.T + t0) * p.dk, p.dk, Cc, p.dk >> 3},
                         {p.V + (bh * rows + r0) * p.dv, p.dv, Mc, p.dv >> 3}};
    stage_in_f32<NTH>(xs, ss);
  }
  if (tid < 64) bs[tid] = tid < Mc ? p.beta[bh * rows + r0 + tid] : 0.f;
  if constexpr (DEC) decay_tables(p.lg + bh * p.T + t0, Cc, p.nh, Ft, Pt, cm);
  // okw: every wait so far completed (as in prep_kernel).
  bool okw = true;
  auto to_mma = [&]() {
    fence_proxy_async_smem();
    um::fence_before();
    okw = !__syncthreads_or(!okw);
    um::fence_after();
  };
  to_mma();
  const uint32_t tb = *tbase_s;
  const uint32_t tA = tb, tB = tb + 64, tC = tb + 128, tD = tb + 192;

  // level 1: [K; Q] K^T, M = 128
  if (tid == 0) {
    const um::Prod ps[1] = {{tA, op(K, false), op(K, false), false, true}};
    um::products(ps);
    um::commit(bar);
  }
  okw = mbar_wait(bar, 0, &g_sticky_err);
  um::fence_after();
  {  // row r = 32 q + lane of the M = 128 accumulator: T row r (r < 64) or P~ row r - 64
    const int r = 32 * q + lane;
    const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + 32 * hh;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c0 = 32 * hh + 16 * half;
      float v[16];
      um::ld16(lb + 16 * half, v);
      if (r < 64) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x = c0 + i < r ? v[i] * bs[c0 + i] : 0.f;
          if constexpr (DEC) x *= c0 + i < r ? Ft[tok_of(r, inh) * kFLd + tok_of(c0 + i, inh)] : 0.f;
          Tf[r * kF32Ld + c0 + i] = x;
        }
      } else {
        const int ti = r - 64;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const bool rd = c0 + i < (ti + 1) * p.nh && c0 + i < Mc;
          v[i] = rd ? v[i] : 0.f;
          if constexpr (DEC) v[i] *= rd ? Ft[ti * kFLd + tok_of(c0 + i, inh)] : 0.f;
        }
        store16(P, ti, c0, v);
      }
    }
  }
  um::fence_before();
  okw = !__syncthreads_or(!okw);
  tri_inv_f32(Tf, Xf, Ys);  // ends with __syncthreads
  for (int i = tid; i < 64 * 8; i += NTH) {  // X -> blocked levels of T^{-1}
    const int row = i >> 3, ch = i & 7;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ch * 8 + j <= row ? Xf[row * kF32Ld + ch * 8 + j] : 0.f;
    store8(Ti, um::boff(row, ch * 8), v);
  }
  if constexpr (DEC) {  // P^ K over Tf / Xf (the inverse is done with them), from K's levels
    __syncthreads();
    scale_rows_levels<NTH>(Ks, K, Mc, Pt, inh);
  }
  to_mma();
  if (okw && tid == 64) {  // T^{-1} (three contiguous levels) to `saved`; its tiles stay untouched
    bulk_s2g(p.Ti + blk * kSavedSet<float>, Ti.t[0], 3 * um::kTileBytes);
    bulk_commit();
  }
  // level 3: W = Ti K (B) (decay: Ti (P^ K)), U' = Ti V (C)
  if (okw && (tid == 0 || tid == 32)) {
    const Lv& Kw = DEC ? Ks : K;
    const um::Prod ps[1] = {{tid == 0 ? tB : tC, op(Ti, false), op(tid == 0 ? Kw : V, true), false}};
    um::products(ps);
    um::commit(bar + 1);
  }
  if (okw) okw = mbar_wait(bar + 1, 0, &g_sticky_err);
  um::fence_after();
  const int row = 16 * q + lane;  // M = 64 accumulators: lanes 0-15 hold rows
  const bool rv = lane < 16;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + 32 * hh;
  if constexpr (DEC)  // c K over P^ K (level 3 has read it), from K's levels
    scale_rows_levels<NTH>(Ks, K, Mc, cm, 1.f);
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // beta W (over Q), beta U' (over V)
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16];
    float w[16], u[16];
    um::ld16_async(lb + 64 + 16 * half, r1);
    um::ld16_async(lb + 128 + 16 * half, r2);
    um::ld_wait();
    um::ld_bind(r1, w);
    um::ld_bind(r2, u);
    if (rv) {
      const float b = bs[row];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        w[i] *= b;
        u[i] *= b;
      }
      store16(BW, row, c0, w);
      store16(BU, row, c0, u);
    }
  }
  to_mma();
  // level 4: K^T (beta W) (A), P~ (beta W) (B), K^T (beta U') (C), P~ (beta U') (D)
  if (okw && tid == 0) {
    const um::Opnd oBW = op(BW, true);
    const um::Prod ps[2] = {{tA, op(DEC ? Ks : K, true), oBW, false}, {tB, op(P, false), oBW, false}};
    um::products(ps);
    um::commit(bar + 1);
  } else if (okw && tid == 32) {
    const um::Opnd oBU = op(BU, true);
    const um::Prod ps[2] = {{tC, op(DEC ? Ks : K, true), oBU, false}, {tD, op(P, false), oBU, false}};
    um::products(ps);
    um::commit(bar + 1);
  }
  float qv[2][16];  // Q row `row`, columns 32*hh.. (fp32, exact), fetched while the products run
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int c0 = 32 * hh + 16 * half;
    const float* qg = p.Q + (bh * p.T + t0 + row) * p.dk + c0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 a = rv && row < Cc && c0 + 4 * k < p.dk
                           ? __ldg(reinterpret_cast<const float4*>(qg + 4 * k))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      qv[half][4 * k] = a.x;
      qv[half][4 * k + 1] = a.y;
      qv[half][4 * k + 2] = a.z;
      qv[half][4 * k + 3] = a.w;
    }
  }
  if (okw) okw = mbar_wait(bar + 1, 1, &g_sticky_err);
  um::fence_after();
  okw = !__syncthreads_or(!okw);
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // Xn, Qt (saved), Bc, Yp (workspace, fp32)
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16], r3[16], r4[16];
    float x[16], qt[16], bc[16], yp[16];
    um::ld16_async(lb + 0 + 16 * half, r1);
    um::ld16_async(lb + 64 + 16 * half, r2);
    um::ld16_async(lb + 128 + 16 * half, r3);
    um::ld16_async(lb + 192 + 16 * half, r4);
    um::ld_wait();
    um::ld_bind(r1, x);
    um::ld_bind(r2, qt);
    um::ld_bind(r3, bc);
    um::ld_bind(r4, yp);
    if (rv) {
      const float pr = DEC ? (row < Cc ? Pt[row] : 0.f) : 1.f;  // P_t of token `row`
      const float pe = DEC ? Pt[Cc - 1] - 1.f : 0.f;             // P_{C-1} - 1 on Xn's diagonal
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        x[i] = -x[i] + (DEC && row == c0 + i && row < p.dk ? pe : 0.f);
        qt[i] = pr * qv[half][i] - qt[i];
      }
      // straight from registers to global memory (one CTA per SM: a bulk-copy
      // drain at the end would hold the SM): Xn, Qt as blocked levels
      if (okw) {
        bf16* xg = p.Xn + blk * kSavedSet<float>;
        bf16* qg = p.Qt + blk * kSavedSet<float>;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int o = um::boff(row, c0 + 8 * h);
          um::store_split8_3(xg, xg + 4096, xg + 8192, o, x + 8 * h);
          um::store_split8_3(qg, qg + 4096, qg + 8192, o, qt + 8 * h);
        }
        if (row < p.dk) row16_f32_to_global(p.Bc + blk * 4096 + row * p.dv, c0, p.dv, bc);
        if (row < Cc) row16_f32_to_global(p.Yp + blk * 4096 + row * p.dv, c0, p.dv, yp);
      }
    }
  }
  um::fence_before();
  __syncthreads();
  if (tid == 64) bulk_wait_read();  // the T^{-1} copy has read its tiles
  if (warp == 0) {
    um::fence_after();
    um::dealloc(tb, 256);
  }
}

// The chunk-serial kernels: one CTA per (b, h, 32 value columns), 8 warps.
// Thread (warp w, lane l < 16) owns row 16*(w%4) + l and columns 16*(w/4)..+15
// of the CTA's state slice, in fp32 registers; the slice is also kept in
// shared memory as blocked bf16 levels (64 x 32 each), the B operand of the
// chunk's MMAs. Per chunk, thread 0 issues the state product and thread 32
// the other product (N = 32) into TMEM; all threads then add them to the state
// and write its new levels. The Xn, Qt levels of the next kRing - 1 chunks are
// staged by bulk copies.
constexpr int kChainThreads = 256;
constexpr int kChainCols = 32;
constexpr int kSTile = 64 * kChainCols * 2;  // one level of a 64 x 32 slice, bytes

// 16 fp32 values at g[0..15] -> v (chunks of 8 starting below `valid`; others 0).
__device__ __forceinline__ void load16_f32(const float* g, int c0, int valid, bool ok, float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (ok && c0 + 8 * h < valid) {
      a = *reinterpret_cast<const float4*>(g + 8 * h);
      b = *reinterpret_cast<const float4*>(g + 8 * h + 4);
    }
    v[8 * h] = a.x; v[8 * h + 1] = a.y; v[8 * h + 2] = a.z; v[8 * h + 3] = a.w;
    v[8 * h + 4] = b.x; v[8 * h + 5] = b.y; v[8 * h + 6] = b.z; v[8 * h + 7] = b.w;
  }
}
__device__ __forceinline__ void store16_f32(float* g, int c0, int valid, const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    if (c0 + 8 * h < valid) {
      *reinterpret_cast<float4*>(g + 8 * h) = make_float4(v[8 * h], v[8 * h + 1], v[8 * h + 2], v[8 * h + 3]);
      *reinterpret_cast<float4*>(g + 8 * h + 4) = make_float4(v[8 * h + 4], v[8 * h + 5], v[8 * h + 6], v[8 * h + 7]);
    }
}
// 16 values -> the output row (bf16 or fp32; chunks of 8 starting below `valid`)
__device__ __forceinline__ void store16_out(bf16* g, int c0, int valid, const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    if (c0 + 8 * h < valid) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = tc::pack_bf16(v[8 * h + 2 * i], v[8 * h + 2 * i + 1]);
      *reinterpret_cast<uint4*>(g + 8 * h) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}
__device__ __forceinline__ void store16_out(float* g, int c0, int valid, const float (&v)[16]) {
  store16_f32(g, c0, valid, v);
}

// ------------------------------------------------------ forward: chain --
//   S_c saved;  y_c = Qt S_c + Yp;  S_{c+1} = S_c + Xn S_c + Bc
// Both products share the state operand, so [Xn; Qt] is staged as one
// M = 128 operand per level (Xn hi, Qt hi, Xn lo, Qt lo[, Xn lo2, Qt lo2])
// and one thread issues 12 (bf16 inputs) or 24 (fp32) MMAs per chunk.
// Accumulator row r sits in TMEM lane r: warps 0, 1, 4, 5 (rows 0-63) own the
// state S, warps 2, 3, 6, 7 (rows 64-127) the output y; lane l of warp w has
// row 32*(w%4) + l, columns 16*(w/4)..+15.
// stage: the levels of [Xn; Qt] (bulk copies) and every thread's 16 additive
// terms (Bc or Yp; cp.async) as float4 [4][thread]
constexpr int kCfAddend = 4 * kChainThreads * 16;
template <typename E>
constexpr int kCfStage = 2 * kLevels<E> * umma::kTileBytes + kCfAddend;
template <typename E>
constexpr size_t kChainFwdSmem = 1024 + kRing * (size_t)kCfStage<E> + kLevels<E> * (size_t)kSTile;

template <typename E>
__global__ void __launch_bounds__(kChainThreads, 1) chain_fwd_kernel(const TcArgs<E> p) {
  namespace um = umma;
  constexpr int L = kLevels<E>;
  extern __shared__ __align__(1024) unsigned char csmem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(csmem);
  uint64_t* mbar = full + kRing;  // MMA completion
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(csmem + 64);
  unsigned char* ring = csmem + 1024;
  bf16* S0 = reinterpret_cast<bf16*>(ring + kRing * kCfStage<E>);
  const Lv Sl = lv(S0, S0 + 64 * kChainCols, L > 2 ? S0 + 2 * 64 * kChainCols : nullptr);
  auto Xt = [&](int s) { return reinterpret_cast<bf16*>(ring + s * kCfStage<E>); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = warp & 3;
  const int cb = 16 * (warp >> 2);
  const bool st = q < 2;                 // state thread (row r of S) or output thread (row r of y)
  const int r = 32 * (q & 1) + lane;     // row within S (state) or within the chunk's tokens (y)
  const int split = blockIdx.x % p.S;
  const long long bh = blockIdx.x / p.S;
  const int c0 = split * kChainCols, ncols = min(kChainCols, p.dv - c0);
  const long long blk0 = bh * p.nchunks;
  E* yg = p.y + bh * p.T * p.dv + c0 + cb;
  float* Hsg = p.Hs + blk0 * p.dk * p.dv + r * p.dv + c0 + cb;
  const bool srow = st && r < p.dk;

  auto stage = [&](int c) {
    bf16* X = Xt(c % kRing);
    if (tid == 0) {
      uint64_t* bar = full + c % kRing;
      const long long blk = blk0 + c;
      mbar_arrive_expect_tx(bar, 2 * L * umma::kTileBytes);
#pragma unroll
      for (int l = 0; l < L; ++l) {
        bulk_g2s(X + 8192 * l, p.Xn + blk * kSavedSet<E> + 4096 * l, umma::kTileBytes, bar);
        bulk_g2s(X + 8192 * l + 4096, p.Qt + blk * kSavedSet<E> + 4096 * l, umma::kTileBytes, bar);
      }
    }
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0);
    float4* ad = reinterpret_cast<float4*>(X + 8192 * L);
    const bool ok = st ? srow : r < Cc;
    const float* g = (st ? p.Bc : p.Yp) + (blk0 + c) * 4096 + r * p.dv + c0 + cb;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool v = ok && cb + 4 * j < ncols;
      cp_async16(ad + j * kChainThreads + tid, v ? g + 4 * j : p.Bc, v ? 16 : 0);
    }
    cp_async_commit();
  };

  if (warp == 0) um::alloc(tbase_s, 32);
  if (tid == 0) {
    for (int s = 0; s < kRing; ++s) mbar_init(full + s, 1);
    mbar_init(mbar, 1);
    mbar_fence_init();
  }
  float hs[16];  // state threads: S row r, columns cb..cb+15 of the slice
  load16_f32(p.H0 + bh * p.dk * p.dv + r * p.dv + c0 + cb, cb, ncols, p.H0 != nullptr && srow, hs);
  if (st) store16_n(Sl, r, cb, kChainCols, kChainCols, hs);
  um::fence_before();
  __syncthreads();
  um::fence_after();
  const uint32_t tb = *tbase_s;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + cb;
  const um::Opnd oS = op_mn(Sl, kChainCols);
  for (int c = 0; c < kRing - 1 && c < p.nchunks; ++c) stage(c);
  if (srow) store16_f32(Hsg, cb, ncols, hs);

  // okw: every wait so far completed. A wait that runs out (recorded in the
  // sticky word) ends the chunk loop in every thread at the next barrier; the
  // CTA then drains the copies it has in flight and writes nothing more.
  bool okw = true;
  int c = 0;
  for (; c < p.nchunks; ++c) {
    const int s = c % kRing;
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0);
    if (c + 1 < p.nchunks)  // the group of chunk c + 1 may still be in flight
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else
      cp_async_wait_all();
    if (okw) okw = mbar_wait(full + s, (unsigned)(c / kRing) & 1u, &g_sticky_err);
    fence_proxy_async_smem();  // the state levels written below in the previous chunk
    um::fence_before();
    // every thread is past chunk c - 1: its stage may be refilled
    if (__syncthreads_or(!okw)) {
      okw = false;
      break;
    }
    um::fence_after();
    if (c + kRing - 1 < p.nchunks) stage(c + kRing - 1);
    const float4* ad = reinterpret_cast<const float4*>(Xt(s) + 8192 * L);
    if (tid == 0) {  // [Xn; Qt] S, M = 128
      const uint32_t X = um::saddr(Xt(s));
      const um::Prod ps[1] = {
          {tb, um::opnd3(X, X + 16384, L > 2 ? X + 32768 : 0u, false), oS, false, true, kChainCols}};
      um::products(ps);
      um::commit(mbar);
    }
    okw = mbar_wait(mbar, (unsigned)c & 1u, &g_sticky_err);
    um::fence_after();
    if (!okw) continue;  // the loop ends at the next chunk's barrier
    float v[16];
    um::ld16(lb, v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 a4 = ad[j * kChainThreads + tid];
      v[4 * j] += a4.x;
      v[4 * j + 1] += a4.y;
      v[4 * j + 2] += a4.z;
      v[4 * j + 3] += a4.w;
    }
    if (st) {
#pragma unroll
      for (int i = 0; i < 16; ++i) hs[i] += v[i];
      store16_n(Sl, r, cb, kChainCols, kChainCols, hs);
      if (srow && c + 1 < p.nchunks) store16_f32(Hsg + (long long)(c + 1) * p.dk * p.dv, cb, ncols, hs);
    } else if (r < Cc) {
      store16_out(yg + (t0 + r) * p.dv, cb, ncols, v);
    }
  }
  if (!okw) {  // drain: the stages of chunks c .. c + kRing - 2 may still be in flight
    cp_async_wait_all();
    if (tid == 0)
      for (int j = c; j < c + kRing - 1 && j < p.nchunks; ++j)
        (void)mbar_wait(full + j % kRing, (unsigned)(j / kRing) & 1u, &g_sticky_err);
  } else if (srow) {
    store16_f32(p.HT + bh * p.dk * p.dv + r * p.dv + c0 + cb, cb, ncols, hs);
  }
  um::fence_before();
  __syncthreads();
  if (warp == 0) {
    um::fence_after();
    um::dealloc(tb, 32);
  }
}

// ----------------------------------------------------- backward: chain --
//   dS'_c (= dS entering from chunk c + 1) saved;  dS_c = dS'_c + Xn^T dS'_c + Qt^T dy_c
// stage: Xn levels, Qt levels (bulk copies), then dy: bf16 inputs as a blocked
// 64 x 32 tile (cp.async); fp32 inputs as raw rows [64][32] (cp.async, 8
// columns per thread), split into three levels by the thread that copied them
// once its copies have landed.
template <typename E>
constexpr int kCbStage = 2 * kLevels<E> * umma::kTileBytes + (kF32<E> ? 64 * kChainCols * 4 : kSTile);
template <typename E>
constexpr size_t kChainBwdSmem = 1024 + kRing * (size_t)kCbStage<E> + kLevels<E> * (size_t)kSTile +
                                 (kF32<E> ? 3 * (size_t)kSTile : 0);

template <typename E>
__global__ void __launch_bounds__(kChainThreads, 1) chain_bwd_kernel(const TcArgs<E> p) {
  namespace um = umma;
  constexpr bool F = kF32<E>;
  constexpr int L = kLevels<E>;
  extern __shared__ __align__(1024) unsigned char csmem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(csmem);
  uint64_t* mbar = full + kRing;
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(csmem + 64);
  unsigned char* ring = csmem + 1024;
  bf16* D0 = reinterpret_cast<bf16*>(ring + kRing * kCbStage<E>);
  const Lv Dl = lv(D0, D0 + 64 * kChainCols, L > 2 ? D0 + 2 * 64 * kChainCols : nullptr);
  bf16* Y0 = D0 + L * 64 * kChainCols;  // fp32 inputs: dy levels of the current step
  const Lv Yl = lv(Y0, Y0 + 64 * kChainCols, Y0 + 2 * 64 * kChainCols);
  auto Xt = [&](int s) { return reinterpret_cast<bf16*>(ring + s * kCbStage<E>); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = warp & 3;
  const int row = 16 * q + lane, cb = 16 * (warp >> 2);
  const bool rv = lane < 16;
  const int split = blockIdx.x % p.S;
  const long long bh = blockIdx.x / p.S;
  const int c0 = split * kChainCols, ncols = min(kChainCols, p.dv - c0);
  const long long blk0 = bh * p.nchunks;
  const E* dyg = p.dy + bh * p.T * p.dv + c0;
  float* dHsg = p.dHs + blk0 * p.dk * p.dv + row * p.dv + c0 + cb;
  const bool srow = rv && row < p.dk;
  const int last = p.nchunks - 1;
  const int yr = tid >> 2, ych = tid & 3;  // dy staging: 64 rows x 4 chunks of 8 columns

  // step qq handles chunk last - qq in ring slot qq % kRing
  auto stage = [&](int qq) {
    const int c = last - qq;
    bf16* X = Xt(qq % kRing);
    if (tid == 0) {
      uint64_t* bar = full + qq % kRing;
      const long long blk = blk0 + c;
      mbar_arrive_expect_tx(bar, 2 * L * umma::kTileBytes);
      bulk_g2s(X, p.Xn + blk * kSavedSet<E>, L * umma::kTileBytes, bar);
      bulk_g2s(X + 4096 * L, p.Qt + blk * kSavedSet<E>, L * umma::kTileBytes, bar);
    }
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0);
    const bool ok = yr < Cc && 8 * ych < ncols;
    const E* src = dyg + (t0 + yr) * p.dv + 8 * ych;
    if constexpr (F) {
      float* raw = reinterpret_cast<float*>(X + 8192 * L) + yr * kChainCols + 8 * ych;
      cp_async16(raw, ok ? src : dyg, ok ? 16 : 0);
      cp_async16(raw + 4, ok ? src + 4 : dyg, ok ? 16 : 0);
    } else {
      bf16* dY = X + 8192 * L;
      cp_async16(dY + um::boff_n(yr, 8 * ych, kChainCols), ok ? src : dyg, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  if (warp == 0) um::alloc(tbase_s, 64);
  if (tid == 0) {
    for (int s = 0; s < kRing; ++s) mbar_init(full + s, 1);
    mbar_init(mbar, 2);
    mbar_fence_init();
  }
  float ds[16];
  load16_f32(p.dHT + bh * p.dk * p.dv + row * p.dv + c0 + cb, cb, ncols, p.dHT != nullptr && srow, ds);
  if (rv) store16_n(Dl, row, cb, kChainCols, kChainCols, ds);
  um::fence_before();
  __syncthreads();
  um::fence_after();
  const uint32_t tb = *tbase_s, tX = tb, tY = tb + 32;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + cb;
  for (int qq = 0; qq < kRing - 1 && qq <= last; ++qq) stage(qq);
  if (srow) store16_f32(dHsg + (long long)last * p.dk * p.dv, cb, ncols, ds);
  const um::Opnd oD = op_mn(Dl, kChainCols);

  // okw: as in chain_fwd_kernel (a wait that runs out ends the loop in every
  // thread at the next barrier, then the CTA drains its copies and stops).
  bool okw = true;
  int qq = 0;
  for (; qq <= last; ++qq) {
    const int c = last - qq, s = qq % kRing;
    if (qq < last)  // the group of step qq + 1 may still be in flight
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else
      cp_async_wait_all();
    if constexpr (F) {  // this thread's dy copies have landed: split them into levels
      const float* raw = reinterpret_cast<const float*>(Xt(s) + 8192 * L) + yr * kChainCols + 8 * ych;
      const float4 a = *reinterpret_cast<const float4*>(raw);
      const float4 b = *reinterpret_cast<const float4*>(raw + 4);
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      store8(Yl, um::boff_n(yr, 8 * ych, kChainCols), v);
    }
    if (okw) okw = mbar_wait(full + s, (unsigned)(qq / kRing) & 1u, &g_sticky_err);
    fence_proxy_async_smem();  // dy and the dS levels written in the previous step
    um::fence_before();
    if (__syncthreads_or(!okw)) {
      okw = false;
      break;
    }
    um::fence_after();
    if (qq + kRing - 1 <= last) stage(qq + kRing - 1);
    const uint32_t X = um::saddr(Xt(s));
    if (tid == 0) {  // Xn^T dS'
      const um::Prod ps[1] = {{tX, um::opnd3(X, X + 8192, L > 2 ? X + 16384 : 0u, true), oD, false,
                               false, kChainCols}};
      um::products(ps);
      um::commit(mbar);
    } else if (tid == 32) {  // Qt^T dy
      const uint32_t Qa = X + 8192 * L;
      const um::Opnd oY = F ? op_mn(Yl, kChainCols) : um::opnd_mn(X + 16384 * L, 0, kChainCols);
      const um::Prod ps[1] = {{tY, um::opnd3(Qa, Qa + 8192, L > 2 ? Qa + 16384 : 0u, true), oY,
                               false, false, kChainCols}};
      um::products(ps);
      um::commit(mbar);
    }
    okw = mbar_wait(mbar, (unsigned)qq & 1u, &g_sticky_err);
    um::fence_after();
    if (!okw) continue;  // the loop ends at the next step's barrier
    uint32_t rx[16], ry[16];
    float xs[16], ys[16];
    um::ld16_async(lb, rx);
    um::ld16_async(lb + 32, ry);
    um::ld_wait();
    um::ld_bind(rx, xs);
    um::ld_bind(ry, ys);
    if (rv) {
#pragma unroll
      for (int i = 0; i < 16; ++i) ds[i] += xs[i] + ys[i];
      store16_n(Dl, row, cb, kChainCols, kChainCols, ds);
    }
    if (srow && c > 0) store16_f32(dHsg + (long long)(c - 1) * p.dk * p.dv, cb, ncols, ds);
  }
  if (!okw) {  // drain: the stages of steps qq .. qq + kRing - 2 may still be in flight
    cp_async_wait_all();
    if (tid == 0)
      for (int j = qq; j < qq + kRing - 1 && j <= last; ++j)
        (void)mbar_wait(full + j % kRing, (unsigned)(j / kRing) & 1u, &g_sticky_err);
  } else if (srow) {
    store16_f32(p.dH0 + bh * p.dk * p.dv + row * p.dv + c0 + cb, cb, ncols, ds);
  }
  um::fence_before();
  __syncthreads();
  if (warp == 0) {
    um::fence_after();
    um::dealloc(tb, 64);
  }
}

// ---------------------------------------------------------------- host --

template <class K, class A>
int launch_tc(K kernel, long long grid, size_t smem, cudaStream_t st, const A& a, int threads) {
  MGS_CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  A args = a;
  void* kargs[] = {&args};
  MGS_CUDA_OK(cudaLaunchKernel((const void*)kernel, dim3((unsigned)grid), dim3(threads), kargs,
                               smem, st));
  return MGS_OK;
}

template <typename E>
int run_tc_impl(bool fwd, const Args<E>& p, long long B, int H, long long T, int nh, int dk, int dv,
                int C, float* saved, void* ws, size_t ws_bytes, cudaStream_t st) {
  const long long BH = B * (long long)H;
  TcArgs<E> a{};
  a.Q = p.Q;
  a.K = p.K;
  a.V = p.V;
  a.beta = p.beta;
  a.H0 = p.H0;
  a.y = p.y;
  a.HT = p.HT;
  a.dy = p.dy;
  a.dHT = p.dHT;
  a.dQ = p.dQ;
  a.dK = p.dK;
  a.dV = p.dV;
  a.dbeta = p.dbeta;
  a.dH0 = p.dH0;
  a.lg = p.lg;
  a.dlg = p.dlg;
  if (a.lg != nullptr && (!kF32<E> || (!fwd && a.dlg == nullptr))) return MGS_UNSUPPORTED;
  a.T = T;
  a.nh = nh;
  a.dk = dk;
  a.dv = dv;
  a.C = C;
  a.nchunks = (int)((T + C - 1) / C);
  a.S = (dv + kChainCols - 1) / kChainCols;  // chain kernels: 32 value columns per CTA
  a.dvs = kChainCols;
  if (BH == 0) return MGS_OK;
  if (saved == nullptr) return MGS_BAD_SHAPE;
  const size_t ncs = (size_t)BH * a.nchunks;
  a.Hs = saved;
  a.Ti = reinterpret_cast<bf16*>(saved + ncs * dk * dv);
  a.Xn = a.Ti + ncs * kSavedSet<E>;
  a.Qt = a.Xn + ncs * kSavedSet<E>;
  if (T > 0 && (ws == nullptr || ws_bytes < tc_workspace_floats(BH, T, dk, dv, C) * sizeof(float)))
    return MGS_WORKSPACE_TOO_SMALL;
  if (fwd) {
    if (T == 0) {
      if (p.H0)
        MGS_CUDA_OK(cudaMemcpyAsync(p.HT, p.H0, (size_t)BH * dk * dv * sizeof(float),
                                    cudaMemcpyDeviceToDevice, st));
      else
        MGS_CUDA_OK(cudaMemsetAsync(p.HT, 0, (size_t)BH * dk * dv * sizeof(float), st));
      return MGS_OK;
    }
    a.Bc = static_cast<float*>(ws);
    a.Yp = a.Bc + ncs * 4096;
    int rc;
    if constexpr (kF32<E>)
      rc = a.lg ? launch_tc(prep_f32_kernel<true>, (long long)ncs, kPrepF32Smem, st, a, kPrepThreads)
                : launch_tc(prep_f32_kernel<false>, (long long)ncs, kPrepF32Smem, st, a, kPrepThreads);
    else
      rc = launch_tc(prep_kernel, (long long)ncs, kPrepSmem, st, a, kPrepThreads);
    if (rc != MGS_OK) return rc;
    return launch_tc(chain_fwd_kernel<E>, BH * a.S, kChainFwdSmem<E>, st, a, kChainThreads);
  }
  if (T == 0) {
    if (p.dHT)
      MGS_CUDA_OK(cudaMemcpyAsync(p.dH0, p.dHT, (size_t)BH * dk * dv * sizeof(float),
                                  cudaMemcpyDeviceToDevice, st));
    else
      MGS_CUDA_OK(cudaMemsetAsync(p.dH0, 0, (size_t)BH * dk * dv * sizeof(float), st));
    return MGS_OK;
  }
  a.dHs = static_cast<float*>(ws);
  int rc = launch_tc(chain_bwd_kernel<E>, BH * a.S, kChainBwdSmem<E>, st, a, kChainThreads);
  if (rc != MGS_OK) return rc;
  if constexpr (kF32<E>)
    if (a.lg)
      return launch_tc(bwd_grads_kernel<E, true>, BH * a.nchunks, kGradSmem<E> + kGradDecaySmem, st,
                       a, kGradThreads);
  return launch_tc(bwd_grads_kernel<E>, BH * a.nchunks, kGradSmem<E>, st, a, kGradThreads);
}

}  // namespace

bool tc_eligible(int dtype, int nh, int dk, int dv, int C) {
  return (dtype == MGS_BF16 || dtype == MGS_F32) && nh >= 1 && C >= 1 && nh * C <= 64 && dk >= 8 &&
         dk <= 64 && dv >= 8 && dv <= 64 && dk % 8 == 0 && dv % 8 == 0;
}

// saved: chunk-start states (fp32), then every chunk's T^{-1}, Xn and Qt
// (bf16 levels -- two for bf16 inputs, three for fp32 -- in the tcgen05
// blocked layout)
size_t tc_saved_floats(long long BH, long long T, int dk, int dv, int C, int dtype) {
  const size_t nc = (size_t)BH * (size_t)((T + C - 1) / C);
  const size_t set = dtype == MGS_F32 ? (size_t)kSavedSet<float> : (size_t)kSavedSet<bf16>;
  return nc * dk * dv + 3 * nc * set / 2;
}

// forward: Bc and Yp (4096 floats each per chunk); backward: dS' per chunk
size_t tc_workspace_floats(long long BH, long long T, int dk, int dv, int C) {
  const size_t nc = (size_t)BH * (size_t)((T + C - 1) / C);
  const size_t bwd = nc * dk * dv, fwd = 2 * nc * 4096;
  return fwd > bwd ? fwd : bwd;
}

int run_tc(bool fwd, const Args<__nv_bfloat16>& p, long long B, int H, long long T, int nh, int dk,
           int dv, int C, float* saved, void* ws, size_t ws_bytes, cudaStream_t st) {
  return run_tc_impl(fwd, p, B, H, T, nh, dk, dv, C, saved, ws, ws_bytes, st);
}
int run_tc(bool fwd, const Args<float>& p, long long B, int H, long long T, int nh, int dk, int dv,
           int C, float* saved, void* ws, size_t ws_bytes, cudaStream_t st) {
  return run_tc_impl(fwd, p, B, H, T, nh, dk, dv, C, saved, ws, ws_bytes, st);
}

}  // namespace delta

// The tensor-core kernels' sticky error word (bounded mbarrier waits that ran
// out); read and cleared through mgs_take_device_error.
unsigned take_error_delta_tc(cudaStream_t s) { return take_sticky_error(s); }

}  // namespace mgs
