// delta_tc.cu -- DeltaMinGRU chunked-WY delta rule on the tensor cores (bf16
// inputs, fp32 state and accumulation).
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
// Kernels (all 64 x 64 chunk products are bf16 mma.sync with split hi/lo
// operands, mma_bf16.cuh; Ti by blocked substitution in fp32):
//   fwd_kernel        one CTA per (b, h, value-column split): walks the chunks
//                     in order with the state slice in registers; writes y,
//                     H_T and every chunk-start state (saved for the backward).
//   bwd_chain_kernel  one CTA per (b, h, split): walks the chunks in reverse,
//                     carrying dS; writes dS' of every chunk and dH0.
//   bwd_grads_kernel  one CTA per (b, h, chunk): every gradient of the chunk
//                     from its saved S and dS'.
// Inputs are staged with cp.async (next chunk prefetched during the current
// one in the two chunk-serial kernels); out-of-range rows and columns are
// zero-filled, which makes every padded product exact (a zero K row gives an
// identity row of T, a zero U row and no state update).
#include "delta_args.cuh"
#include "mma_bf16.cuh"

namespace mgs {
namespace delta {
namespace {

using bf16 = __nv_bfloat16;
using tc::kLd;
using tc::Op;

constexpr int kTcThreads = 256;
constexpr int kTile = 64 * kLd;            // bf16 elements of one 64 x 64 tile
constexpr int kTileBytes = kTile * 2;      // 9216
constexpr int kTld = 66;                   // fp32 leading dimension of T / T^{-1}
constexpr int kF32Bytes = 64 * kTld * 4;   // 16896
constexpr int kStageBytes = 3 * kTileBytes + 256;  // 3 tiles + beta[64] (fp32)

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

__device__ __forceinline__ int up16(int x) { return (x + 15) & ~15; }

// 64 rows x (NCH * 8 columns) bf16 block of a row-major global matrix (leading
// dimension ld elements) into a tile; rows >= nrows / chunks >= ncols8 zero.
template <int NCH, int NTHR = kTcThreads>
__device__ __forceinline__ void stage_rows(bf16* tile, const bf16* g, long long ld, int nrows,
                                           int valid_ch) {
  for (int i = threadIdx.x; i < 64 * NCH; i += NTHR) {
    const int row = i / NCH, ch = i - row * NCH;
    const bool ok = row < nrows && ch < valid_ch;
    cp_async16(tile + row * kLd + ch * 8, ok ? g + row * ld + ch * 8 : g, ok ? 16 : 0);
  }
}

struct Ident {
  __device__ float operator()(int, int, float x) const { return x; }
};
struct Neg {
  __device__ float operator()(int, int, float x) const { return -x; }
};

// Ti = T^{-1} for the unit lower-triangular T = I + strict_lower(T) of a chunk,
// as split bf16 tiles (X). Inputs: the strictly-lower part of T as split tiles
// (TS) and in fp32 (Tf, only its four diagonal 16 x 16 blocks are read).
//   1. diagonal blocks D_b^{-1} by forward substitution (one thread per column)
//   2. X_10 = -D_1^{-1} T_10 D_0^{-1} and X_32 = -D_3^{-1} T_32 D_2^{-1} (warps 0, 1)
//   3. X[32:64, 0:32] = -X[32:64, 32:64] (T[32:64, 0:32] X[0:32, 0:32])  (warps 0-3)
// with every block product on the tensor cores (split operands, fp32 accumulate).
// X's strictly-upper 16 x 16 blocks must be zero on entry (they are never
// written); Y is scratch (two tiles).
__device__ void tri_inv_tc(const float* Tf, Op TS, bf16* XH, bf16* XL, bf16* YH, bf16* YL) {
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid < 64) {
    const int o = (tid >> 4) * 16, j = tid & 15;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < i; ++k) s = fmaf(Tf[(o + i) * kTld + o + k], x[k], s);
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

// 64 x 64 bf16 tile <-> dense global 64 x 64 (16-byte vectors, all threads).
template <int NTHR = kTcThreads>
__device__ __forceinline__ void tile_to_global(const bf16* t, bf16* g) {
  for (int i = threadIdx.x; i < 64 * 8; i += NTHR) {
    const int row = i >> 3, ch = i & 7;
    *reinterpret_cast<uint4*>(g + row * 64 + ch * 8) =
        *reinterpret_cast<const uint4*>(t + row * kLd + ch * 8);
  }
}
template <int NTHR = kTcThreads>
__device__ __forceinline__ void tile_from_global_async(bf16* t, const bf16* g) {
  for (int i = threadIdx.x; i < 64 * 8; i += NTHR) {
    const int row = i >> 3, ch = i & 7;
    cp_async16(t + row * kLd + ch * 8, g + row * 64 + ch * 8, 16);
  }
}


// c[nt] tile rows m0, cols n0 (fragment layout) -> fp32 global matrix (ld),
// rows < nrows, cols < ncols.
template <int NT>
__device__ __forceinline__ void frag_to_global(const float (&c)[NT][4], float* g, long long ld,
                                               int m0, int n0, int nrows, int ncols) {
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = tc::frag_row(m0, 2 * h), col = tc::frag_col(n0, j, 0);
      if (row < nrows && col < ncols)
        *reinterpret_cast<float2*>(g + row * ld + col) = make_float2(c[j][2 * h], c[j][2 * h + 1]);
    }
}

template <int NT>
__device__ __forceinline__ void frag_to_global_bf16(const float (&c)[NT][4], bf16* g, long long ld,
                                                    int m0, int n0, int nrows, int ncols) {
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = tc::frag_row(m0, 2 * h), col = tc::frag_col(n0, j, 0);
      if (row < nrows && col < ncols)
        *reinterpret_cast<uint32_t*>(g + row * ld + col) = tc::pack_bf16(c[j][2 * h], c[j][2 * h + 1]);
    }
}

template <int NT>
__device__ __forceinline__ void frag_from_global(float (&c)[NT][4], const float* g, long long ld,
                                                 int m0, int n0, int nrows, int ncols) {
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = tc::frag_row(m0, 2 * h), col = tc::frag_col(n0, j, 0);
      float2 v = make_float2(0.f, 0.f);
      if (row < nrows && col < ncols) v = *reinterpret_cast<const float2*>(g + row * ld + col);
      c[j][2 * h] = v.x;
      c[j][2 * h + 1] = v.y;
    }
}

// ---- chunk matrices from K K^T and Q K^T (exact bf16 products, fp32 sums).
// Warp w: row tile w & 3; warps 0-3 one product, warps 4-7 the other.

// P = (Q K^T) diag(beta) * read  as split tiles (NT n-tiles at columns n0..)
template <int NT>
__device__ __forceinline__ void store_P(const float (&acc)[NT][4], const float* bs, int nh, int Mc,
                                        int m0, int n0, bf16* PH, bf16* PL) {
  tc::store_split(acc, PH, PL, m0, n0, [&](int r, int cl, float x) {
    return (cl < (r + 1) * nh && cl < Mc) ? x * bs[cl] : 0.f;
  });
}

// T's strict lower part (K K^T diag(beta)) as fp32 (diagonal blocks) and split tiles.
template <int NT>
__device__ __forceinline__ void store_T(const float (&acc)[NT][4], const float* bs, int m0, int n0,
                                        float* Tf, bf16* TH, bf16* TL) {
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int row = tc::frag_row(m0, v), col = tc::frag_col(n0, j, v);
      if ((col >> 4) == (row >> 4)) Tf[row * kTld + col] = col < row ? acc[j][v] * bs[col] : 0.f;
    }
  tc::store_split(acc, TH, TL, m0, n0,
                  [&](int r, int cl, float x) { return cl < r ? x * bs[cl] : 0.f; });
}

struct TcArgs {
  const bf16* Q;
  const bf16* K;
  const bf16* V;
  const bf16* beta;
  const float* H0;
  bf16* y;
  float* HT;
  const bf16* dy;
  const float* dHT;
  bf16* dQ;
  bf16* dK;
  bf16* dV;
  bf16* dbeta;
  float* dH0;
  float* Hs;    // (BH, nchunks, dk, dv) chunk-start states
  bf16* Ti;     // (BH, nchunks, 2, 64, 64) T^{-1} of every chunk, split hi / lo
  float* dHs;   // (BH, nchunks, dk, dv) gradient of each chunk's output state
  long long T;
  int nh, dk, dv, C, nchunks, S, dvs;
};

// ------------------------------------------------------------ forward --
// smem: 2 stages {K, Q, V_s, beta} | Ti h/l | W h/l (inverse scratch first) |
//       P h/l | S h/l | U h/l (T fp32 first) | bU h/l (T split first)
constexpr size_t kFwdSmem = 2 * kStageBytes + 12 * (size_t)kTileBytes;
constexpr int kSerialThreads = 512;  // 16 warps: warp (mt, q) = (w & 3, w >> 2)

// Warp tiling of the chunk-serial kernels: rows 16*mt; 64-wide products in
// 16-column quarters (q), the DVS value columns in quarters of DVS/4, and the
// two masked K K^T / Q K^T products as (matrix q >> 1, 32-column half q & 1).
template <int DVS>
__global__ void __launch_bounds__(kSerialThreads, 1) fwd_kernel(const TcArgs p) {
  constexpr int NTQ = DVS / 32;  // n-tiles of a warp's quarter of the value columns
  constexpr int NTH = kSerialThreads;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* rest = smem + 2 * kStageBytes;
  bf16* TiH = reinterpret_cast<bf16*>(rest);
  bf16* TiL = TiH + kTile;
  bf16* WH = TiL + kTile;
  bf16* WL = WH + kTile;
  bf16* PH = WL + kTile;
  bf16* PL = PH + kTile;
  bf16* SH = PL + kTile;
  bf16* SL = SH + kTile;
  bf16* UH = SL + kTile;
  bf16* UL = UH + kTile;
  bf16* BUH = UL + kTile;
  bf16* BUL = BUH + kTile;
  float* Tf = reinterpret_cast<float*>(UH);
  bf16 *TH = BUH, *TL = BUL, *YH = WH, *YL = WL;
  auto Kt = [&](int s) { return reinterpret_cast<bf16*>(smem + s * kStageBytes); };
  auto Qt = [&](int s) { return Kt(s) + kTile; };
  auto Vt = [&](int s) { return Kt(s) + 2 * kTile; };
  auto Bt = [&](int s) { return reinterpret_cast<float*>(smem + s * kStageBytes + 3 * kTileBytes); };

  const int tid = threadIdx.x, warp = tid >> 5, mt = warp & 3, q = warp >> 2;
  const int m0 = 16 * mt, nv = q * (DVS / 4), mat = q >> 1, hf = q & 1;
  const int split = blockIdx.x % p.S;
  const long long bh = blockIdx.x / p.S;
  const int c0 = split * p.dvs, ncols = min(p.dvs, p.dv - c0);
  const int kd = up16(p.dk);
  const long long rows = p.T * p.nh;
  const bf16* Kg = p.K + bh * rows * p.dk;
  const bf16* Vg = p.V + bh * rows * p.dv + c0;
  const bf16* Qg = p.Q + bh * p.T * p.dk;
  const bf16* bg = p.beta + bh * rows;
  bf16* yg = p.y + bh * p.T * p.dv + c0;
  float* Hsg = p.Hs + bh * (long long)p.nchunks * p.dk * p.dv + c0;
  bf16* Tig = p.Ti + bh * (long long)p.nchunks * 2 * 4096;

  auto stage = [&](int c, int s) {
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
    stage_rows<8, NTH>(Kt(s), Kg + t0 * p.nh * p.dk, p.dk, Mc, p.dk >> 3);
    stage_rows<8, NTH>(Qt(s), Qg + t0 * p.dk, p.dk, Cc, p.dk >> 3);
    stage_rows<DVS / 8, NTH>(Vt(s), Vg + t0 * p.nh * p.dv, p.dv, Mc, ncols >> 3);
    cp_async_commit();
  };
  // beta of a chunk, as raw bf16 bits: the next chunk's values are loaded a
  // chunk ahead and converted only when stored, so no warp waits on the load.
  auto beta_of = [&](int c) -> unsigned short {
    const long long r0 = (long long)c * p.C * p.nh;
    const int Mc = (int)min((long long)p.C * p.nh, rows - r0);
    return tid < Mc ? reinterpret_cast<const unsigned short*>(bg)[r0 + tid] : (unsigned short)0;
  };
  auto bf = [](unsigned short raw) { return __uint_as_float((unsigned)raw << 16); };

  // state slice: d_k rows m0.., value columns nv.. of this split
  float hs[NTQ][4];
  if (p.H0)
    frag_from_global(hs, p.H0 + bh * p.dk * p.dv + c0, p.dv, m0, nv, p.dk, ncols);
  else
    tc::zero(hs);
  tc::store_split(hs, SH, SL, m0, nv, Ident());
  zero_upper_blocks<NTH>(TiH, TiL);
  stage(0, 0);
  if (tid < 64) Bt(0)[tid] = bf(beta_of(0));
  unsigned short bnext = 0;

  for (int c = 0; c < p.nchunks; ++c) {
    const int s = c & 1;
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
    cp_async_wait_all();
    __syncthreads();
    if (c + 1 < p.nchunks) {
      stage(c + 1, s ^ 1);
      if (tid < 64) bnext = beta_of(c + 1);
    }
    const bf16* K = Kt(s);
    const bf16* Q = Qt(s);
    const bf16* V = Vt(s);
    const float* bs = Bt(s);
    frag_to_global(hs, Hsg + (long long)c * p.dk * p.dv, p.dv, m0, nv, p.dk, ncols);

    {
      float acc[4][4];
      tc::zero(acc);
      const int ncol = mat == 0 ? m0 + 16 : min(64, (m0 + 16) * p.nh);
      const int np = min(2, max(0, (ncol - 32 * hf + 15) / 16));
      tc::gemm<4, false, false>(acc, Op{mat == 0 ? K : Q, nullptr}, m0, Op{K, nullptr}, 32 * hf,
                                0, kd, np);
      if (mat == 0)
        store_T(acc, bs, m0, 32 * hf, Tf, TH, TL);
      else
        store_P(acc, bs, p.nh, Mc, m0, 32 * hf, PH, PL);
    }
    __syncthreads();
    tri_inv_tc(Tf, Op{TH, TL}, TiH, TiL, YH, YL);
    if (split == 0) {
      tile_to_global<NTH>(TiH, Tig + (long long)c * 8192);
      tile_to_global<NTH>(TiL, Tig + (long long)c * 8192 + 4096);
    }

    // W = Ti K (rows m0, d_k columns 16q..), U' = Ti V (value columns nv..)
    {
      float w[2][4];
      tc::zero(w);
      tc::gemm<2, false, true>(w, Op{TiH, TiL}, m0, Op{K, nullptr}, 16 * q, 0, m0 + 16);
      tc::store_split(w, WH, WL, m0, 16 * q, Ident());
    }
    float u[NTQ][4];
    tc::zero(u);
    tc::gemm<NTQ, false, true>(u, Op{TiH, TiL}, m0, Op{V, nullptr}, nv, 0, m0 + 16);
    __syncthreads();

    // U = U' - W S
    {
      float ws[NTQ][4];
      tc::zero(ws);
      tc::gemm<NTQ, false, true>(ws, Op{WH, WL}, m0, Op{SH, SL}, nv, 0, kd);
#pragma unroll
      for (int j = 0; j < NTQ; ++j)
#pragma unroll
        for (int v = 0; v < 4; ++v) u[j][v] -= ws[j][v];
    }
    tc::store_split(u, UH, UL, m0, nv, Ident());
    tc::store_split(u, BUH, BUL, m0, nv, [&](int r, int, float x) { return x * bs[r]; });
    __syncthreads();

    // y = Q S + P U (token rows m0..)
    {
      float yv[NTQ][4];
      tc::zero(yv);
      tc::gemm<NTQ, false, true>(yv, Op{Q, nullptr}, m0, Op{SH, SL}, nv, 0, kd);
      tc::gemm<NTQ, false, true>(yv, Op{PH, PL}, m0, Op{UH, UL}, nv, 0,
                                 min(64, up16((m0 + 16) * p.nh)));
      frag_to_global_bf16(yv, yg + t0 * p.dv, p.dv, m0, nv, Cc, ncols);
    }
    // S += K^T (beta U) (d_k rows m0..)
    tc::gemm<NTQ, true, true>(hs, Op{K, nullptr}, m0, Op{BUH, BUL}, nv, 0, up16(Mc));
    __syncthreads();
    tc::store_split(hs, SH, SL, m0, nv, Ident());
    if (tid < 64 && c + 1 < p.nchunks) Bt(s ^ 1)[tid] = bf(bnext);
  }
  frag_to_global(hs, p.HT + bh * p.dk * p.dv + c0, p.dv, m0, nv, p.dk, ncols);
}

// ----------------------------------------------------- backward: chain --
// smem: 2 stages {K, Q, dy_s, Ti h, Ti l, beta} | P h/l | dS h/l | dU h/l | Gn h/l
constexpr int kChainStage = 5 * kTileBytes + 256;
constexpr size_t kChainSmem = 2 * (size_t)kChainStage + 8 * (size_t)kTileBytes;

template <int DVS>
__global__ void __launch_bounds__(kSerialThreads, 1) bwd_chain_kernel(const TcArgs p) {
  constexpr int NTQ = DVS / 32;
  constexpr int NTH = kSerialThreads;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* rest = smem + 2 * kChainStage;
  bf16* PH = reinterpret_cast<bf16*>(rest);
  bf16* PL = PH + kTile;
  bf16* DH = PL + kTile;
  bf16* DL = DH + kTile;
  bf16* dUH = DL + kTile;
  bf16* dUL = dUH + kTile;
  bf16* GH = dUL + kTile;
  bf16* GL = GH + kTile;
  auto Kt = [&](int s) { return reinterpret_cast<bf16*>(smem + s * kChainStage); };
  auto Qt = [&](int s) { return Kt(s) + kTile; };
  auto Dt = [&](int s) { return Kt(s) + 2 * kTile; };
  auto TiHt = [&](int s) { return Kt(s) + 3 * kTile; };
  auto TiLt = [&](int s) { return Kt(s) + 4 * kTile; };
  auto Bt = [&](int s) { return reinterpret_cast<float*>(smem + s * kChainStage + 5 * kTileBytes); };

  const int tid = threadIdx.x, warp = tid >> 5, mt = warp & 3, q = warp >> 2;
  const int m0 = 16 * mt, nv = q * (DVS / 4);
  const int split = blockIdx.x % p.S;
  const long long bh = blockIdx.x / p.S;
  const int c0 = split * p.dvs, ncols = min(p.dvs, p.dv - c0);
  const int kd = up16(p.dk);
  const long long rows = p.T * p.nh;
  const bf16* Kg = p.K + bh * rows * p.dk;
  const bf16* Qg = p.Q + bh * p.T * p.dk;
  const bf16* dyg = p.dy + bh * p.T * p.dv + c0;
  const bf16* bg = p.beta + bh * rows;
  const bf16* Tig = p.Ti + bh * (long long)p.nchunks * 2 * 4096;
  float* dHsg = p.dHs + bh * (long long)p.nchunks * p.dk * p.dv + c0;

  auto stage = [&](int c, int s) {
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
    stage_rows<8, NTH>(Kt(s), Kg + t0 * p.nh * p.dk, p.dk, Mc, p.dk >> 3);
    stage_rows<8, NTH>(Qt(s), Qg + t0 * p.dk, p.dk, Cc, p.dk >> 3);
    stage_rows<DVS / 8, NTH>(Dt(s), dyg + t0 * p.dv, p.dv, Cc, ncols >> 3);
    tile_from_global_async<NTH>(TiHt(s), Tig + (long long)c * 8192);
    tile_from_global_async<NTH>(TiLt(s), Tig + (long long)c * 8192 + 4096);
    cp_async_commit();
  };
  // beta of a chunk, as raw bf16 bits: the next chunk's values are loaded a
  // chunk ahead and converted only when stored, so no warp waits on the load.
  auto beta_of = [&](int c) -> unsigned short {
    const long long r0 = (long long)c * p.C * p.nh;
    const int Mc = (int)min((long long)p.C * p.nh, rows - r0);
    return tid < Mc ? reinterpret_cast<const unsigned short*>(bg)[r0 + tid] : (unsigned short)0;
  };
  auto bf = [](unsigned short raw) { return __uint_as_float((unsigned)raw << 16); };

  float ds[NTQ][4];
  if (p.dHT)
    frag_from_global(ds, p.dHT + bh * p.dk * p.dv + c0, p.dv, m0, nv, p.dk, ncols);
  else
    tc::zero(ds);
  tc::store_split(ds, DH, DL, m0, nv, Ident());
  const int last = p.nchunks - 1;
  stage(last, 0);
  if (tid < 64) Bt(0)[tid] = bf(beta_of(last));
  unsigned short bnext = 0;

  for (int qq = 0; qq < p.nchunks; ++qq) {
    const int c = last - qq, s = qq & 1;
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
    cp_async_wait_all();
    __syncthreads();
    if (c > 0) {
      stage(c - 1, s ^ 1);
      if (tid < 64) bnext = beta_of(c - 1);
    }
    const bf16* K = Kt(s);
    const bf16* Q = Qt(s);
    const bf16* dY = Dt(s);
    const Op Ti{TiHt(s), TiLt(s)};
    const float* bs = Bt(s);
    frag_to_global(ds, dHsg + (long long)c * p.dk * p.dv, p.dv, m0, nv, p.dk, ncols);

    // P (token rows m0, micro-step columns 16q..)
    {
      float acc[2][4];
      tc::zero(acc);
      const int ncol = min(64, (m0 + 16) * p.nh) - 16 * q;
      tc::gemm<2, false, false>(acc, Op{Q, nullptr}, m0, Op{K, nullptr}, 16 * q, 0, kd,
                                ncol <= 0 ? 0 : 1);
      store_P(acc, bs, p.nh, Mc, m0, 16 * q, PH, PL);
    }
    __syncthreads();

    // dU = P^T dy + beta * (K dS')   (micro-step rows m0..)
    {
      float du[NTQ][4], db[NTQ][4];
      tc::zero(du);
      tc::zero(db);
      tc::gemm<NTQ, false, true>(db, Op{K, nullptr}, m0, Op{DH, DL}, nv, 0, kd);
      tc::gemm<NTQ, true, true>(du, Op{PH, PL}, m0, Op{dY, nullptr}, nv, (m0 / p.nh) & ~15,
                                up16(Cc));
#pragma unroll
      for (int j = 0; j < NTQ; ++j)
#pragma unroll
        for (int v = 0; v < 4; ++v) du[j][v] += bs[tc::frag_row(m0, v)] * db[j][v];
      tc::store_split(du, dUH, dUL, m0, nv, Ident());
    }
    __syncthreads();
    // Gn = -Ti^T dU
    {
      float g[NTQ][4];
      tc::zero(g);
      tc::gemm<NTQ, true, true>(g, Ti, m0, Op{dUH, dUL}, nv, m0, 64);
      tc::store_split(g, GH, GL, m0, nv, Neg());
    }
    __syncthreads();
    // dS = dS' + Q^T dy + K^T Gn   (d_k rows m0..)
    tc::gemm<NTQ, true, true>(ds, Op{Q, nullptr}, m0, Op{dY, nullptr}, nv, 0, up16(Cc));
    tc::gemm<NTQ, true, true>(ds, Op{K, nullptr}, m0, Op{GH, GL}, nv, 0, up16(Mc));
    tc::store_split(ds, DH, DL, m0, nv, Ident());
    if (tid < 64 && c > 0) Bt(s ^ 1)[tid] = bf(bnext);
  }
  frag_to_global(ds, p.dH0 + bh * p.dk * p.dv + c0, p.dv, m0, nv, p.dk, ncols);
}

// ----------------------------------------------------- backward: grads --
// smem: K | Q | dy | V | beta, dbeta | S h/l | dS' h/l | KK f32 | QK f32 |
//       R8 U h/l | R9 (W h/l -> Gn h/l) | R10 (Ti h/l -> dKK h/l) |
//       R11 (P h/l -> dS_ h/l) | bU h/l | dU h/l
constexpr size_t kGradSmem = 4 * (size_t)kTileBytes + 512 + 4 * (size_t)kTileBytes +
                             2 * (size_t)kF32Bytes + 12 * (size_t)kTileBytes;

constexpr int kGradThreads = 512;  // 16 warps: warp (mt, q) = (w & 3, w >> 2)

__global__ void __launch_bounds__(kGradThreads, 1) bwd_grads_kernel(const TcArgs p) {
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* K = reinterpret_cast<bf16*>(smem);
  bf16* Q = K + kTile;
  bf16* dY = Q + kTile;
  bf16* V = dY + kTile;
  float* bs = reinterpret_cast<float*>(V + kTile);
  float* dbs = bs + 64;
  bf16* SH = reinterpret_cast<bf16*>(dbs + 64);
  bf16* SL = SH + kTile;
  bf16* DH = SL + kTile;
  bf16* DL = DH + kTile;
  float* KKf = reinterpret_cast<float*>(DL + kTile);
  float* QKf = KKf + 64 * kTld;
  bf16* R8 = reinterpret_cast<bf16*>(QKf + 64 * kTld);
  bf16* R9 = R8 + 2 * kTile;
  bf16* R10 = R9 + 2 * kTile;
  bf16* R11 = R10 + 2 * kTile;
  bf16* BUH = R11 + 2 * kTile;
  bf16* BUL = BUH + kTile;
  bf16* dUH = BUL + kTile;
  bf16* dUL = dUH + kTile;
  bf16 *UH = R8, *UL = R8 + kTile;
  bf16 *WH = R9, *WL = R9 + kTile, *GH = R9, *GL = R9 + kTile;
  bf16 *TiH = R10, *TiL = R10 + kTile, *dKH = R10, *dKL = R10 + kTile;
  bf16 *PH = R11, *PL = R11 + kTile, *dSH = R11, *dSL = R11 + kTile;

  constexpr int NTH = kGradThreads;
  const int tid = threadIdx.x, warp = tid >> 5, mt = warp & 3, q = warp >> 2;
  const int m0 = 16 * mt, n0 = 16 * q;       // 16 x 16 tiles of the 64 x 64 products
  const int hf = q & 1, mat = q >> 1;        // 16 x 32 tiles of the masked products
  const int c = blockIdx.x % p.nchunks;
  const long long bh = blockIdx.x / p.nchunks;
  const long long t0 = (long long)c * p.C;
  const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
  const int kd = up16(p.dk), kv = up16(p.dv);
  const long long r0 = t0 * p.nh;
  const long long rows = p.T * p.nh;
  const long long sofs = (bh * p.nchunks + c) * (long long)p.dk * p.dv;

  stage_rows<8, NTH>(K, p.K + (bh * rows + r0) * p.dk, p.dk, Mc, p.dk >> 3);
  stage_rows<8, NTH>(Q, p.Q + (bh * p.T + t0) * p.dk, p.dk, Cc, p.dk >> 3);
  stage_rows<8, NTH>(dY, p.dy + (bh * p.T + t0) * p.dv, p.dv, Cc, p.dv >> 3);
  stage_rows<8, NTH>(V, p.V + (bh * rows + r0) * p.dv, p.dv, Mc, p.dv >> 3);
  tile_from_global_async<NTH>(TiH, p.Ti + (bh * p.nchunks + c) * 8192);
  tile_from_global_async<NTH>(TiL, p.Ti + (bh * p.nchunks + c) * 8192 + 4096);
  cp_async_commit();
  if (tid < 64) {
    bs[tid] = tid < Mc ? __bfloat162float(p.beta[bh * rows + r0 + tid]) : 0.f;
    dbs[tid] = 0.f;
  }
  // S (chunk-start state) and dS' -> split tiles (rows d_k, cols d_v)
  for (int i = tid; i < 64 * 32; i += NTH) {
    const int row = i >> 5, col = (i & 31) << 1;
    float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
    if (row < p.dk && col < p.dv) {
      a = *reinterpret_cast<const float2*>(p.Hs + sofs + row * p.dv + col);
      b = *reinterpret_cast<const float2*>(p.dHs + sofs + row * p.dv + col);
    }
    uint32_t h, l;
    tc::split_pack(a.x, a.y, h, l);
    *reinterpret_cast<uint32_t*>(SH + row * kLd + col) = h;
    *reinterpret_cast<uint32_t*>(SL + row * kLd + col) = l;
    tc::split_pack(b.x, b.y, h, l);
    *reinterpret_cast<uint32_t*>(DH + row * kLd + col) = h;
    *reinterpret_cast<uint32_t*>(DL + row * kLd + col) = l;
  }
  cp_async_wait_all();
  __syncthreads();

  // K K^T (warps mat 0) / Q K^T (mat 1): row tile m0, columns 32*hf..
  {
    float acc[4][4];
    tc::zero(acc);
    const int ncol = mat == 0 ? m0 + 16 : min(64, (m0 + 16) * p.nh);
    const int np = min(2, max(0, (ncol - 32 * hf + 15) / 16));
    tc::gemm<4, false, false>(acc, Op{mat == 0 ? K : Q, nullptr}, m0, Op{K, nullptr}, 32 * hf, 0,
                              kd, np);
    float* dst = mat == 0 ? KKf : QKf;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int v = 0; v < 4; ++v)
        dst[tc::frag_row(m0, v) * kTld + tc::frag_col(32 * hf, j, v)] = acc[j][v];
    if (mat == 1)
      tc::store_split(acc, PH, PL, m0, 32 * hf, [&](int r, int cl, float x) {
        return (cl < (r + 1) * p.nh && cl < Mc) ? x * bs[cl] : 0.f;
      });
  }

  // W = Ti K, U' = Ti V (rows m0, columns n0..n0+15)
  float u[2][4];
  {
    float w[2][4];
    tc::zero(w);
    tc::gemm<2, false, true>(w, Op{TiH, TiL}, m0, Op{K, nullptr}, n0, 0, m0 + 16);
    tc::store_split(w, WH, WL, m0, n0, Ident());
    tc::zero(u);
    tc::gemm<2, false, true>(u, Op{TiH, TiL}, m0, Op{V, nullptr}, n0, 0, m0 + 16);
  }
  __syncthreads();
  // U = U' - W S;  dbU = K dS';  dU = P^T dy + beta dbU;  dbeta += rowsum(U * dbU)
  {
    float ws[2][4], db[2][4], du[2][4];
    tc::zero(ws);
    tc::zero(db);
    tc::zero(du);
    tc::gemm<2, false, true>(ws, Op{WH, WL}, m0, Op{SH, SL}, n0, 0, kd);
    tc::gemm<2, false, true>(db, Op{K, nullptr}, m0, Op{DH, DL}, n0, 0, kd);
    tc::gemm<2, true, true>(du, Op{PH, PL}, m0, Op{dY, nullptr}, n0, (m0 / p.nh) & ~15, up16(Cc));
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        u[j][v] -= ws[j][v];
        rs[v >> 1] += u[j][v] * db[j][v];
        du[j][v] += bs[tc::frag_row(m0, v)] * db[j][v];
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
    }
    if ((tid & 3) == 0) {
      atomicAdd(&dbs[tc::frag_row(m0, 0)], rs[0]);
      atomicAdd(&dbs[tc::frag_row(m0, 2)], rs[1]);
    }
    tc::store_split(u, UH, UL, m0, n0, Ident());
    tc::store_split(u, BUH, BUL, m0, n0, [&](int r, int, float x) { return x * bs[r]; });
    tc::store_split(du, dUH, dUL, m0, n0, Ident());
  }
  __syncthreads();
  // G = Ti^T dU -> dV; Gn = -G
  {
    float g[2][4];
    tc::zero(g);
    tc::gemm<2, true, true>(g, Op{TiH, TiL}, m0, Op{dUH, dUL}, n0, m0, 64);
    frag_to_global_bf16(g, p.dV + (bh * rows + r0) * p.dv, p.dv, m0, n0, Mc, p.dv);
    tc::store_split(g, GH, GL, m0, n0, [](int, int, float x) { return -x; });
  }
  __syncthreads();
  // warp (mat, mt, hf): mat 0: dS_ = (dy U^T) beta * read; mat 1: dKK = (Gn U^T) beta * strict
  {
    float acc[4][4];
    tc::zero(acc);
    const bool m1 = mat != 0;
    const int ncol = m1 ? min(64, m0 + 16) : min(64, (m0 + 16) * p.nh);
    const int np = min(2, max(0, (ncol - 32 * hf + 15) / 16));
    tc::gemm<4, false, false>(acc, m1 ? Op{GH, GL} : Op{dY, nullptr}, m0, Op{UH, UL}, 32 * hf, 0,
                              kv, np);
    // masked product, dbeta column terms, split store
    float cs[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      cs[j][0] = cs[j][1] = 0.f;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int row = tc::frag_row(m0, v), col = tc::frag_col(32 * hf, j, v);
        const bool keep = m1 ? (col < row && col < Mc) : (col < (row + 1) * p.nh && col < Mc);
        const float x = keep ? acc[j][v] : 0.f;
        cs[j][v & 1] += x * (m1 ? KKf[row * kTld + col] : QKf[row * kTld + col]);
        acc[j][v] = x * bs[col];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float x = cs[j][e];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        if ((tid & 31) < 4) atomicAdd(&dbs[tc::frag_col(32 * hf, j, e)], x);
      }
    tc::store_split(acc, m1 ? dKH : dSH, m1 ? dKL : dSL, m0, 32 * hf, Ident());
  }
  __syncthreads();
  // dQ (token rows m0, d_k columns n0..) = dy S^T + dS_ K
  {
    float dq[2][4];
    tc::zero(dq);
    tc::gemm<2, false, false>(dq, Op{dY, nullptr}, m0, Op{SH, SL}, n0, 0, kv);
    tc::gemm<2, false, true>(dq, Op{dSH, dSL}, m0, Op{K, nullptr}, n0, 0,
                             min(64, up16((m0 + 16) * p.nh)));
    frag_to_global_bf16(dq, p.dQ + (bh * p.T + t0) * p.dk, p.dk, m0, n0, Cc, p.dk);
  }
  // dK (micro-step rows m0, d_k columns n0..) =
  //   (beta U) dS'^T + dS_^T Q + Gn S^T + dKK K + dKK^T K
  {
    float dk[2][4];
    tc::zero(dk);
    tc::gemm<2, false, false>(dk, Op{BUH, BUL}, m0, Op{DH, DL}, n0, 0, kv);
    tc::gemm<2, true, true>(dk, Op{dSH, dSL}, m0, Op{Q, nullptr}, n0, (m0 / p.nh) & ~15, up16(Cc));
    tc::gemm<2, false, false>(dk, Op{GH, GL}, m0, Op{SH, SL}, n0, 0, kv);
    tc::gemm<2, false, true>(dk, Op{dKH, dKL}, m0, Op{K, nullptr}, n0, 0, m0 + 16);
    tc::gemm<2, true, true>(dk, Op{dKH, dKL}, m0, Op{K, nullptr}, n0, m0, 64);
    frag_to_global_bf16(dk, p.dK + (bh * rows + r0) * p.dk, p.dk, m0, n0, Mc, p.dk);
  }
  __syncthreads();
  if (tid < Mc) p.dbeta[bh * rows + r0 + tid] = __float2bfloat16_rn(dbs[tid]);
}

// ---------------------------------------------------------------- host --

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Value-column splits per (b, h) for the chunk-serial kernels: two when that
// still fits one wave of SMs (halves each CTA's serial work), else one.
int splits_for(long long BH, int dv) {
  return (dv > 32 && 2 * BH <= (long long)sm_count()) ? 2 : 1;
}

template <class K>
int launch_tc(K kernel, long long grid, size_t smem, cudaStream_t st, const TcArgs& a,
              int threads = kTcThreads) {
  MGS_CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  TcArgs args = a;
  void* kargs[] = {&args};
  MGS_CUDA_OK(cudaLaunchKernel((const void*)kernel, dim3((unsigned)grid), dim3(threads), kargs,
                               smem, st));
  return MGS_OK;
}

}  // namespace

bool tc_eligible(int dtype, int nh, int dk, int dv, int C) {
  return dtype == MGS_BF16 && nh >= 1 && C >= 1 && nh * C <= 64 && dk >= 8 && dk <= 64 &&
         dv >= 8 && dv <= 64 && dk % 8 == 0 && dv % 8 == 0;
}

// saved: chunk-start states (fp32) then every chunk's T^{-1} (split bf16, 64 x 64 x 2)
size_t tc_saved_floats(long long BH, long long T, int dk, int dv, int C) {
  const size_t nc = (size_t)BH * (size_t)((T + C - 1) / C);
  return nc * dk * dv + nc * 4096;
}

size_t tc_workspace_floats(long long BH, long long T, int dk, int dv, int C) {
  return (size_t)BH * (size_t)((T + C - 1) / C) * dk * dv;
}

int run_tc(bool fwd, const Args<__nv_bfloat16>& p, long long B, int H, long long T, int nh, int dk,
           int dv, int C, float* saved, void* ws, size_t ws_bytes, cudaStream_t st) {
  const long long BH = B * (long long)H;
  TcArgs a{};
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
  a.T = T;
  a.nh = nh;
  a.dk = dk;
  a.dv = dv;
  a.C = C;
  a.nchunks = (int)((T + C - 1) / C);
  a.S = splits_for(BH, dv);
  a.dvs = ((dv + a.S - 1) / a.S + 7) & ~7;
  const bool narrow = a.dvs <= 32;
  if (BH == 0) return MGS_OK;
  if (saved == nullptr) return MGS_BAD_SHAPE;
  a.Hs = saved;
  a.Ti = reinterpret_cast<bf16*>(saved + (size_t)BH * a.nchunks * dk * dv);
  if (fwd) {
    if (T == 0) {
      if (p.H0)
        MGS_CUDA_OK(cudaMemcpyAsync(p.HT, p.H0, (size_t)BH * dk * dv * sizeof(float),
                                    cudaMemcpyDeviceToDevice, st));
      else
        MGS_CUDA_OK(cudaMemsetAsync(p.HT, 0, (size_t)BH * dk * dv * sizeof(float), st));
      return MGS_OK;
    }
    return narrow ? launch_tc(fwd_kernel<32>, BH * a.S, kFwdSmem, st, a, kSerialThreads)
                  : launch_tc(fwd_kernel<64>, BH * a.S, kFwdSmem, st, a, kSerialThreads);
  }
  if (T == 0) {
    if (p.dHT)
      MGS_CUDA_OK(cudaMemcpyAsync(p.dH0, p.dHT, (size_t)BH * dk * dv * sizeof(float),
                                  cudaMemcpyDeviceToDevice, st));
    else
      MGS_CUDA_OK(cudaMemsetAsync(p.dH0, 0, (size_t)BH * dk * dv * sizeof(float), st));
    return MGS_OK;
  }
  if (ws == nullptr || ws_bytes < tc_workspace_floats(BH, T, dk, dv, C) * sizeof(float))
    return MGS_WORKSPACE_TOO_SMALL;
  a.dHs = static_cast<float*>(ws);
  int rc = narrow ? launch_tc(bwd_chain_kernel<32>, BH * a.S, kChainSmem, st, a, kSerialThreads)
                  : launch_tc(bwd_chain_kernel<64>, BH * a.S, kChainSmem, st, a, kSerialThreads);
  if (rc != MGS_OK) return rc;
  return launch_tc(bwd_grads_kernel, BH * a.nchunks, kGradSmem, st, a, kGradThreads);
}

}  // namespace delta
}  // namespace mgs
