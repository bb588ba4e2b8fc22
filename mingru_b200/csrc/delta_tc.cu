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
// Each chunk is an affine map of the state, S' = S + Xn S + Bc with
// Xn = -K^T diag(beta) W and Bc = K^T diag(beta) U', read out as
// y = Qt S + Yp with Qt = Q - P W and Yp = P U'; the adjoint chain is
// dS = dS' + Xn^T dS' + Qt^T dy. So every product that does not involve the
// state runs in parallel over all chunks, and the two chunk-serial kernels do
// one state product per chunk.
//
// Kernels (the 64 x 64 chunk products run on the tcgen05 tensor cores with
// split hi/lo bf16 operands, umma.cuh; T^{-1} by blocked substitution, its
// 16 x 16 blocks on mma.sync, mma_bf16.cuh):
//   prep_kernel       one CTA per (b, h, chunk): T^{-1} (saved), Xn, Qt
//                     (saved), Bc, Yp (forward workspace).
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
// Tiles kept in `saved` (T^{-1}, Xn, Qt) use the shared-memory layout (64 rows
// of kLd elements), so one contiguous bulk copy stages a tile.
constexpr int kSavedTile = 64 * kLd;
constexpr long long kSavedPair = 2 * kSavedTile;
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
  bf16* Xn;     // (BH, nchunks, 2, 64, 64) -K^T diag(beta) W, split
  bf16* Qt;     // (BH, nchunks, 2, 64, 64) Q - P W, split
  float* Bc;    // (BH, nchunks, 4096) K^T diag(beta) U' as [dk][dv] (forward workspace)
  float* Yp;    // (BH, nchunks, 4096) P U' as [C][dv] (forward workspace)
  float* dHs;   // (BH, nchunks, dk, dv) gradient of each chunk's output state
  long long T;
  int nh, dk, dv, C, nchunks, S, dvs;
};

// ----------------------------------------------------- backward: grads --
// One CTA per (b, h, chunk), two CTAs per SM: every gradient of the chunk from
// its saved S, T^{-1} and dS', on the tcgen05 tensor cores (umma.cuh). Two
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
// Shared tiles (blocked, 8 KB): 0 K | 1 Q | 2 dY | 3, 4 S | 5, 6 dS' -> dKK |
//   7, 8 Ti -> Gn | 9 V -> -W hi -> U hi | 10, 11 P -> dU -> dS_ | 12 -W lo -> U lo
constexpr int kGradThreads = 256;
constexpr int kGradTiles = 13;
constexpr size_t kGradSmem = 1024 + kGradTiles * (size_t)umma::kTileBytes + 2048;
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

// Padded shared tile -> blocked global tile (16-byte chunks, all threads).
template <int NTHR>
__device__ __forceinline__ void tile_to_global_blocked(const bf16* t, bf16* g) {
  for (int i = threadIdx.x; i < 64 * 8; i += NTHR) {
    const int row = i >> 3, ch = i & 7;
    *reinterpret_cast<uint4*>(g + umma::boff(row, ch * 8)) =
        *reinterpret_cast<const uint4*>(t + row * kLd + ch * 8);
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

__global__ void __launch_bounds__(kGradThreads, 2) bwd_grads_kernel(const TcArgs p) {
  namespace um = umma;
  extern __shared__ __align__(1024) unsigned char gsmem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(gsmem);  // [0] MMA batches, [1] T^{-1} copy
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(gsmem + 64);
  bf16* tiles = reinterpret_cast<bf16*>(gsmem + 1024);
  auto T = [&](int i) { return tiles + i * (um::kTileBytes / 2); };
  bf16 *K = T(0), *Q = T(1), *dY = T(2), *SH = T(3), *SL = T(4), *DH = T(5), *DL = T(6),
       *TiH = T(7), *TiL = T(8), *V = T(9);
  bf16 *dKH = T(5), *dKL = T(6), *GH = T(7), *GL = T(8), *WH = T(9), *WL = T(12), *UH = T(9),
       *UL = T(12), *PH = T(10), *PL = T(11), *dUH = T(10), *dUL = T(11), *dSH = T(10),
       *dSL = T(11);
  float* bs = reinterpret_cast<float*>(T(kGradTiles));
  float* rpart = bs + 64;      // [2 column halves][64 rows]: sum_col U * dbU
  float* cpart = rpart + 128;  // [8 warps][32 columns]: masked-product column sums

  constexpr int NTH = kGradThreads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hh = warp >> 2, row = 16 * q + lane;
  const bool rv = lane < 16;  // this lane holds row `row` of the 64-row accumulators
  const int c = blockIdx.x % p.nchunks;
  const long long bh = blockIdx.x / p.nchunks;
  const long long t0 = (long long)c * p.C;
  const int Cc = (int)min((long long)p.C, p.T - t0), Mc = Cc * p.nh;
  const long long r0 = t0 * p.nh, rows = p.T * p.nh;
  const long long blk = bh * p.nchunks + c;
  const long long sofs = blk * (long long)p.dk * p.dv;

  if (warp == 0) um::alloc(tbase_s, kGradTmemCols);
  if (tid == 0) {
    mbar_init(bar, 2);  // MMA batches: one commit from each issuing thread
    mbar_init(bar + 1, 1);
    mbar_fence_init();
  }
  stage_blocked<NTH>(K, p.K + (bh * rows + r0) * p.dk, p.dk, Mc, p.dk >> 3);
  stage_blocked<NTH>(Q, p.Q + (bh * p.T + t0) * p.dk, p.dk, Cc, p.dk >> 3);
  stage_blocked<NTH>(dY, p.dy + (bh * p.T + t0) * p.dv, p.dv, Cc, p.dv >> 3);
  stage_blocked<NTH>(V, p.V + (bh * rows + r0) * p.dv, p.dv, Mc, p.dv >> 3);
  cp_async_commit();
  um::fence_before();
  __syncthreads();  // barriers initialised, TMEM base written
  if (tid == 0) {
    mbar_arrive_expect_tx(bar + 1, 2 * um::kTileBytes);
    bulk_g2s(TiH, p.Ti + blk * kSavedPair, um::kTileBytes, bar + 1);
    bulk_g2s(TiL, p.Ti + blk * kSavedPair + 4096, um::kTileBytes, bar + 1);
  }
  {  // S (chunk-start state) and dS' (fp32 [dk][dv]) -> split blocked tiles
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
      uint32_t ph[4], pl[4], qh[4], ql[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tc::split_pack(av[2 * j], av[2 * j + 1], ph[j], pl[j]);
        tc::split_pack(bv[2 * j], bv[2 * j + 1], qh[j], ql[j]);
      }
      const int o = um::boff(r, cb * 8);
      *reinterpret_cast<uint4*>(SH + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
      *reinterpret_cast<uint4*>(SL + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
      *reinterpret_cast<uint4*>(DH + o) = make_uint4(qh[0], qh[1], qh[2], qh[3]);
      *reinterpret_cast<uint4*>(DL + o) = make_uint4(ql[0], ql[1], ql[2], ql[3]);
    }
  }
  if (tid < 64) bs[tid] = tid < Mc ? __bfloat162float(p.beta[bh * rows + r0 + tid]) : 0.f;
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
  // load two 16-column halves of this thread's 32 columns from NA accumulators
  // at column offsets off[] (one wait), as v[acc][half][16]
  auto S_ = [](const bf16* t) { return um::saddr(t); };

  // level 1
  to_mma();
  if (okw && tid == 0) {
    const um::Opnd oTi = um::opnd(S_(TiH), S_(TiL), false);
    const um::Prod ps[2] = {{tA, oTi, um::opnd(S_(K), 0, true), false},
                            {tB, oTi, um::opnd(S_(V), 0, true), false}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {
    const um::Prod ps[2] = {{tC, um::opnd(S_(K), 0, false), um::opnd(S_(DH), S_(DL), true), false},
                            {tD, um::opnd(S_(Q), 0, false), um::opnd(S_(K), 0, false), false}};
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
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int cl = c0 + i;
        v[i] = (cl < (row + 1) * p.nh && cl < Mc) ? v[i] * bs[cl] : 0.f;
        w[i] = -w[i];
      }
      um::store_split16(PH, PL, row, c0, v);
      um::store_split16(WH, WL, row, c0, w);
    }
  }
  // level 2
  to_mma();
  if (okw && tid == 0) {
    const um::Prod ps[1] = {{tB, um::opnd(S_(WH), S_(WL), false), um::opnd(S_(SH), S_(SL), true), true}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {
    const um::Prod ps[1] = {{tA, um::opnd(S_(PH), S_(PL), true), um::opnd(S_(dY), 0, true), false}};
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
        const float b = bs[row];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          rs += u[i] * db[i];
          pd[i] += b * db[i];
        }
        um::store_split16(UH, UL, row, c0, u);
        um::store_split16(dUH, dUL, row, c0, pd);
      }
    }
    if (rv) rpart[hh * 64 + row] = rs;
  }
  // level 3
  to_mma();
  if (okw && tid == 0) {  // G = Ti^T dU as (Ti^T dU_hi) + (Ti_hi^T dU_lo) in C and D
    const um::Prod ps[2] = {
        {tC, um::opnd(S_(TiH), S_(TiL), true), um::opnd(S_(dUH), 0, true), false},
        {tD, um::opnd(S_(TiH), 0, true), um::opnd(S_(dUL), 0, true), false}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {  // U dS'^T in A
    const um::Prod ps[1] = {{tA, um::opnd(S_(UH), S_(UL), false), um::opnd(S_(DH), S_(DL), false), false}};
    um::products(ps);
    um::commit(bar);
  }
  wait_mma();
  float uds[2][16];  // U dS'^T of this thread's row, held until the last epilogue
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // dV = G; Gn = -G
    const int c0 = 32 * hh + 16 * half;
    uint32_t r1[16], r2[16], r3[16];
    float g[16], g2[16];
    um::ld16_async(lb + 128 + 16 * half, r1);
    um::ld16_async(lb + 192 + 16 * half, r2);
    um::ld16_async(lb + 0 + 16 * half, r3);
    um::ld_wait();
    um::ld_bind(r1, g);
    um::ld_bind(r2, g2);
    um::ld_bind(r3, uds[half]);
    if (rv) {
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] += g2[i];
      if (okw && row < Mc) row16_to_global(p.dV + (bh * rows + r0 + row) * p.dv, c0, p.dv, g);
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] = -g[i];
      um::store_split16(GH, GL, row, c0, g);
    }
  }
  // level 4
  to_mma();
  if (okw && tid == 0) {  // Gn U^T in B, K K^T in C
    const um::Prod ps[2] = {{tB, um::opnd(S_(GH), S_(GL), false), um::opnd(S_(UH), S_(UL), false), false},
                            {tC, um::opnd(S_(K), 0, false), um::opnd(S_(K), 0, false), false}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {  // dy U^T in A, Q K^T in D
    const um::Prod ps[2] = {{tA, um::opnd(S_(dY), 0, false), um::opnd(S_(UH), S_(UL), false), false},
                            {tD, um::opnd(S_(Q), 0, false), um::opnd(S_(K), 0, false), false}};
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
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int cl = c0 + i;
        const float x = (rv && cl < (row + 1) * p.nh && cl < Mc) ? ds[i] : 0.f;
        const float y = (rv && cl < row && cl < Mc) ? dk[i] : 0.f;
        e[i] = rv ? x * qk[i] + y * kk[i] : 0.f;
        ds[i] = x * bs[cl];
        dk[i] = y * bs[cl];
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
        um::store_split16(dSH, dSL, row, c0, ds);
        um::store_split16(dKH, dKL, row, c0, dk);
      }
    }
    cpart[warp * 32 + lane] = cs;
  }
  // level 5
  to_mma();
  if (okw && tid == 0) {  // dQ in A, Gn S^T in C
    const um::Opnd oS = um::opnd(S_(SH), S_(SL), false);
    const um::Prod ps[3] = {{tA, um::opnd(S_(dY), 0, false), oS, false},
                            {tC, um::opnd(S_(GH), S_(GL), false), oS, false},
                            {tA, um::opnd(S_(dSH), S_(dSL), false), um::opnd(S_(K), 0, true), true}};
    um::products(ps);
    um::commit(bar);
  } else if (okw && tid == 32) {  // dS_^T Q + dKK K in B, dKK^T K in D
    const um::Opnd oKmn = um::opnd(S_(K), 0, true);
    const um::Prod ps[3] = {{tB, um::opnd(S_(dSH), S_(dSL), true), um::opnd(S_(Q), 0, true), false},
                            {tD, um::opnd(S_(dKH), S_(dKL), true), oKmn, false},
                            {tB, um::opnd(S_(dKH), S_(dKL), false), oKmn, true}};
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
    if (okw && rv && row < Cc) row16_to_global(p.dQ + (bh * p.T + t0 + row) * p.dk, c0, p.dk, v);
    if (okw && rv && row < Mc) {
      const float b = bs[row];
#pragma unroll
      for (int i = 0; i < 16; ++i) v2[i] += v3[i] + v4[i] + b * uds[half][i];
      row16_to_global(p.dK + (bh * rows + r0 + row) * p.dk, c0, p.dk, v2);
    }
  }
  um::fence_before();
  __syncthreads();
  if (okw && tid < Mc) {  // dbeta = row sums of U * dbU + column sums of the masked products
    const int h2 = tid >> 5, cl = tid & 31;
    const float d = (rpart[tid] + rpart[64 + tid]) +
                    (cpart[(4 * h2) * 32 + cl] + cpart[(4 * h2 + 1) * 32 + cl]) +
                    (cpart[(4 * h2 + 2) * 32 + cl] + cpart[(4 * h2 + 3) * 32 + cl]);
    p.dbeta[bh * rows + r0 + tid] = __float2bfloat16_rn(d);
  }
  if (warp == 0) {
    um::fence_after();
    um::dealloc(tb, kGradTmemCols);
  }
}

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

// 16 fp32 values of row r (columns c0..) -> global row (columns < ncols).
__device__ __forceinline__ void row16_f32_to_global(float* g, int c0, int ncols, const float (&v)[16]) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (c0 + 4 * k < ncols)
      *reinterpret_cast<float4*>(g + c0 + 4 * k) = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

__global__ void __launch_bounds__(kPrepThreads, 2) prep_kernel(const TcArgs p) {
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
    bulk_s2g(p.Ti + blk * kSavedPair, TiH, um::kTileBytes);
    bulk_s2g(p.Ti + blk * kSavedPair + 4096, TiL, um::kTileBytes);
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
    bulk_s2g(p.Xn + blk * kSavedPair, XsH, 2 * um::kTileBytes);  // hi, lo contiguous
    bulk_s2g(p.Qt + blk * kSavedPair, QsH, 2 * um::kTileBytes);
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

// Thread 0: stage the saved tile pairs Xn and Qt of one chunk (blocked, hi and
// lo contiguous) with bulk copies completing on `bar`: X receives Xn hi, Xn lo,
// Qt hi, Qt lo.
__device__ __forceinline__ void stage_xq(bf16* X, const TcArgs& p, long long blk, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, 4 * umma::kTileBytes);
  bulk_g2s(X, p.Xn + blk * kSavedPair, 2 * umma::kTileBytes, bar);
  bulk_g2s(X + 8192, p.Qt + blk * kSavedPair, 2 * umma::kTileBytes, bar);
}

// The chunk-serial kernels: one CTA per (b, h, 32 value columns), 8 warps.
// Thread (warp w, lane l < 16) owns row 16*(w%4) + l and columns 16*(w/4)..+15
// of the CTA's state slice, in fp32 registers; the slice is also kept as a
// split blocked tile (64 x 32) in shared memory, the B operand of the chunk's
// MMAs. Per chunk, thread 0 issues the state product and thread 32 the other
// product (12 and 8-12 tcgen05 MMAs, N = 32) into TMEM; all threads then add
// them to the state and write the new split tile. The Xn, Qt tiles of the next
// kRing - 1 chunks are staged by bulk copies.
constexpr int kChainThreads = 256;
constexpr int kChainCols = 32;
constexpr int kSTile = 64 * kChainCols * 2;  // one split half of a 64 x 32 slice, bytes

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

// ------------------------------------------------------ forward: chain --
//   S_c saved;  y_c = Qt S_c + Yp;  S_{c+1} = S_c + Xn S_c + Bc
// Both products share the state operand, so [Xn; Qt] is staged as one
// M = 128 operand (Xn hi, Qt hi, Xn lo, Qt lo) and one thread issues 12 MMAs
// per chunk. Accumulator row r sits in TMEM lane r: warps 0, 1, 4, 5 (rows
// 0-63) own the state S, warps 2, 3, 6, 7 (rows 64-127) the output y; lane l of
// warp w has row 32*(w%4) + l, columns 16*(w/4)..+15.
// stage: [Xn; Qt] hi and lo (bulk copies) and every thread's 16 additive terms
// (Bc or Yp; cp.async) as float4 [4][thread]
constexpr int kCfAddend = 4 * kChainThreads * 16;
constexpr int kCfStage = 4 * umma::kTileBytes + kCfAddend;
constexpr size_t kChainFwdSmem = 1024 + kRing * (size_t)kCfStage + 2 * (size_t)kSTile;

__global__ void __launch_bounds__(kChainThreads, 1) chain_fwd_kernel(const TcArgs p) {
  namespace um = umma;
  extern __shared__ __align__(1024) unsigned char csmem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(csmem);
  uint64_t* mbar = full + kRing;  // MMA completion
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(csmem + 64);
  unsigned char* ring = csmem + 1024;
  bf16* SH = reinterpret_cast<bf16*>(ring + kRing * kCfStage);
  bf16* SL = SH + 64 * kChainCols;
  auto Xt = [&](int s) { return reinterpret_cast<bf16*>(ring + s * kCfStage); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = warp & 3;
  const int cb = 16 * (warp >> 2);
  const bool st = q < 2;                 // state thread (row r of S) or output thread (row r of y)
  const int r = 32 * (q & 1) + lane;     // row within S (state) or within the chunk's tokens (y)
  const int split = blockIdx.x % p.S;
  const long long bh = blockIdx.x / p.S;
  const int c0 = split * kChainCols, ncols = min(kChainCols, p.dv - c0);
  const long long blk0 = bh * p.nchunks;
  bf16* yg = p.y + bh * p.T * p.dv + c0 + cb;
  float* Hsg = p.Hs + blk0 * p.dk * p.dv + r * p.dv + c0 + cb;
  const bool srow = st && r < p.dk;

  auto stage = [&](int c) {
    bf16* X = Xt(c % kRing);
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0);
    if (tid == 0) {
      uint64_t* bar = full + c % kRing;
      const long long blk = blk0 + c;
      mbar_arrive_expect_tx(bar, 4 * umma::kTileBytes);
      bulk_g2s(X, p.Xn + blk * kSavedPair, umma::kTileBytes, bar);
      bulk_g2s(X + 4096, p.Qt + blk * kSavedPair, umma::kTileBytes, bar);
      bulk_g2s(X + 8192, p.Xn + blk * kSavedPair + 4096, umma::kTileBytes, bar);
      bulk_g2s(X + 12288, p.Qt + blk * kSavedPair + 4096, umma::kTileBytes, bar);
    }
    float4* ad = reinterpret_cast<float4*>(X + 16384);
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
  if (st) um::store_split16_n(SH, SL, r, cb, kChainCols, kChainCols, hs);
  um::fence_before();
  __syncthreads();
  um::fence_after();
  const uint32_t tb = *tbase_s;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + cb;
  const um::Opnd oS = um::opnd_mn(um::saddr(SH), um::saddr(SL), kChainCols);
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
    fence_proxy_async_smem();  // the split state written below in the previous chunk
    um::fence_before();
    // every thread is past chunk c - 1: its stage may be refilled
    if (__syncthreads_or(!okw)) {
      okw = false;
      break;
    }
    um::fence_after();
    if (c + kRing - 1 < p.nchunks) stage(c + kRing - 1);
    const float4* ad = reinterpret_cast<const float4*>(Xt(s) + 16384);
    if (tid == 0) {  // [Xn; Qt] S, M = 128
      const uint32_t X = um::saddr(Xt(s));
      const um::Prod ps[1] = {{tb, um::opnd(X, X + 16384, false), oS, false, true, kChainCols}};
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
      um::store_split16_n(SH, SL, r, cb, kChainCols, kChainCols, hs);
      if (srow && c + 1 < p.nchunks) store16_f32(Hsg + (long long)(c + 1) * p.dk * p.dv, cb, ncols, hs);
    } else if (r < Cc) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (cb + 8 * h < ncols) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) w[i] = tc::pack_bf16(v[8 * h + 2 * i], v[8 * h + 2 * i + 1]);
          *reinterpret_cast<uint4*>(yg + (t0 + r) * p.dv + 8 * h) = make_uint4(w[0], w[1], w[2], w[3]);
        }
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
constexpr int kCbStage = 4 * umma::kTileBytes + kSTile;  // Xn h/l, Qt h/l, dy (64 x 32)
constexpr size_t kChainBwdSmem = 1024 + kRing * (size_t)kCbStage + 2 * (size_t)kSTile;

__global__ void __launch_bounds__(kChainThreads, 1) chain_bwd_kernel(const TcArgs p) {
  namespace um = umma;
  extern __shared__ __align__(1024) unsigned char csmem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(csmem);
  uint64_t* mbar = full + kRing;
  uint32_t* tbase_s = reinterpret_cast<uint32_t*>(csmem + 64);
  unsigned char* ring = csmem + 1024;
  bf16* DH = reinterpret_cast<bf16*>(ring + kRing * kCbStage);
  bf16* DL = DH + 64 * kChainCols;
  auto Xt = [&](int s) { return reinterpret_cast<bf16*>(ring + s * kCbStage); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = warp & 3;
  const int row = 16 * q + lane, cb = 16 * (warp >> 2);
  const bool rv = lane < 16;
  const int split = blockIdx.x % p.S;
  const long long bh = blockIdx.x / p.S;
  const int c0 = split * kChainCols, ncols = min(kChainCols, p.dv - c0);
  const long long blk0 = bh * p.nchunks;
  const bf16* dyg = p.dy + bh * p.T * p.dv + c0;
  float* dHsg = p.dHs + blk0 * p.dk * p.dv + row * p.dv + c0 + cb;
  const bool srow = rv && row < p.dk;
  const int last = p.nchunks - 1;

  // step qq handles chunk last - qq in ring slot qq % kRing
  auto stage = [&](int qq) {
    const int c = last - qq;
    bf16* X = Xt(qq % kRing);
    if (tid == 0) stage_xq(X, p, blk0 + c, full + qq % kRing);
    const long long t0 = (long long)c * p.C;
    const int Cc = (int)min((long long)p.C, p.T - t0);
    bf16* dY = X + 16384;
    const int r = tid >> 2, ch = tid & 3;  // 64 rows x 4 chunks of 8 columns
    const bool ok = r < Cc && 8 * ch < ncols;
    const bf16* src = dyg + (t0 + r) * p.dv + 8 * ch;
    cp_async16(dY + um::boff_n(r, 8 * ch, kChainCols), ok ? src : dyg, ok ? 16 : 0);
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
  if (rv) um::store_split16_n(DH, DL, row, cb, kChainCols, kChainCols, ds);
  um::fence_before();
  __syncthreads();
  um::fence_after();
  const uint32_t tb = *tbase_s, tX = tb, tY = tb + 32;
  const uint32_t lb = tb + ((uint32_t)(32 * q) << 16) + cb;
  for (int qq = 0; qq < kRing - 1 && qq <= last; ++qq) stage(qq);
  if (srow) store16_f32(dHsg + (long long)last * p.dk * p.dv, cb, ncols, ds);
  const um::Opnd oD = um::opnd_mn(um::saddr(DH), um::saddr(DL), kChainCols);

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
    if (okw) okw = mbar_wait(full + s, (unsigned)(qq / kRing) & 1u, &g_sticky_err);
    fence_proxy_async_smem();  // dy (cp.async) and the split dS written in the previous step
    um::fence_before();
    if (__syncthreads_or(!okw)) {
      okw = false;
      break;
    }
    um::fence_after();
    if (qq + kRing - 1 <= last) stage(qq + kRing - 1);
    const uint32_t X = um::saddr(Xt(s));
    if (tid == 0) {  // Xn^T dS'
      const um::Prod ps[1] = {{tX, um::opnd(X, X + 8192, true), oD, false, false, kChainCols}};
      um::products(ps);
      um::commit(mbar);
    } else if (tid == 32) {  // Qt^T dy
      const um::Prod ps[1] = {{tY, um::opnd(X + 16384, X + 24576, true),
                               um::opnd_mn(X + 32768, 0, kChainCols), false, false, kChainCols}};
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
      um::store_split16_n(DH, DL, row, cb, kChainCols, kChainCols, ds);
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

// saved: chunk-start states (fp32), then every chunk's T^{-1}, Xn and Qt
// (split bf16 tile pairs, hi then lo, in the tcgen05 blocked layout)
size_t tc_saved_floats(long long BH, long long T, int dk, int dv, int C) {
  const size_t nc = (size_t)BH * (size_t)((T + C - 1) / C);
  return nc * dk * dv + 3 * nc * (size_t)kSavedPair / 2;
}

// forward: Bc and Yp (4096 floats each per chunk); backward: dS' per chunk
size_t tc_workspace_floats(long long BH, long long T, int dk, int dv, int C) {
  const size_t nc = (size_t)BH * (size_t)((T + C - 1) / C);
  const size_t bwd = nc * dk * dv, fwd = 2 * nc * 4096;
  return fwd > bwd ? fwd : bwd;
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
  a.S = (dv + kChainCols - 1) / kChainCols;  // chain kernels: 32 value columns per CTA
  a.dvs = kChainCols;
  if (BH == 0) return MGS_OK;
  if (saved == nullptr) return MGS_BAD_SHAPE;
  const size_t ncs = (size_t)BH * a.nchunks;
  a.Hs = saved;
  a.Ti = reinterpret_cast<bf16*>(saved + ncs * dk * dv);
  a.Xn = a.Ti + ncs * kSavedPair;
  a.Qt = a.Xn + ncs * kSavedPair;
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
    const int rc = launch_tc(prep_kernel, (long long)ncs, kPrepSmem, st, a, kPrepThreads);
    if (rc != MGS_OK) return rc;
    return launch_tc(chain_fwd_kernel, BH * a.S, kChainFwdSmem, st, a, kChainThreads);
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
  int rc = launch_tc(chain_bwd_kernel, BH * a.S, kChainBwdSmem, st, a, kChainThreads);
  if (rc != MGS_OK) return rc;
  return launch_tc(bwd_grads_kernel, BH * a.nchunks, kGradSmem, st, a, kGradThreads);
}

}  // namespace delta

// The tensor-core kernels' sticky error word (bounded mbarrier waits that ran
// out); read and cleared through mgs_take_device_error.
unsigned take_error_delta_tc(cudaStream_t s) { return take_sticky_error(s); }

}  // namespace mgs
