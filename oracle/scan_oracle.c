/*
 * scan_oracle.c -- CPU oracle for the mingru scan family. TEST INFRASTRUCTURE
 * ONLY: it is linked by tests/, by __graft_entry__.smoke() as the checker and
 * by bench.py's CPU-baseline leg, never by the product path (mingru_b200/).
 *
 * Each function restates, as a plain sequential recurrence, the algorithm of
 * the reference (chris-santiago/minGRU, package `mingru`; "min_gru.py" =
 * src/mingru/min_gru.py, "triton_scans.py" = src/mingru/triton_scans.py,
 * "test_scan_ops.py" = tests/test_scan_ops.py). Sequential loops are the
 * reference's own oracle form (test_scan_ops.py:62-110); the parity pins in
 * tests/ check these functions against golden vectors produced by the
 * reference itself (tests/golden/make_golden.py).
 *
 * Every body is written once over SCALAR and instantiated for double (the
 * ground truth the GPU kernels are gated against) and float (the timed CPU
 * baseline, same arithmetic type as the reference's fp32 path). Independent
 * lanes run in parallel under OpenMP; the time loop is sequential.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define IDX3(b, t, d, T, D) (((int64_t)(b) * (T) + (t)) * (D) + (d))

/* ----------------------------------------------------------------------- */
/* parallel_scan_log (min_gru.py:755-807; sequential form test_scan_ops.py:62-70):
 *   h_0 = exp(lv[0]); h_t = exp(lc[t-1]) h_{t-1} + exp(lv[t]),  out[t-1] = h_t.
 * Backward (hand-derived adjoint of the same recurrence, equal to autograd
 * through min_gru.py:804-807):
 *   G_t = g_t + a_{t+1} G_{t+1};  dlc_t = G_t a_t h_{t-1};  dlv_t = G_t b_t (t>=1);
 *   dlv_0 = a_1 G_1 h_0.                                                     */
#define DEF_LOG_SCAN(S, SUF)                                                              \
  void orc_log_scan_fwd_##SUF(const S* lc, const S* lv, S* h, int64_t B, int64_t T,       \
                              int64_t D) {                                                \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t b = 0; b < B; ++b)                                                       \
      for (int64_t d = 0; d < D; ++d) {                                                   \
        S x = EXP_##SUF(lv[IDX3(b, 0, d, T + 1, D)]);                                     \
        for (int64_t t = 0; t < T; ++t) {                                                 \
          x = EXP_##SUF(lc[IDX3(b, t, d, T, D)]) * x + EXP_##SUF(lv[IDX3(b, t + 1, d, T + 1, D)]); \
          h[IDX3(b, t, d, T, D)] = x;                                                     \
        }                                                                                 \
      }                                                                                   \
  }                                                                                       \
  void orc_log_scan_bwd_##SUF(const S* lc, const S* lv, const S* gh, S* dlc, S* dlv,      \
                              int64_t B, int64_t T, int64_t D) {                          \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t b = 0; b < B; ++b)                                                       \
      for (int64_t d = 0; d < D; ++d) {                                                   \
        S* hs = (S*)malloc(sizeof(S) * (size_t)(T + 1));                                  \
        hs[0] = EXP_##SUF(lv[IDX3(b, 0, d, T + 1, D)]);                                   \
        for (int64_t t = 1; t <= T; ++t)                                                  \
          hs[t] = EXP_##SUF(lc[IDX3(b, t - 1, d, T, D)]) * hs[t - 1] +                     \
                  EXP_##SUF(lv[IDX3(b, t, d, T + 1, D)]);                                 \
        S G = 0, a_next = 0;                                                              \
        for (int64_t t = T; t >= 1; --t) {                                                \
          G = gh[IDX3(b, t - 1, d, T, D)] + a_next * G;                                   \
          const S at = EXP_##SUF(lc[IDX3(b, t - 1, d, T, D)]);                            \
          dlc[IDX3(b, t - 1, d, T, D)] = G * at * hs[t - 1];                              \
          dlv[IDX3(b, t, d, T + 1, D)] = G * EXP_##SUF(lv[IDX3(b, t, d, T + 1, D)]);       \
          a_next = at;                                                                    \
        }                                                                                 \
        dlv[IDX3(b, 0, d, T + 1, D)] = (T > 0) ? a_next * G * hs[0] : 0;                   \
        free(hs);                                                                         \
      }                                                                                   \
  }

/* ----------------------------------------------------------------------- */
/* linear_scan (min_gru.py:1454-1510; sequential form test_scan_ops.py:73-83):
 *   A_t = a_t A_{t-1}, Bc_t = a_t Bc_{t-1} + b_t, A_0 = 1, Bc_0 = 0.
 * Backward: the adjoint of triton_scans.py:1013-1024.                         */
#define DEF_LINEAR_SCAN(S, SUF)                                                           \
  void orc_linear_scan_fwd_##SUF(const S* a, const S* b, S* A, S* Bc, int64_t B,          \
                                 int64_t T, int64_t D) {                                  \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t bi = 0; bi < B; ++bi)                                                    \
      for (int64_t d = 0; d < D; ++d) {                                                   \
        S xa = 1, xb = 0;                                                                 \
        for (int64_t t = 0; t < T; ++t) {                                                 \
          const int64_t o = IDX3(bi, t, d, T, D);                                         \
          xb = a[o] * xb + b[o];                                                          \
          xa = a[o] * xa;                                                                 \
          A[o] = xa;                                                                      \
          Bc[o] = xb;                                                                     \
        }                                                                                 \
      }                                                                                   \
  }                                                                                       \
  void orc_linear_scan_bwd_##SUF(const S* a, const S* A, const S* Bc, const S* gA,        \
                                 const S* gB, S* da, S* db, int64_t B, int64_t T,         \
                                 int64_t D) {                                             \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t bi = 0; bi < B; ++bi)                                                    \
      for (int64_t d = 0; d < D; ++d) {                                                   \
        S GA = 0, GB = 0, a_next = 0;                                                     \
        for (int64_t t = T - 1; t >= 0; --t) {                                            \
          const int64_t o = IDX3(bi, t, d, T, D);                                         \
          GA = gA[o] + a_next * GA;                                                       \
          GB = gB[o] + a_next * GB;                                                       \
          const S Ap = t > 0 ? A[o - D] : (S)1;                                           \
          const S Bp = t > 0 ? Bc[o - D] : (S)0;                                          \
          da[o] = GA * Ap + GB * Bp;                                                      \
          db[o] = GB;                                                                     \
          a_next = a[o];                                                                  \
        }                                                                                 \
      }                                                                                   \
  }

/* ----------------------------------------------------------------------- */
/* matrix_affine_scan / matrix_scan (min_gru.py:1513-1655; sequential form
 * test_scan_ops.py:86-110): Abar_t = A_t Abar_{t-1}, Bbar_t = A_t Bbar_{t-1} + B_t.
 * Layout A (B,T,n,k,k), Bm (B,T,n,k,v). Backward = triton_scans.py:823-959:
 *   GA_t = gA_t + A_{t+1}^T GA_{t+1};  GB_t = gB_t + A_{t+1}^T GB_{t+1};
 *   dA_t = GA_t Abar_{t-1}^T + GB_t Bbar_{t-1}^T;  dB_t = GB_t.              */
#define DEF_AFFINE_SCAN(S, SUF)                                                           \
  void orc_affine_scan_fwd_##SUF(const S* Am, const S* Bm, S* Ab, S* Bb, int64_t B,       \
                                 int64_t T, int64_t n, int k, int v) {                    \
    const int64_t kk = (int64_t)k * k, kv = (int64_t)k * v;                               \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t bi = 0; bi < B; ++bi)                                                    \
      for (int64_t ni = 0; ni < n; ++ni) {                                                \
        S* xa = (S*)malloc(sizeof(S) * (size_t)(2 * kk + 2 * kv));                        \
        S* xb = xa + kk;                                                                  \
        S* ta = xb + kv;                                                                  \
        S* tb = ta + kk;                                                                  \
        for (int i = 0; i < k; ++i)                                                       \
          for (int j = 0; j < k; ++j) xa[i * k + j] = (S)(i == j);                        \
        for (int64_t q = 0; q < kv; ++q) xb[q] = 0;                                       \
        for (int64_t t = 0; t < T; ++t) {                                                 \
          const S* At = Am + ((bi * T + t) * n + ni) * kk;                                \
          const S* Bt = Bm + ((bi * T + t) * n + ni) * kv;                                \
          for (int i = 0; i < k; ++i) {                                                   \
            for (int j = 0; j < k; ++j) {                                                 \
              S s = 0;                                                                    \
              for (int p = 0; p < k; ++p) s += At[i * k + p] * xa[p * k + j];             \
              ta[i * k + j] = s;                                                          \
            }                                                                             \
            for (int j = 0; j < v; ++j) {                                                 \
              S s = 0;                                                                    \
              for (int p = 0; p < k; ++p) s += At[i * k + p] * xb[p * v + j];             \
              tb[i * v + j] = s + Bt[i * v + j];                                          \
            }                                                                             \
          }                                                                               \
          memcpy(xa, ta, sizeof(S) * (size_t)kk);                                         \
          memcpy(xb, tb, sizeof(S) * (size_t)kv);                                         \
          memcpy(Ab + ((bi * T + t) * n + ni) * kk, xa, sizeof(S) * (size_t)kk);          \
          memcpy(Bb + ((bi * T + t) * n + ni) * kv, xb, sizeof(S) * (size_t)kv);          \
        }                                                                                 \
        free(xa);                                                                         \
      }                                                                                   \
  }                                                                                       \
  void orc_affine_scan_bwd_##SUF(const S* Am, const S* Ab, const S* Bb, const S* gA,      \
                                 const S* gB, S* dA, S* dB, int64_t B, int64_t T,         \
                                 int64_t n, int k, int v) {                               \
    const int64_t kk = (int64_t)k * k, kv = (int64_t)k * v;                               \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t bi = 0; bi < B; ++bi)                                                    \
      for (int64_t ni = 0; ni < n; ++ni) {                                                \
        S* GA = (S*)calloc((size_t)(2 * kk + 2 * kv), sizeof(S));                         \
        S* GB = GA + kk;                                                                  \
        S* ta = GB + kv;                                                                  \
        S* tb = ta + kk;                                                                  \
        const S* Anext = NULL;                                                            \
        for (int64_t t = T - 1; t >= 0; --t) {                                            \
          const int64_t oa = ((bi * T + t) * n + ni) * kk, ob = ((bi * T + t) * n + ni) * kv; \
          for (int p = 0; p < k; ++p) {                                                   \
            for (int j = 0; j < k; ++j) {                                                 \
              S s = gA[oa + p * k + j];                                                   \
              if (Anext)                                                                  \
                for (int i = 0; i < k; ++i) s += Anext[i * k + p] * GA[i * k + j];        \
              ta[p * k + j] = s;                                                          \
            }                                                                             \
            for (int j = 0; j < v; ++j) {                                                 \
              S s = gB[ob + p * v + j];                                                   \
              if (Anext)                                                                  \
                for (int i = 0; i < k; ++i) s += Anext[i * k + p] * GB[i * v + j];        \
              tb[p * v + j] = s;                                                          \
            }                                                                             \
          }                                                                               \
          memcpy(GA, ta, sizeof(S) * (size_t)kk);                                         \
          memcpy(GB, tb, sizeof(S) * (size_t)kv);                                         \
          const S* Ap = t > 0 ? Ab + oa - n * kk : NULL;                                  \
          const S* Bp = t > 0 ? Bb + ob - n * kv : NULL;                                  \
          for (int i = 0; i < k; ++i)                                                     \
            for (int j = 0; j < k; ++j) {                                                 \
              S s = 0;                                                                    \
              for (int p = 0; p < k; ++p) s += GA[i * k + p] * (Ap ? Ap[j * k + p] : (S)(j == p)); \
              if (Bp)                                                                     \
                for (int w = 0; w < v; ++w) s += GB[i * v + w] * Bp[j * v + w];           \
              dA[oa + i * k + j] = s;                                                     \
            }                                                                             \
          memcpy(dB + ob, GB, sizeof(S) * (size_t)kv);                                    \
          Anext = Am + oa;                                                                \
        }                                                                                 \
        free(GA);                                                                         \
      }                                                                                   \
  }

/* ----------------------------------------------------------------------- */
/* Angle-fused Givens / rotation scan (triton_scans.py:1038-1291; module maths
 * min_gru.py:2583-2599 and 2137-2150). Per (b, block): optionally v[1] *= scale
 * (has_scale), then R rounds v'[p] = cos v[p] + sgn[r,p] sin v[perm[r,p]] with
 * angles theta[b,t,blk,r,p2p[r,p]], then v *= gamma (has_decay), then v += b.
 * Layouts: theta (B,T,n,R,half); scale/gamma (B,T,n); b/out (B,T,n,k);
 * h0 (B,n,k); perm/sgn/p2p (R,k). Backward: exact per-step adjoint reading
 * h_{t-1} from `out` (triton_scans.py:1124-1291).                            */
#define DEF_ANGLE_SCAN(S, SUF)                                                            \
  void orc_angle_scan_fwd_##SUF(const S* theta, const S* scale, const S* gamma,           \
                                const S* bb, const S* h0, const int32_t* perm,            \
                                const S* sgn, const int32_t* p2p, S* out, int64_t B,      \
                                int64_t T, int64_t n, int R, int k, int has_scale,        \
                                int has_decay) {                                          \
    const int half = k / 2;                                                               \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t bi = 0; bi < B; ++bi)                                                    \
      for (int64_t ni = 0; ni < n; ++ni) {                                                \
        S v[64], w[64];                                                                   \
        for (int p = 0; p < k; ++p) v[p] = h0[(bi * n + ni) * k + p];                     \
        for (int64_t t = 0; t < T; ++t) {                                                 \
          const int64_t sc = (bi * T + t) * n + ni;                                       \
          if (has_scale) v[1] *= scale[sc];                                               \
          for (int r = 0; r < R; ++r) {                                                   \
            const S* th = theta + (sc * R + r) * half;                                    \
            for (int p = 0; p < k; ++p) {                                                 \
              const S a = th[p2p[r * k + p]];                                             \
              w[p] = COS_##SUF(a) * v[p] + sgn[r * k + p] * SIN_##SUF(a) * v[perm[r * k + p]]; \
            }                                                                             \
            for (int p = 0; p < k; ++p) v[p] = w[p];                                      \
          }                                                                               \
          if (has_decay)                                                                  \
            for (int p = 0; p < k; ++p) v[p] *= gamma[sc];                                \
          for (int p = 0; p < k; ++p) {                                                   \
            v[p] += bb[sc * k + p];                                                       \
            out[sc * k + p] = v[p];                                                       \
          }                                                                               \
        }                                                                                 \
      }                                                                                   \
  }                                                                                       \
  void orc_angle_scan_bwd_##SUF(const S* theta, const S* scale, const S* gamma,           \
                                const S* h0, const S* out, const S* gout,                 \
                                const int32_t* perm, const S* sgn, const int32_t* p2p,    \
                                S* dtheta, S* dscale, S* dgamma, S* db, S* dh0,           \
                                int64_t B, int64_t T, int64_t n, int R, int k,            \
                                int has_scale, int has_decay) {                           \
    const int half = k / 2;                                                               \
    _Pragma("omp parallel for collapse(2) schedule(static)")                              \
    for (int64_t bi = 0; bi < B; ++bi)                                                    \
      for (int64_t ni = 0; ni < n; ++ni) {                                                \
        S g[64], vv[17][64], a[64], tmp[64];                                              \
        for (int p = 0; p < k; ++p) g[p] = 0;                                             \
        for (int64_t t = T - 1; t >= 0; --t) {                                            \
          const int64_t sc = (bi * T + t) * n + ni;                                       \
          const S* hp = t > 0 ? out + (sc - n) * k : h0 + (bi * n + ni) * k;              \
          for (int p = 0; p < k; ++p) vv[0][p] = hp[p];                                   \
          const S d = has_scale ? scale[sc] : (S)1;                                       \
          if (has_scale) vv[0][1] *= d;                                                   \
          for (int r = 0; r < R; ++r) {                                                   \
            const S* th = theta + (sc * R + r) * half;                                    \
            for (int p = 0; p < k; ++p) {                                                 \
              const S an = th[p2p[r * k + p]];                                            \
              vv[r + 1][p] = COS_##SUF(an) * vv[r][p] +                                   \
                             sgn[r * k + p] * SIN_##SUF(an) * vv[r][perm[r * k + p]];     \
            }                                                                             \
          }                                                                               \
          for (int p = 0; p < k; ++p) {                                                   \
            const S gbar = gout[sc * k + p] + g[p];                                       \
            db[sc * k + p] = gbar;                                                        \
            a[p] = gbar;                                                                  \
          }                                                                               \
          if (has_decay) {                                                                \
            S s = 0;                                                                      \
            for (int p = 0; p < k; ++p) s += a[p] * vv[R][p];                             \
            dgamma[sc] = s;                                                               \
            for (int p = 0; p < k; ++p) a[p] *= gamma[sc];                                \
          } else {                                                                        \
            dgamma[sc] = 0;                                                               \
          }                                                                               \
          for (int r = R - 1; r >= 0; --r) {                                              \
            const S* th = theta + (sc * R + r) * half;                                    \
            S* dth = dtheta + (sc * R + r) * half;                                        \
            for (int m = 0; m < half; ++m) dth[m] = 0;                                    \
            for (int p = 0; p < k; ++p) {                                                 \
              const S an = th[p2p[r * k + p]];                                            \
              const S c = COS_##SUF(an), s = SIN_##SUF(an);                               \
              dth[p2p[r * k + p]] += a[p] * (-s * vv[r][p] + sgn[r * k + p] * c * vv[r][perm[r * k + p]]); \
            }                                                                             \
            for (int p = 0; p < k; ++p) {                                                 \
              const S an = th[p2p[r * k + p]];                                            \
              tmp[p] = COS_##SUF(an) * a[p];                                              \
            }                                                                             \
            for (int p = 0; p < k; ++p) {                                                 \
              const int q = perm[r * k + p];                                              \
              const S anq = th[p2p[r * k + p]];                                           \
              tmp[q] += sgn[r * k + p] * SIN_##SUF(anq) * a[p];                           \
            }                                                                             \
            for (int p = 0; p < k; ++p) a[p] = tmp[p];                                    \
          }                                                                               \
          if (has_scale) {                                                                \
            dscale[sc] = a[1] * hp[1];                                                    \
            a[1] *= d;                                                                    \
          } else {                                                                        \
            dscale[sc] = 0;                                                               \
          }                                                                               \
          for (int p = 0; p < k; ++p) g[p] = a[p];                                        \
        }                                                                                 \
        for (int p = 0; p < k; ++p) dh0[(bi * n + ni) * k + p] = g[p];                    \
      }                                                                                   \
  }

#define EXP_f64 exp
#define EXP_f32 expf
#define COS_f64 cos
#define COS_f32 cosf
#define SIN_f64 sin
#define SIN_f32 sinf

DEF_LOG_SCAN(double, f64)
DEF_LOG_SCAN(float, f32)
DEF_LINEAR_SCAN(double, f64)
DEF_LINEAR_SCAN(float, f32)
DEF_AFFINE_SCAN(double, f64)
DEF_AFFINE_SCAN(float, f32)
DEF_ANGLE_SCAN(double, f64)
DEF_ANGLE_SCAN(float, f32)

int orc_version(void) { return 1; }

/* Thread count of the OpenMP loops (launchers such as torchrun export
 * OMP_NUM_THREADS=1; the CPU baseline wants every host core). */
#ifdef _OPENMP
#include <omp.h>
void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int orc_get_threads(void) { return omp_get_max_threads(); }
#else
void orc_set_threads(int n) { (void)n; }
int orc_get_threads(void) { return 1; }
#endif
