/*
 * mingru_scan.h -- C ABI of the B200 (sm_100a) scan kernels behind the mingru
 * scan family.
 *
 * Every entry point takes plain device pointers, int64 sizes, a dtype code, a
 * caller-owned workspace and a CUDA stream (as `void*`), and returns an
 * `mgs_status`. Nothing here allocates device memory, synchronises the host
 * or keeps per-call global state: outputs, gradients, saved carries and
 * workspaces are allocated by the caller (the torch extension uses torch's
 * caching allocator on the current stream). All tensors are dense, C-ordered
 * and 16-byte aligned where the kernels vectorise; the wrappers check this
 * and return MGS_BAD_ALIGNMENT / MGS_BAD_SHAPE instead of launching.
 *
 * Each function cites the reference interface it replaces (paths are inside
 * the chris-santiago/minGRU project, package `mingru`, files
 * src/mingru/min_gru.py = "min_gru.py" and src/mingru/triton_scans.py =
 * "triton_scans.py").
 */
#ifndef MINGRU_SCAN_H
#define MINGRU_SCAN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference signals a declined kernel with
 * `ScanFallback` (triton_scans.py:166) and silently runs eager; this ABI has
 * no fallback: every failure is returned and raised by the caller. */
typedef enum mgs_status {
  MGS_OK = 0,
  MGS_BAD_SHAPE = 1,          /* inconsistent / negative sizes            */
  MGS_BAD_DTYPE = 2,          /* dtype code not supported by this op      */
  MGS_BAD_ALIGNMENT = 3,      /* a pointer is not aligned as required     */
  MGS_UNSUPPORTED = 4,        /* shape outside the kernel envelope        */
  MGS_LAUNCH_FAILED = 5,      /* cudaLaunch / cudaMemsetAsync error       */
  MGS_LOOKBACK_TIMEOUT = 6,   /* a decoupled look-back wait hit its bound */
  MGS_WORKSPACE_TOO_SMALL = 7 /* workspace / carry buffer under-sized     */
} mgs_status;

/* Element type of the tensors an op reads and writes. Arithmetic and every
 * carried state are fp32 regardless (the reference kernels load, upcast to
 * fp32, accumulate in fp32 and store in the input dtype: triton_scans.py:1312). */
typedef enum mgs_dtype { MGS_F32 = 0, MGS_BF16 = 1, MGS_F16 = 2 } mgs_dtype;

/* Library version (major*10000 + minor*100 + patch). */
int mgs_version(void);

/* Human-readable name of a status code (static storage). */
const char* mgs_status_string(int status);

/* Sticky device-side error word of the current device (look-back timeouts).
 * Synchronises `stream`, returns the accumulated MGS_* bits (0 if clean) and
 * clears them. Kernels never trap: a bounded wait that runs out records
 * MGS_LOOKBACK_TIMEOUT here and lets the launch finish. */
int mgs_take_device_error(void* stream);

/* ------------------------------------------------------------------------ */
/* linear_scan: h_t = a_t * h_{t-1} + b_t, returns (A, Bc) with
 * A_t = prod_{s<=t} a_s and Bc_t the h_0 = 0 solution.
 * Replaces min_gru.py:1454 `linear_scan(a, b)` (eager doubling at
 * min_gru.py:1501-1510) and its Triton kernels triton_scans.py:702-751
 * (forward) / 961-1036 (backward), ops linear_scan_fwd / linear_scan_bwd
 * (triton_scans.py:1318, 1392) and their autograd (triton_scans.py:1465-1487).
 * Layout: a, b, A, Bc, da, db, gA, gBc are (B, T, D) C-contiguous.           */

/* Bytes of look-back workspace one forward or backward call needs. */
size_t mgs_linear_scan_workspace_size(int64_t B, int64_t T, int64_t D, int dtype);
/* Bytes of the forward carries the backward consumes (fp32 chunk-start
 * states, a few percent of one input tensor). */
size_t mgs_linear_scan_carry_size(int64_t B, int64_t T, int64_t D, int dtype);

/* Forward. `carries` may be NULL (no backward will follow). */
int mgs_linear_scan_fwd(const void* a, const void* b, void* A, void* Bc,
                        void* carries, int64_t B, int64_t T, int64_t D,
                        int dtype, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Backward: given the forward inputs (a, b), the carries the forward wrote
 * and the output grads (gA, gBc), write (da, db). Recomputes A_{t-1},
 * Bc_{t-1} in registers from the carries instead of reading saved outputs. */
int mgs_linear_scan_bwd(const void* a, const void* b, const void* gA,
                        const void* gBc, const void* carries, void* da,
                        void* db, int64_t B, int64_t T, int64_t D, int dtype,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Size of the fixed device scratch behind mgs_linear_scan_fwd_noalloc. */
#define MGS_NOALLOC_SCRATCH_BYTES (32u << 20)

/* linear_scan forward that allocates nothing. No counterpart in the reference
 * (which has no C ABI); it exists for callers that cannot hand the library a
 * workspace -- code inside a region where allocation is forbidden or would
 * synchronise (a latency-critical serving loop, a pre-reserved memory pool,
 * an FFI host with no device allocator of its own). Same arguments and
 * results as mgs_linear_scan_fwd minus the workspace: the look-back scratch
 * lives in a file-scope device array of MGS_NOALLOC_SCRATCH_BYTES that every
 * GPU which loads the library keeps until the process exits.
 *  - The first call on a device resolves that array's device address (with
 *    the device current); make that first call before any stream capture.
 *  - Every call on a device shares the one array; the call clears what must
 *    start at zero. Calls whose executions overlap on the GPU (other streams,
 *    other host threads) race on it: serialise them.
 *  - Shapes whose scratch would exceed MGS_NOALLOC_SCRATCH_BYTES return
 *    MGS_WORKSPACE_TOO_SMALL (use mgs_linear_scan_fwd for those). */
int mgs_linear_scan_fwd_noalloc(const void* a, const void* b, void* A, void* Bc, void* carries,
                                int64_t B, int64_t T, int64_t D, int dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* Sequence-parallel helpers (the sequence split over ranks in time order).
 * No counterpart in the reference (single-device); they replace the
 * full-tensor fix-up a sharded scan would otherwise need.
 *  - *_carry_fwd: one read-only pass over a slice; writes per channel the
 *    slice's composed forward element, fp32 (NF, B, D): linear (A, B) with
 *    x -> A x + B; log (alpha, nu) with x -> logaddexp(x + alpha, nu) over
 *    rows 1..T of log_values.
 *  - *_carry_bwd: the slice's composed reverse adjoint element, fp32: linear
 *    (P, Q_A, Q_B), log (P, Q), with Y -> P Y + Q the adjoint the slice passes
 *    to its left given the one entering from its right.
 *  - *_fwd_fixup / *_bwd_fixup: the scans of mgs_linear_scan_* and
 *    mgs_log_scan_* started from a carried-in state (linear: carry_in
 *    (2, B, D) = (A_in, B_in); log: log_h_in (B, D) in place of
 *    log_values[:, 0]) and, backward, from the adjoints entering from the
 *    right (linear (2, B, D), log (B, D)): every output is the full-length
 *    scan's, with no separate fix-up pass.
 * Workspace of the *_carry_* calls: mgs_scan_carry_workspace_size bytes.   */
size_t mgs_scan_carry_workspace_size(int64_t B, int64_t T, int64_t D);
int mgs_linear_scan_carry_fwd(const void* a, const void* b, float* carry, int64_t B, int64_t T,
                              int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                              void* stream);
int mgs_linear_scan_carry_bwd(const void* a, const void* gA, const void* gBc, float* carry,
                              int64_t B, int64_t T, int64_t D, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream);
int mgs_linear_scan_fwd_fixup(const void* a, const void* b, const float* carry_in, void* A,
                              void* Bc, void* carries, int64_t B, int64_t T, int64_t D, int dtype,
                              void* workspace, size_t workspace_bytes, void* stream);
int mgs_linear_scan_bwd_fixup(const void* a, const void* b, const void* gA, const void* gBc,
                              const void* carries, const float* adjoint_in, void* da, void* db,
                              int64_t B, int64_t T, int64_t D, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream);
int mgs_log_scan_carry_fwd(const void* log_coeffs, const void* log_values, float* carry, int64_t B,
                           int64_t T, int64_t D, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream);
int mgs_log_scan_carry_bwd(const void* log_coeffs, const void* grad_h, float* carry, int64_t B,
                           int64_t T, int64_t D, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream);
int mgs_log_scan_fwd_fixup(const void* log_coeffs, const void* log_values, const float* log_h_in,
                           void* h, void* carries, int64_t B, int64_t T, int64_t D, int dtype,
                           void* workspace, size_t workspace_bytes, void* stream);
int mgs_log_scan_bwd_fixup(const void* log_coeffs, const void* log_values, const float* log_h_in,
                           const void* grad_h, const void* carries, const float* adjoint_in,
                           void* dlog_coeffs, void* dlog_values, int64_t B, int64_t T, int64_t D,
                           int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Time-out test hooks. No counterpart in the reference (its Triton kernels
 * have no cross-CTA waits). Each makes one bounded device-side wait run out
 * on purpose, with a poll bound of `spin_limit`, so that a test can check the
 * time-out path end to end: the launch completes, the error words carry
 * MGS_LOOKBACK_TIMEOUT, mgs_take_device_error reports it and the context
 * stays usable. Nothing here can hang: every wait involved is bounded.
 *
 * mgs_test_lookback_timeout: the fp32 linear_scan forward on its look-back
 * path (shapes too narrow for the strip path, T > 64) with the tile counter
 * started at 1, so the look-back behind tile 0 waits on a flag that nothing
 * sets; the workspace header's error word (offset 4) receives the bit.
 * Returns MGS_UNSUPPORTED for shapes that do not take that path. Outputs of
 * the first tile are left unwritten.
 * mgs_test_mbarrier_timeout: one CTA waits on an mbarrier nothing arrives on;
 * `err_word` (device u32) receives the bit.                                   */
int mgs_test_lookback_timeout(const void* a, const void* b, void* A, void* Bc, int64_t B,
                              int64_t T, int64_t D, void* workspace, size_t workspace_bytes,
                              int64_t spin_limit, void* stream);
int mgs_test_mbarrier_timeout(void* err_word, int64_t spin_limit, void* stream);

/* ------------------------------------------------------------------------ */
/* parallel_scan_log: h_t = a_t h_{t-1} + b_t in log space, a_t =
 * exp(log_coeffs[:, t-1]), b_t = exp(log_values[:, t]), h_0 =
 * exp(log_values[:, 0]); returns h_1..h_T.
 * Replaces min_gru.py:755 `parallel_scan_log(log_coeffs, log_values)`
 * (eager cumsum + logcumsumexp, min_gru.py:804-807), its Triton forward
 * triton_scans.py:753-821 / op parallel_scan_log_fwd (triton_scans.py:1336)
 * and its recompute-through-eager backward (triton_scans.py:1489-1552).
 * Layout: log_coeffs, h, grad_h, dlog_coeffs (B, T, D); log_values,
 * dlog_values (B, T+1, D); all C-contiguous.                                 */

size_t mgs_log_scan_workspace_size(int64_t B, int64_t T, int64_t D, int dtype);
size_t mgs_log_scan_carry_size(int64_t B, int64_t T, int64_t D, int dtype);

int mgs_log_scan_fwd(const void* log_coeffs, const void* log_values, void* h, void* carries,
                     int64_t B, int64_t T, int64_t D, int dtype, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Backward: (dlog_coeffs, dlog_values) of sum(h * grad_h), recomputing the
 * log-states from the forward carries (hand-derived adjoint, no autograd). */
int mgs_log_scan_bwd(const void* log_coeffs, const void* log_values, const void* grad_h,
                     const void* carries, void* dlog_coeffs, void* dlog_values, int64_t B,
                     int64_t T, int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ------------------------------------------------------------------------ */
/* MinGRU gate scan: parallel_scan_log fed straight from MinGRU's
 * pre-activations. Replaces the coefficient prologue of MinGRU.forward
 * (min_gru.py:1383-1397: log_coeffs = -softplus(k), log_values =
 * cat[log h_0, -softplus(-k) + log_g(x~)], log_g at min_gru.py:751-752)
 * followed by parallel_scan_log (min_gru.py:1394). k = linear_z(x),
 * x~ = linear_h(x), h, dk, dx~ are (B, T, D); log_h0, dlog_h0 are (B, D).
 * fp32 shapes on the parallel_scan_log column path form the log
 * coefficients in shared memory (they never exist in HBM); other shapes and
 * 16-bit storage form them in the workspace with one elementwise kernel.
 * The backward returns dk, dx~ and dlog_h0 directly.                       */

size_t mgs_log_gate_scan_workspace_size(int64_t B, int64_t T, int64_t D, int dtype);
size_t mgs_log_gate_scan_carry_size(int64_t B, int64_t T, int64_t D, int dtype);

int mgs_log_gate_scan_fwd(const void* k, const void* x, const void* log_h0, void* h, void* carries,
                          int64_t B, int64_t T, int64_t D, int dtype, void* workspace,
                          size_t workspace_bytes, void* stream);

int mgs_log_gate_scan_bwd(const void* k, const void* x, const void* log_h0, const void* grad_h,
                          const void* carries, void* dk, void* dx, void* dlog_h0, int64_t B,
                          int64_t T, int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ------------------------------------------------------------------------ */
/* matrix_affine_scan / matrix_scan: H_t = A_t H_{t-1} + B_t per block,
 * A (B, T, n, k, k), Bm (B, T, n, k, v); returns Abar_t (running product,
 * Abar_0 = I) and Bbar_t (the H_0 = 0 solution). matrix_scan is k = 2, v = 1
 * with b (B, T, n, 2) viewed as (B, T, n, 2, 1).
 * Replaces min_gru.py:1584 `matrix_affine_scan(A, Bm)` and min_gru.py:1513
 * `matrix_scan(M, b)` (eager doubling, min_gru.py:1570-1581, 1647-1655), the
 * Triton kernels triton_scans.py:629-700 / 823-959, ops affine_scan_fwd /
 * affine_scan_bwd (triton_scans.py:1293, 1359) and the SCAN_IMPLS wrappers
 * (triton_scans.py:2492-2563). k, v in {1, 2, 4, 8, 16} with k (k + v) <= 72
 * use register-resident look-back kernels; any other 1 <= k, v <= 64 uses a
 * sequential per-block kernel whose backward reads the saved outputs.       */

size_t mgs_affine_scan_workspace_size(int64_t B, int64_t T, int64_t n, int k, int v, int dtype);
/* 0 when the (k, v) uses the sequential kernels: then the backward needs
 * Abar, Bbar (the saved forward outputs) instead of carries. */
size_t mgs_affine_scan_carry_size(int64_t B, int64_t T, int64_t n, int k, int v, int dtype);

int mgs_affine_scan_fwd(const void* A, const void* Bm, void* Abar, void* Bbar, void* carries,
                        int64_t B, int64_t T, int64_t n, int k, int v, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Backward: (dA, dBm) of sum(Abar * gAbar) + sum(Bbar * gBbar). Abar/Bbar may
 * be NULL when carries are used (register path). */
int mgs_affine_scan_bwd(const void* A, const void* Bm, const void* Abar, const void* Bbar,
                        const void* gAbar, const void* gBbar, const void* carries, void* dA,
                        void* dBm, int64_t B, int64_t T, int64_t n, int k, int v, int dtype,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Angle-fused Givens / rotation scan (GivensMinGRU, RotationMinGRU).
 * Per (b, block): [v[1] *= scale], R rounds of plane rotations
 * v'[p] = cos v[p] + sgn[r,p] sin v[perm[r,p]] with angle
 * theta[b,t,blk,r,p2p[r,p]], [v *= gamma], v += b; h_t = v.
 * Layouts: theta (B, T, n, R, k/2); scale, gamma (B, T, n); b, h (B, T, n, k);
 * h0 (B, n, k); perm, p2p int32 (R, k); sgn float32 (R, k) -- device memory.
 * Replaces angle_scan_impl (triton_scans.py:1743-1812), the ops angle_scan_fwd /
 * angle_scan_bwd (triton_scans.py:1579-1704) and their Triton kernels
 * (triton_scans.py:1038-1291), called from GivensMinGRU / RotationMinGRU
 * (min_gru.py:2727-2774, 2269-2314).
 * `brickwall` != 0 states that perm/sgn/p2p are the brick-wall layout both
 * mixers build (round r pairs (i, i+1 mod k), i = r%2, r%2+2, ...; sgn -1 on
 * i, +1 on i+1; p2p = plane index): k in {2, 4, 8} with R <= 4 then runs the
 * register look-back kernels, which derive the planes from (k, r) and do not
 * read the metadata. Otherwise (or brickwall == 0) a sequential per-block
 * kernel reads the metadata; its backward reads the stored states `h`.    */

size_t mgs_angle_scan_workspace_size(int64_t B, int64_t T, int64_t n, int R, int k,
                                     int brickwall, int dtype);
/* Register look-back kernels: k*k floats per block and time tile (the linear
 * part of each forward tile aggregate, which the backward reuses transposed);
 * a forward that will be differentiated passes a buffer of this size as
 * `carries` (NULL otherwise) and the backward gets the same buffer back.
 * 0 when the sequential kernels are used. */
size_t mgs_angle_scan_carry_size(int64_t B, int64_t T, int64_t n, int R, int k, int brickwall,
                                 int dtype);

int mgs_angle_scan_fwd(const void* theta, const void* scale, const void* gamma, const void* b,
                       const void* h0, const int32_t* perm, const float* sgn, const int32_t* p2p,
                       void* h, void* carries, int64_t B, int64_t T, int64_t n, int R, int k,
                       int has_scale, int has_decay, int brickwall, int dtype, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Backward: (dtheta, dscale, dgamma, db, dh0) of sum(h * grad_h). dscale /
 * dgamma are written only when has_scale / has_decay (the caller zeroes them
 * otherwise). Both paths read the stored states `h`; the register path also
 * needs the forward's `carries`. */
int mgs_angle_scan_bwd(const void* theta, const void* scale, const void* gamma, const void* b,
                       const void* h0, const int32_t* perm, const float* sgn, const int32_t* p2p,
                       const void* h, const void* grad_h, const void* carries, void* dtheta,
                       void* dscale, void* dgamma, void* db, void* dh0, int64_t B, int64_t T,
                       int64_t n, int R, int k, int has_scale, int has_decay, int brickwall,
                       int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* DeltaMinGRU chunked-WY delta rule (decay off).
 * Q (B, H, T, dk); K (B, H, T, nh, dk); V (B, H, T, nh, dv); beta (B, H, T, nh)
 * in the op dtype; H0, H_T (B, H, dk, dv) fp32; y (B, H, T, dv) op dtype.
 * Per chunk of `chunk` tokens (M = nh * chunk micro-steps):
 *   T = I + strict_lower(K K^T) * beta[col];  U = T^{-1} (V - K S);
 *   y = Q S + ((Q K^T) * beta[col] * read_mask) U;  S <- S + K^T (beta * U).
 * Replaces delta_scan_impl (triton_scans.py:2403-2447) -- the Triton forward
 * trio (triton_scans.py:1859-2322), _DeltaScanFn (triton_scans.py:2324-2401)
 * and the torch backward _delta_backward_torch (triton_scans.py:473-605) --
 * called from DeltaMinGRU._delta_fused_forward (min_gru.py:3565-3609); eager
 * oracle DeltaMinGRU._forward_chunked (min_gru.py:3152-3255).
 * Envelope: dk <= 128, dv <= 64 (wider d_v runs as independent column blocks,
 * one call each), any chunk >= 1 and nh whose one-token chunk fits shared
 * memory. The chunked form is exact for any chunk length, so the kernels may
 * run shorter chunks than `chunk` (whole tokens; nh * chunk <= 64 on the
 * tensor-core kernels, which bf16 and fp32 inputs with dk, dv <= 64, multiples
 * of 8, take): results differ only by rounding. The size queries return 0
 * outside the envelope and the entry points MGS_UNSUPPORTED.
 * `saved` (mgs_delta_saved_size bytes) is written by the forward and read by
 * the backward (chunk-start states and per-chunk maps; its layout depends on
 * the path the size query picked for these arguments).                     */

size_t mgs_delta_saved_size(int64_t B, int H, int64_t T, int nh, int dk, int dv, int chunk,
                            int dtype);
size_t mgs_delta_workspace_size(int64_t B, int H, int64_t T, int nh, int dk, int dv, int chunk,
                                int dtype);

int mgs_delta_fwd(const void* Q, const void* K, const void* V, const void* beta, const float* H0,
                  void* y, float* H_T, void* saved, int64_t B, int H, int64_t T, int nh, int dk,
                  int dv, int chunk, int dtype, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Backward: (dQ, dK, dV, dbeta, dH0) of sum(y * dy) + sum(H_T * dH_T). */
int mgs_delta_bwd(const void* Q, const void* K, const void* V, const void* beta, const void* saved,
                  const void* dy, const float* dH_T, void* dQ, void* dK, void* dV, void* dbeta,
                  float* dH0, int64_t B, int H, int64_t T, int nh, int dk, int dv, int chunk,
                  int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* DeltaMinGRU with per-token time decay (decay active). Same layouts as
 * mgs_delta_*, plus log_gamma (B, H, T) fp32: the per-token log decay
 * -lambda * dt (<= 0) of each head; the backward also writes dlog_gamma
 * (B, H, T) fp32. Replaces DeltaMinGRU._forward_chunked_gated
 * (min_gru.py:3290-3448) and its span sums _span_log_decay
 * (min_gru.py:3257-3288), which the reference runs eagerly only (its Triton
 * path declines decay). The incoming state of each token decays by
 * gamma_t = exp(log_gamma_t) before the token's nh micro-steps; every decay
 * factor is exp of a chunk-relative span sum of log_gamma (no division, no
 * difference of running sums). CUDA-core kernels (fp32 arithmetic) for every
 * dtype; envelope as mgs_delta_* (the shared-memory budget picks the chunk). */
size_t mgs_delta_gated_saved_size(int64_t B, int H, int64_t T, int nh, int dk, int dv, int chunk,
                                  int dtype);
size_t mgs_delta_gated_workspace_size(int64_t B, int H, int64_t T, int nh, int dk, int dv,
                                      int chunk, int dtype);
int mgs_delta_gated_fwd(const void* Q, const void* K, const void* V, const void* beta,
                        const float* H0, const float* log_gamma, void* y, float* H_T, void* saved,
                        int64_t B, int H, int64_t T, int nh, int dk, int dv, int chunk, int dtype,
                        void* workspace, size_t workspace_bytes, void* stream);
int mgs_delta_gated_bwd(const void* Q, const void* K, const void* V, const void* beta,
                        const float* log_gamma, const void* saved, const void* dy,
                        const float* dH_T, void* dQ, void* dK, void* dV, void* dbeta, float* dH0,
                        float* dlog_gamma, int64_t B, int H, int64_t T, int nh, int dk, int dv,
                        int chunk, int dtype, void* workspace, size_t workspace_bytes,
                        void* stream);

/* ------------------------------------------------------------------------ */
/* Streaming step: one token's recurrence update per mixer, one kernel each.
 * Replaces the per-token torch op chains of MinGRU.step (min_gru.py:1399-1448),
 * SignedMinGRU.step (min_gru.py:1858-1901), RotationMinGRU.step
 * (min_gru.py:2316-2359), GivensMinGRU.step (min_gru.py:2776-2818) and
 * DeltaMinGRU.step (min_gru.py:3611-3688), which MinGRUStack.step
 * (min_gru.py:4289-4336) calls per layer. Inputs are the outputs of the
 * mixers' linear projections (pre-activations) and the previous state, all in
 * the op dtype, C-contiguous; `gamma` (the decay factor exp(-lambda dt) at the
 * state's granularity) may be NULL (no decay). The new state may overwrite
 * the previous one (same pointer). fp32 arithmetic.
 *   mingru:   k, xh, h_prev, gamma, h (B, D):
 *             h = gamma (1 - sigmoid(k)) h_prev + sigmoid(k) g(xh)
 *   signed:   z, s, xh, h_prev, gamma, h (B, D):
 *             h = gamma tanh(s) [(1 - sigmoid(z)) if coupled] h_prev + sigmoid(z) xh
 *   rotation: theta, u, gamma (B, n); z, xh, h_prev, h (B, 2n):
 *             per block h = gamma R(theta) diag(1, tanh u) h_prev + sigmoid(z) xh
 *   givens:   theta (B, n, R, k/2); gamma (B, n); z, xh, h_prev, h (B, n*k),
 *             k in {2, 4, 8, 16, 32, 64}: R brick-wall rounds, gamma, + sigmoid(z) xh
 *   delta:    q (B, H, dk), k (B, H, nh, dk), v (B, H, nh, dv), beta (B, H, nh),
 *             gamma (B, H), H_prev, H (B, H, dk, dv), y (B, H, dv):
 *             H = gamma H_prev; per micro-step H += beta k (v - k^T H)^T; y = H^T q */
int mgs_mingru_step(const void* k, const void* xh, const void* h_prev, const void* gamma, void* h,
                    int64_t B, int64_t D, int dtype, void* stream);
int mgs_signed_step(const void* z, const void* s, const void* xh, const void* h_prev,
                    const void* gamma, int coupled, void* h, int64_t B, int64_t D, int dtype,
                    void* stream);
int mgs_rotation_step(const void* theta, const void* u, const void* z, const void* xh,
                      const void* h_prev, const void* gamma, void* h, int64_t B, int64_t n,
                      int dtype, void* stream);
int mgs_givens_step(const void* theta, const void* z, const void* xh, const void* h_prev,
                    const void* gamma, void* h, int64_t B, int64_t n, int R, int k, int dtype,
                    void* stream);
int mgs_delta_step(const void* q, const void* k, const void* v, const void* beta, const void* gamma,
                   const void* H_prev, void* y, void* H, int64_t B, int heads, int nh, int dk,
                   int dv, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINGRU_SCAN_H */
