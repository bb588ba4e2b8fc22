// sp.cu -- per-slice carries for sequence parallelism (very long T split over
// ranks in time order).
//
// The reference is single-device. With the sequence split into slices, a rank
// needs only two per-channel summaries of every other slice: the composed
// forward element (the state a slice maps its incoming state to) and the
// composed reverse adjoint element (the adjoint a slice passes to its left).
// These kernels compute them for one slice without writing any output:
//   linear_scan  forward (A, B): x -> A x + B, A = prod a, B = the slice's h_0 = 0 end state
//                reverse (P, Q_A, Q_B): Y -> P Y + Q, P = prod a,
//                        Q = the slice's own adjoint contribution (Y_t = a_t (g_t + Y_{t+1}))
//   parallel_scan_log forward (alpha, nu): x -> logaddexp(x + alpha, nu) over log states
//                reverse (P, Q) of Y_t = a_t (g_t + Y_{t+1}), a = exp(log a)
// Each slice's summaries are all-gathered; a rank composes the earlier
// slices' forward summaries into the state its slice starts from and the later
// slices' reverse summaries into the adjoint entering from its right, and the
// *_fixup entry points (linear_scan.cu, log_scan.cu) then scan the slice from
// those carries inside the scan kernels.
//
// Layout: a segmented reduction. Thread = one (b, d) channel of one time
// segment (consecutive threads = consecutive channels, so every step is a
// coalesced row read), then one thread per channel combines the segments in
// time order. Reads each input once; writes NF floats per channel.
#include "common.cuh"

namespace mgs {
namespace sp {

constexpr int kThreads = 256;

__device__ __forceinline__ float logaddexp_f(float p, float q) {
  const float m = fmaxf(p, q);
  if (m == -INFINITY || m == INFINITY) return m;
  return m + log1pf(expf(fminf(p, q) - m));
}

// Forward ops walk t = t0 .. t1-1; reverse ops walk t = t1-1 .. t0.
// compose(x, y, o): x applied first, then y (forward: x earlier in time;
// reverse: x later in time).
struct LinFwd {
  static constexpr int NF = 2;
  static constexpr bool kReverse = false;
  __device__ static void ident(float* x) { x[0] = 1.f; x[1] = 0.f; }
  template <typename E>
  __device__ static void step(float* x, const E* const* in, size_t i, size_t, long long) {
    const float a = to_f32<E>(in[0][i]);
    x[1] = fmaf(a, x[1], to_f32<E>(in[1][i]));
    x[0] *= a;
  }
  __device__ static void compose(const float* x, const float* y, float* o) {
    o[1] = fmaf(y[0], x[1], y[1]);
    o[0] = y[0] * x[0];
  }
};

struct LinRev {
  static constexpr int NF = 3;
  static constexpr bool kReverse = true;
  __device__ static void ident(float* x) { x[0] = 1.f; x[1] = 0.f; x[2] = 0.f; }
  template <typename E>
  __device__ static void step(float* x, const E* const* in, size_t i, size_t, long long) {
    const float a = to_f32<E>(in[0][i]);
    x[1] = a * (to_f32<E>(in[1][i]) + x[1]);
    x[2] = a * (to_f32<E>(in[2][i]) + x[2]);
    x[0] *= a;
  }
  __device__ static void compose(const float* x, const float* y, float* o) {
    o[1] = fmaf(y[0], x[1], y[1]);
    o[2] = fmaf(y[0], x[2], y[2]);
    o[0] = y[0] * x[0];
  }
};

// log values are (B, T+1, D): step t reads row t+1 (`i1`).
struct LogFwd {
  static constexpr int NF = 2;
  static constexpr bool kReverse = false;
  __device__ static void ident(float* x) { x[0] = 0.f; x[1] = -INFINITY; }
  template <typename E>
  __device__ static void step(float* x, const E* const* in, size_t i, size_t i1, long long) {
    const float c = to_f32<E>(in[0][i]);
    x[1] = logaddexp_f(x[1] + c, to_f32<E>(in[1][i1]));
    x[0] += c;
  }
  __device__ static void compose(const float* x, const float* y, float* o) {
    o[1] = logaddexp_f(x[1] + y[0], y[1]);
    o[0] = x[0] + y[0];
  }
};

struct LogRev {
  static constexpr int NF = 2;
  static constexpr bool kReverse = true;
  __device__ static void ident(float* x) { x[0] = 1.f; x[1] = 0.f; }
  template <typename E>
  __device__ static void step(float* x, const E* const* in, size_t i, size_t, long long) {
    const float a = expf(to_f32<E>(in[0][i]));
    x[1] = a * (to_f32<E>(in[1][i]) + x[1]);
    x[0] *= a;
  }
  __device__ static void compose(const float* x, const float* y, float* o) {
    o[1] = fmaf(y[0], x[1], y[1]);
    o[0] = y[0] * x[0];
  }
};

struct Ins {
  const void* p[3];
};

template <typename E, class Op>
__global__ void __launch_bounds__(kThreads) segment_kernel(Ins ins, float* part, long long B,
                                                           long long T, long long D, int nseg) {
  const long long BD = B * D;
  const long long ch = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= BD) return;
  const int seg = blockIdx.y;
  const long long len = (T + nseg - 1) / nseg;
  const long long t0 = (long long)seg * len, t1 = t0 + len < T ? t0 + len : T;
  const long long b = ch / D, d = ch - b * D;
  const E* in[3] = {static_cast<const E*>(ins.p[0]), static_cast<const E*>(ins.p[1]),
                    static_cast<const E*>(ins.p[2])};
  float x[Op::NF];
  Op::ident(x);
  for (long long k = 0; k < t1 - t0; ++k) {
    const long long t = Op::kReverse ? t1 - 1 - k : t0 + k;
    Op::template step<E>(x, in, (size_t)((b * T + t) * D + d), (size_t)((b * (T + 1) + t + 1) * D + d),
                         t);
  }
#pragma unroll
  for (int f = 0; f < Op::NF; ++f) part[((size_t)seg * Op::NF + f) * BD + ch] = x[f];
}

template <class Op>
__global__ void __launch_bounds__(kThreads) combine_kernel(const float* part, float* agg,
                                                           long long BD, int nseg) {
  const long long ch = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= BD) return;
  float x[Op::NF], y[Op::NF], o[Op::NF];
  Op::ident(x);
  for (int k = 0; k < nseg; ++k) {
    const int seg = Op::kReverse ? nseg - 1 - k : k;
#pragma unroll
    for (int f = 0; f < Op::NF; ++f) y[f] = part[((size_t)seg * Op::NF + f) * BD + ch];
    Op::compose(x, y, o);
#pragma unroll
    for (int f = 0; f < Op::NF; ++f) x[f] = o[f];
  }
#pragma unroll
  for (int f = 0; f < Op::NF; ++f) agg[(size_t)f * BD + ch] = x[f];
}

inline int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

// Time segments: enough (channel, segment) threads to fill the GPU, at least
// 16 steps per segment.
inline int segments(long long B, long long T, long long D) {
  const long long BD = B * D, want = 2048LL * sm_count();
  long long n = BD > 0 ? (want + BD - 1) / BD : 1;
  const long long cap = T / 16 > 1 ? T / 16 : 1;
  if (n > cap) n = cap;
  if (n > 4096) n = 4096;
  return (int)(n < 1 ? 1 : n);
}

inline size_t workspace_bytes(long long B, long long T, long long D) {
  const size_t n = (size_t)segments(B, T, D) * 3 * (size_t)(B * D) * sizeof(float);
  return n < 256 ? 256 : n;
}

template <typename E, class Op>
int run(Ins ins, float* agg, long long B, long long T, long long D, void* ws, size_t ws_bytes,
        cudaStream_t st) {
  const long long BD = B * D;
  if (BD == 0) return MGS_OK;
  if (agg == nullptr || !aligned(agg, 4)) return MGS_BAD_ALIGNMENT;
  if (T == 0) {  // an empty slice: the identity element (combining zero segments)
    combine_kernel<Op><<<(unsigned)((BD + kThreads - 1) / kThreads), kThreads, 0, st>>>(
        nullptr, agg, BD, 0);
    return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
  }
  const int nseg = segments(B, T, D);
  if (ws == nullptr || ws_bytes < (size_t)nseg * Op::NF * BD * sizeof(float))
    return MGS_WORKSPACE_TOO_SMALL;
  float* part = static_cast<float*>(ws);
  const dim3 grid((unsigned)((BD + kThreads - 1) / kThreads), (unsigned)nseg);
  segment_kernel<E, Op><<<grid, kThreads, 0, st>>>(ins, part, B, T, D, nseg);
  if (cudaGetLastError() != cudaSuccess) return MGS_LAUNCH_FAILED;
  combine_kernel<Op><<<(unsigned)((BD + kThreads - 1) / kThreads), kThreads, 0, st>>>(part, agg, BD,
                                                                                        nseg);
  return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED;
}

template <class Op>
int dispatch(Ins ins, float* agg, long long B, long long T, long long D, int dtype, void* ws,
             size_t ws_bytes, cudaStream_t st) {
  if (B < 0 || T < 0 || D < 0) return MGS_BAD_SHAPE;
  switch (dtype) {
    case MGS_F32: return run<float, Op>(ins, agg, B, T, D, ws, ws_bytes, st);
    case MGS_BF16: return run<__nv_bfloat16, Op>(ins, agg, B, T, D, ws, ws_bytes, st);
    case MGS_F16: return run<__half, Op>(ins, agg, B, T, D, ws, ws_bytes, st);
    default: return MGS_BAD_DTYPE;
  }
}

}  // namespace sp
}  // namespace mgs

extern "C" {

size_t mgs_scan_carry_workspace_size(int64_t B, int64_t T, int64_t D) {
  if (B < 0 || T < 0 || D < 0) return 0;
  return mgs::sp::workspace_bytes(B, T, D);
}

int mgs_linear_scan_carry_fwd(const void* a, const void* b, float* carry, int64_t B, int64_t T,
                              int64_t D, int dtype, void* workspace, size_t workspace_bytes,
                              void* stream) {
  return mgs::sp::dispatch<mgs::sp::LinFwd>({{a, b, nullptr}}, carry, B, T, D, dtype, workspace,
                                            workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mgs_linear_scan_carry_bwd(const void* a, const void* gA, const void* gBc, float* carry,
                              int64_t B, int64_t T, int64_t D, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return mgs::sp::dispatch<mgs::sp::LinRev>({{a, gA, gBc}}, carry, B, T, D, dtype, workspace,
                                            workspace_bytes, static_cast<cudaStream_t>(stream));
}

int mgs_log_scan_carry_fwd(const void* log_coeffs, const void* log_values, float* carry, int64_t B,
                           int64_t T, int64_t D, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  return mgs::sp::dispatch<mgs::sp::LogFwd>({{log_coeffs, log_values, nullptr}}, carry, B, T, D,
                                            dtype, workspace, workspace_bytes,
                                            static_cast<cudaStream_t>(stream));
}

int mgs_log_scan_carry_bwd(const void* log_coeffs, const void* grad_h, float* carry, int64_t B,
                           int64_t T, int64_t D, int dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  return mgs::sp::dispatch<mgs::sp::LogRev>({{log_coeffs, grad_h, nullptr}}, carry, B, T, D, dtype,
                                            workspace, workspace_bytes,
                                            static_cast<cudaStream_t>(stream));
}

}  // extern "C"
