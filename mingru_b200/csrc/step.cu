// step.cu -- fused per-token recurrence updates for the mixers' step() (the
// O(1)-per-token streaming / decoding path).
//
// Reference behaviour: MinGRU.step (min_gru.py:1399-1448), SignedMinGRU.step
// (min_gru.py:1858-1901), RotationMinGRU.step (min_gru.py:2316-2359),
// GivensMinGRU.step (min_gru.py:2776-2818) and DeltaMinGRU.step
// (min_gru.py:3611-3688); MinGRUStack.step (min_gru.py:4289-4336) calls them
// layer by layer. In the reference each step is a chain of small torch ops
// (sigmoid, tanh, products, rotations, per-micro-step einsums), one launch
// each; here the whole recurrence update of one token is one kernel. The
// linear projections that feed it stay GEMMs (cuBLAS through torch); these
// kernels take their outputs (the pre-activations) and the previous state.
//
// All arithmetic is fp32; inputs, states and outputs are in the op dtype.
// The output may alias the previous state (each element, or each delta
// state column, is read by the thread that writes it, before it is written).
#include "common.cuh"

namespace mgs {
namespace step {

constexpr int kThreads = 256;

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }

// g(x) = x + 1/2 (x >= 0), sigmoid(x) (x < 0)   (min_gru.py:723)
__device__ __forceinline__ float g_act(float x) { return x >= 0.f ? x + 0.5f : sigm(x); }

inline unsigned blocks_for(long long n) {
  long long b = (n + kThreads - 1) / kThreads;
  if (b < 1) b = 1;
  if (b > 65535LL * 4) b = 65535LL * 4;
  return (unsigned)b;
}

// MinGRU: h = gamma (1 - z) h_prev + z g(x~), z = sigmoid(k).
template <typename E>
__global__ void __launch_bounds__(kThreads) mingru_kernel(const E* k, const E* xh, const E* hp,
                                                          const E* gamma, E* h, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float z = sigm(to_f32<E>(k[i]));
    float a = 1.f - z;
    if (gamma) a *= to_f32<E>(gamma[i]);
    h[i] = from_f32<E>(fmaf(a, to_f32<E>(hp[i]), z * g_act(to_f32<E>(xh[i]))));
  }
}

// SignedMinGRU: h = a h_prev + z x~, a = gamma * ((1 - z) tanh(s) if coupled else tanh(s)).
template <typename E>
__global__ void __launch_bounds__(kThreads) signed_kernel(const E* zp, const E* sp, const E* xh,
                                                          const E* hp, const E* gamma, int coupled,
                                                          E* h, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float z = sigm(to_f32<E>(zp[i]));
    float a = tanhf(to_f32<E>(sp[i]));
    if (coupled) a *= 1.f - z;
    if (gamma) a *= to_f32<E>(gamma[i]);
    h[i] = from_f32<E>(fmaf(a, to_f32<E>(hp[i]), z * to_f32<E>(xh[i])));
  }
}

// RotationMinGRU, per 2-block j: v' = gamma R(theta) diag(1, tanh u) v + sigmoid(z) x~.
template <typename E>
__global__ void __launch_bounds__(kThreads) rotation_kernel(const E* th, const E* u, const E* zp,
                                                            const E* xh, const E* hp,
                                                            const E* gamma, E* h, long long nb) {
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < nb;
       j += (long long)gridDim.x * blockDim.x) {
    float s, c;
    sincosf(to_f32<E>(th[j]), &s, &c);
    const float d = tanhf(to_f32<E>(u[j]));
    const float v0 = to_f32<E>(hp[2 * j]), v1 = d * to_f32<E>(hp[2 * j + 1]);
    float o0 = c * v0 - s * v1, o1 = s * v0 + c * v1;
    if (gamma) {
      const float gm = to_f32<E>(gamma[j]);
      o0 *= gm;
      o1 *= gm;
    }
    h[2 * j] = from_f32<E>(fmaf(sigm(to_f32<E>(zp[2 * j])), to_f32<E>(xh[2 * j]), o0));
    h[2 * j + 1] = from_f32<E>(fmaf(sigm(to_f32<E>(zp[2 * j + 1])), to_f32<E>(xh[2 * j + 1]), o1));
  }
}

// GivensMinGRU, per k-block: R brick-wall rounds (round r rotates planes
// (i, i+1 mod k), i = r%2 + 2m, by theta[r][m]), then gamma, then + sigmoid(z) x~.
template <typename E, int K>
__global__ void __launch_bounds__(kThreads) givens_kernel(const E* th, const E* zp, const E* xh,
                                                          const E* hp, const E* gamma, E* h,
                                                          long long nb, int R) {
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < nb;
       j += (long long)gridDim.x * blockDim.x) {
    float v[K];
#pragma unroll
    for (int i = 0; i < K; ++i) v[i] = to_f32<E>(hp[j * K + i]);
    const E* t = th + j * (long long)R * (K / 2);
    for (int r = 0; r < R; ++r) {
      const int o = r & 1;
#pragma unroll
      for (int m = 0; m < K / 2; ++m) {
        const int a = (o + 2 * m) % K, b = (a + 1) % K;
        float s, c;
        sincosf(to_f32<E>(t[r * (K / 2) + m]), &s, &c);
        const float va = v[a], vb = v[b];
        v[a] = c * va - s * vb;
        v[b] = s * va + c * vb;
      }
    }
    const float gm = gamma ? to_f32<E>(gamma[j]) : 1.f;
#pragma unroll
    for (int i = 0; i < K; ++i)
      h[j * K + i] = from_f32<E>(fmaf(gm, v[i], sigm(to_f32<E>(zp[j * K + i])) * to_f32<E>(xh[j * K + i])));
  }
}

// DeltaMinGRU, one CTA per (b, head): H <- gamma H, then per micro-step m
// H <- H + beta_m k_m (v_m - k_m^T H)^T, and y = H^T q. Thread j owns state
// column j (dk values in shared memory), so columns never interact.
template <typename E>
__global__ void __launch_bounds__(128) delta_kernel(const E* q, const E* k, const E* v,
                                                    const E* beta, const E* gamma, const E* Hp,
                                                    E* y, E* H, int nh, int dk, int dv) {
  extern __shared__ float dsm[];
  float* sk = dsm;              // nh x dk
  float* sq = sk + nh * dk;     // dk
  float* sH = sq + dk;          // dk x dv (column j at sH[i * dv + j])
  const long long bh = blockIdx.x;
  for (int i = threadIdx.x; i < nh * dk; i += blockDim.x) sk[i] = to_f32<E>(k[bh * nh * dk + i]);
  for (int i = threadIdx.x; i < dk; i += blockDim.x) sq[i] = to_f32<E>(q[bh * dk + i]);
  __syncthreads();
  const float gm = gamma ? to_f32<E>(gamma[bh]) : 1.f;
  for (int j = threadIdx.x; j < dv; j += blockDim.x) {
    const E* hp = Hp + bh * (long long)dk * dv + j;
    float* col = sH + j;
    for (int i = 0; i < dk; ++i) col[i * dv] = gm * to_f32<E>(hp[(long long)i * dv]);
    for (int m = 0; m < nh; ++m) {
      const float* km = sk + m * dk;
      float kh = 0.f;
      for (int i = 0; i < dk; ++i) kh = fmaf(km[i], col[i * dv], kh);
      const float w = to_f32<E>(beta[bh * nh + m]) *
                      (to_f32<E>(v[(bh * nh + m) * (long long)dv + j]) - kh);
      for (int i = 0; i < dk; ++i) col[i * dv] = fmaf(km[i], w, col[i * dv]);
    }
    float yo = 0.f;
    E* ho = H + bh * (long long)dk * dv + j;
    for (int i = 0; i < dk; ++i) {
      yo = fmaf(sq[i], col[i * dv], yo);
      ho[(long long)i * dv] = from_f32<E>(col[i * dv]);
    }
    y[bh * dv + j] = from_f32<E>(yo);
  }
}

template <class F>
int by_dtype(int dtype, F&& f) {
  switch (dtype) {
    case MGS_F32: return f(float{});
    case MGS_BF16: return f(__nv_bfloat16{});
    case MGS_F16: return f(__half{});
    default: return MGS_BAD_DTYPE;
  }
}

inline int launched() { return cudaGetLastError() == cudaSuccess ? MGS_OK : MGS_LAUNCH_FAILED; }

}  // namespace step
}  // namespace mgs

extern "C" {

int mgs_mingru_step(const void* k, const void* xh, const void* h_prev, const void* gamma, void* h,
                    int64_t B, int64_t D, int dtype, void* stream) {
  if (B < 0 || D < 0) return MGS_BAD_SHAPE;
  const long long n = B * D;
  if (n == 0) return MGS_OK;
  return mgs::step::by_dtype(dtype, [&](auto e) {
    using E = decltype(e);
    mgs::step::mingru_kernel<E><<<mgs::step::blocks_for(n), mgs::step::kThreads, 0,
                                  static_cast<cudaStream_t>(stream)>>>(
        static_cast<const E*>(k), static_cast<const E*>(xh), static_cast<const E*>(h_prev),
        static_cast<const E*>(gamma), static_cast<E*>(h), n);
    return mgs::step::launched();
  });
}

int mgs_signed_step(const void* z, const void* s, const void* xh, const void* h_prev,
                    const void* gamma, int coupled, void* h, int64_t B, int64_t D, int dtype,
                    void* stream) {
  if (B < 0 || D < 0) return MGS_BAD_SHAPE;
  const long long n = B * D;
  if (n == 0) return MGS_OK;
  return mgs::step::by_dtype(dtype, [&](auto e) {
    using E = decltype(e);
    mgs::step::signed_kernel<E><<<mgs::step::blocks_for(n), mgs::step::kThreads, 0,
                                  static_cast<cudaStream_t>(stream)>>>(
        static_cast<const E*>(z), static_cast<const E*>(s), static_cast<const E*>(xh),
        static_cast<const E*>(h_prev), static_cast<const E*>(gamma), coupled, static_cast<E*>(h),
        n);
    return mgs::step::launched();
  });
}

int mgs_rotation_step(const void* theta, const void* u, const void* z, const void* xh,
                      const void* h_prev, const void* gamma, void* h, int64_t B, int64_t n,
                      int dtype, void* stream) {
  if (B < 0 || n < 0) return MGS_BAD_SHAPE;
  const long long nb = B * n;
  if (nb == 0) return MGS_OK;
  return mgs::step::by_dtype(dtype, [&](auto e) {
    using E = decltype(e);
    mgs::step::rotation_kernel<E><<<mgs::step::blocks_for(nb), mgs::step::kThreads, 0,
                                    static_cast<cudaStream_t>(stream)>>>(
        static_cast<const E*>(theta), static_cast<const E*>(u), static_cast<const E*>(z),
        static_cast<const E*>(xh), static_cast<const E*>(h_prev), static_cast<const E*>(gamma),
        static_cast<E*>(h), nb);
    return mgs::step::launched();
  });
}

int mgs_givens_step(const void* theta, const void* z, const void* xh, const void* h_prev,
                    const void* gamma, void* h, int64_t B, int64_t n, int R, int k, int dtype,
                    void* stream) {
  if (B < 0 || n < 0 || R < 1) return MGS_BAD_SHAPE;
  const long long nb = B * n;
  if (nb == 0) return MGS_OK;
  return mgs::step::by_dtype(dtype, [&](auto e) {
    using E = decltype(e);
    auto st = static_cast<cudaStream_t>(stream);
    const unsigned g = mgs::step::blocks_for(nb);
    auto args = [&](auto kern) {
      kern<<<g, mgs::step::kThreads, 0, st>>>(
          static_cast<const E*>(theta), static_cast<const E*>(z), static_cast<const E*>(xh),
          static_cast<const E*>(h_prev), static_cast<const E*>(gamma), static_cast<E*>(h), nb, R);
      return mgs::step::launched();
    };
    switch (k) {
      case 2: return args(mgs::step::givens_kernel<E, 2>);
      case 4: return args(mgs::step::givens_kernel<E, 4>);
      case 8: return args(mgs::step::givens_kernel<E, 8>);
      case 16: return args(mgs::step::givens_kernel<E, 16>);
      case 32: return args(mgs::step::givens_kernel<E, 32>);
      case 64: return args(mgs::step::givens_kernel<E, 64>);
      default: return (int)MGS_UNSUPPORTED;
    }
  });
}

int mgs_delta_step(const void* q, const void* k, const void* v, const void* beta, const void* gamma,
                   const void* H_prev, void* y, void* H, int64_t B, int heads, int nh, int dk,
                   int dv, int dtype, void* stream) {
  if (B < 0 || heads < 0 || nh < 1 || dk < 1 || dv < 1) return MGS_BAD_SHAPE;
  const long long bh = B * (long long)heads;
  if (bh == 0) return MGS_OK;
  const size_t smem = ((size_t)nh * dk + dk + (size_t)dk * dv) * sizeof(float);
  if (smem > 227 * 1024 || bh > 0x7fffffffLL) return MGS_UNSUPPORTED;
  return mgs::step::by_dtype(dtype, [&](auto e) -> int {
    using E = decltype(e);
    auto kern = mgs::step::delta_kernel<E>;
    MGS_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<(unsigned)bh, 128, smem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const E*>(q), static_cast<const E*>(k), static_cast<const E*>(v),
        static_cast<const E*>(beta), static_cast<const E*>(gamma), static_cast<const E*>(H_prev),
        static_cast<E*>(y), static_cast<E*>(H), nh, dk, dv);
    return mgs::step::launched();
  });
}

}  // extern "C"
