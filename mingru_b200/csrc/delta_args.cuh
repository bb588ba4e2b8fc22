// delta_args.cuh -- kernel arguments of the DeltaMinGRU chunked-WY delta rule,
// shared by the fp32 CUDA-core kernels (delta.cu) and the bf16 tensor-core
// kernels (delta_tc.cu).
#pragma once

#include "common.cuh"

namespace mgs {
namespace delta {

constexpr int kMaxM = 64;   // nh * chunk micro-steps per chunk on the tensor-core kernels

template <typename E>
struct Args {
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
  float* Ac;      // (BH, nchunks, dk, dk)  chunk transition, saved for the backward
  float* Bc;      // (BH, nchunks, dk, dv)  chunk injection (forward scratch)
  float* Hb;      // (BH, nchunks, dk, dv)  chunk-start states, saved for the backward
  float* Ec;      // (BH, nchunks, dk, dv)  backward scratch
  float* dSo;     // (BH, nchunks, dk, dv)  gradient w.r.t. each chunk's output state
  const float* lg;  // (BH, T) per-token log decay (<= 0), or null: no decay
  float* dlg;       // (BH, T) its gradient (backward with decay)
  long long T_;
  int H, nh, dk, dv, C, nchunks;
};

// Tensor-core path (bf16 and fp32 inputs): eligibility, buffer sizes and launch.
bool tc_eligible(int dtype, int nh, int dk, int dv, int C);
size_t tc_saved_floats(long long BH, long long T, int dk, int dv, int C, int dtype);
size_t tc_workspace_floats(long long BH, long long T, int dk, int dv, int C);
int run_tc(bool fwd, const Args<__nv_bfloat16>& p, long long B, int H, long long T, int nh, int dk,
           int dv, int C, float* saved, void* ws, size_t ws_bytes, cudaStream_t st);
int run_tc(bool fwd, const Args<float>& p, long long B, int H, long long T, int nh, int dk, int dv,
           int C, float* saved, void* ws, size_t ws_bytes, cudaStream_t st);

}  // namespace delta
}  // namespace mgs
