// capi.cu -- library-wide C ABI entry points (version, status strings and the
// sticky device error word that bounded look-back waits write into).
#include <cuda_runtime.h>

#include "../../include/mingru_scan.h"

namespace mgs {
// One sticky error word per translation unit; each kernel file exports its reader.
unsigned take_error_linear(cudaStream_t s);
unsigned take_error_log(cudaStream_t s);
unsigned take_error_affine(cudaStream_t s);
unsigned take_error_angle(cudaStream_t s);
unsigned take_error_delta_tc(cudaStream_t s);
}  // namespace mgs

extern "C" {

int mgs_version(void) { return 100; /* 0.1.0 */ }

const char* mgs_status_string(int status) {
  switch (status) {
    case MGS_OK: return "ok";
    case MGS_BAD_SHAPE: return "bad shape";
    case MGS_BAD_DTYPE: return "unsupported dtype";
    case MGS_BAD_ALIGNMENT: return "misaligned pointer";
    case MGS_UNSUPPORTED: return "shape outside the kernel envelope";
    case MGS_LAUNCH_FAILED: return "CUDA launch failed";
    case MGS_LOOKBACK_TIMEOUT: return "look-back wait exceeded its bound";
    case MGS_WORKSPACE_TOO_SMALL: return "workspace or carry buffer too small";
    default: return "unknown status";
  }
}

int mgs_take_device_error(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned bits = 0u;
  bits |= mgs::take_error_linear(s);
  bits |= mgs::take_error_log(s);
  bits |= mgs::take_error_affine(s);
  bits |= mgs::take_error_angle(s);
  bits |= mgs::take_error_delta_tc(s);
  return (int)bits;
}

}  // extern "C"
