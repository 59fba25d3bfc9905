// gate_up GEMM + SwiGLU epilogue (placeholder until the tcgen05 kernel lands).
#include "kernels.h"

namespace cascade {
cudaError_t launch_gateup(const GateUpLaunch&, const void*, const void*, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_gateup_window(const void*, void*, int64_t, int32_t, int32_t, int32_t, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace cascade
