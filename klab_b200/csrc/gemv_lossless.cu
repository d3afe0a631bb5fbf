// Lossless FP32 weight instantiations (x FP32): W_LF32 and W_FP28.
#include "gemv_launch.cuh"

namespace klab {
cudaError_t gemv_run_lossless(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  if (s.xfmt != X_F32) return cudaErrorNotSupported;
  if (wfmt == W_LF32) return run_fx<W_LF32, X_F32>(p, s, stream, occ);
  if (wfmt == W_FP28) return run_fx<W_FP28, X_F32>(p, s, stream, occ);
  return cudaErrorNotSupported;
}
}  // namespace klab
