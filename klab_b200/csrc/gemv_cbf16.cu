// Lossless BF16 codec v1 instantiations (x BF16).
#include "gemv_launch.cuh"

namespace klab {
cudaError_t gemv_run_cbf16(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  if (wfmt == W_CBF16 && s.xfmt == X_BF16) return run_fx<W_CBF16, X_BF16>(p, s, stream, occ);
  return cudaErrorNotSupported;
}
}  // namespace klab
