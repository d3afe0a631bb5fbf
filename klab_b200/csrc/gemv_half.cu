// 16/32-bit weight instantiations: BF16 (x BF16), FP16 (x FP16), FP32 (x FP32).
#include "gemv_launch.cuh"

namespace klab {
cudaError_t gemv_run_half(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  if (wfmt == W_BF16 && s.xfmt == X_BF16) return run_fx<W_BF16, X_BF16>(p, s, stream, occ);
  if (wfmt == W_F16 && s.xfmt == X_F16) return run_fx<W_F16, X_F16>(p, s, stream, occ);
  if (wfmt == W_F32 && s.xfmt == X_F32) return run_fx<W_F32, X_F32>(p, s, stream, occ);
  return cudaErrorNotSupported;
}
}  // namespace klab
