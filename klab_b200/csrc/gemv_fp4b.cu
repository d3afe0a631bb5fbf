// FP4 E2M1 with an E4M3 scale per 16 and an FP32 global scale (x BF16/FP16/FP32).
#include "gemv_launch.cuh"

namespace klab {
cudaError_t gemv_run_fp4b(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  if (wfmt == W_FP4_G16E) {
    if (s.xfmt == X_BF16) return run_fx<W_FP4_G16E, X_BF16>(p, s, stream, occ);
    if (s.xfmt == X_F16) return run_fx<W_FP4_G16E, X_F16>(p, s, stream, occ);
    if (s.xfmt == X_F32) return run_fx<W_FP4_G16E, X_F32>(p, s, stream, occ);
  }
  return cudaErrorNotSupported;
}
}  // namespace klab
