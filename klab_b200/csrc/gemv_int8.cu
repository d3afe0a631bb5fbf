// INT8 weight instantiations: per-row scale (x BF16) and per-64 scale (x BF16/FP16/FP32).
#include "gemv_launch.cuh"

namespace klab {
cudaError_t gemv_run_int8(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  if (wfmt == W_I8_ROW) {
    if (s.xfmt == X_BF16) return run_fx<W_I8_ROW, X_BF16>(p, s, stream, occ);
    if (s.xfmt == X_F16) return run_fx<W_I8_ROW, X_F16>(p, s, stream, occ);
    if (s.xfmt == X_F32) return run_fx<W_I8_ROW, X_F32>(p, s, stream, occ);
  } else if (wfmt == W_I8_G64) {
    if (s.xfmt == X_BF16) return run_fx<W_I8_G64, X_BF16>(p, s, stream, occ);
    if (s.xfmt == X_F16) return run_fx<W_I8_G64, X_F16>(p, s, stream, occ);
    if (s.xfmt == X_F32) return run_fx<W_I8_G64, X_F32>(p, s, stream, occ);
  }
  return cudaErrorNotSupported;
}
}  // namespace klab
