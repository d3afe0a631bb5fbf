// Host-side launch of stream_gemv_kernel instantiations (one .cu per weight
// format includes this and instantiates its (x format, x mode, M-tile) set).
#pragma once
#include <cuda_runtime.h>

#include "stream_gemv.cuh"

namespace klab {

struct LaunchShape {
  int xfmt;        // XFmt
  int xmode;       // XMode
  int mt;          // tokens per tile: 1, 2, 4 or 8
  dim3 grid;
  size_t smem;
  bool pdl;
};

template <int F, int X, int XM, int MT>
cudaError_t launch_one(const GemvParams& p, const LaunchShape& s, cudaStream_t stream) {
  auto kernel = stream_gemv_kernel<F, X, XM, MT>;
  // The opt-in shared-memory limit is a per-function attribute; setting it is
  // cheap and legal during stream capture.
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(s.smem));
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = s.grid;
  cfg.blockDim = dim3(warps_for(F, MT) * 32, 1, 1);
  cfg.dynamicSmemBytes = s.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = s.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int F, int X, int XM, int MT>
int occupancy_one(size_t smem) {
  int blocks = 0;
  auto kernel = stream_gemv_kernel<F, X, XM, MT>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, warps_for(F, MT) * 32, smem) != cudaSuccess)
    return 0;
  return blocks;
}

template <int F, int X, int XM>
cudaError_t run_mt(const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  switch (s.mt) {
#define KLAB_MT_CASE(MT)                                             \
  case MT:                                                           \
    if (occ) {                                                       \
      *occ = occupancy_one<F, X, XM, MT>(s.smem);                    \
      return cudaSuccess;                                            \
    }                                                                \
    return launch_one<F, X, XM, MT>(p, s, stream);
    KLAB_MT_CASE(1)
    KLAB_MT_CASE(2)
    KLAB_MT_CASE(4)
    KLAB_MT_CASE(8)
#undef KLAB_MT_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

// Launch (occ == nullptr) or query CTAs per SM (occ != nullptr) for one
// (weight format, x format) pair.
template <int F, int X>
cudaError_t run_fx(const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ) {
  if (s.xmode == XM_SMEM) return run_mt<F, X, XM_SMEM>(p, s, stream, occ);
  if (s.xmode == XM_GLOBAL) return run_mt<F, X, XM_GLOBAL>(p, s, stream, occ);
  // 16-bit x staging exists for every 16-bit x.
  if constexpr (X != X_F32) return run_mt<F, X, XM_SMEM16>(p, s, stream, occ);
  return cudaErrorNotSupported;
}

// Defined in gemv_<family>.cu; dispatch on (wfmt, s.xfmt). Unsupported pairs
// return cudaErrorNotSupported.
cudaError_t gemv_run_half(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ);
cudaError_t gemv_run_cbf16(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ);
cudaError_t gemv_run_int8(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ);
cudaError_t gemv_run_fp4a(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ);
cudaError_t gemv_run_fp4b(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ);
cudaError_t gemv_run_lossless(int wfmt, const GemvParams& p, const LaunchShape& s, cudaStream_t stream, int* occ);

}  // namespace klab
