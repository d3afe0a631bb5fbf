// Internal declarations shared by the CUDA translation units of libklab_b200.
#pragma once
#include <cuda_runtime.h>

#include "../../include/klab_b200.h"

namespace klab {
// Tensor-core projection for token tiles (kind 0: BF16 weights, 1: INT8 + per-row scale).
int tc_gemm_launch(int kind, const void* x, int ldx, const void* w, const float* scales, void* out, int ldo,
                   int out_f32, int m, int n, int k, int* status, cudaStream_t stream);
// Device address of the status word on the current device (nullptr on error).
int* device_status_address();
cudaError_t launch_cbf16_unpack(const void* payload, const unsigned* metadata, void* out, int n, int k,
                                cudaStream_t stream);
cudaError_t launch_int8_dequant(const void* codes, const float* scales, int group, float* out, int n, int k,
                                cudaStream_t stream);
cudaError_t launch_fp4_dequant(const void* packed, const void* scales, int kind, const float* gscale, float* out,
                               int n, int k, cudaStream_t stream);
cudaError_t launch_add_rmsnorm(const void* res, const void* y, const void* w, void* x, void* xn, int m, int d,
                               float eps, cudaStream_t stream);
cudaError_t launch_silu_mul(const void* gu, void* out, int m, int inter, cudaStream_t stream);
cudaError_t launch_residual_rmsnorm(const float* x, const float* residual, const float* weight, float* y, int m,
                                    int k, float eps, cudaStream_t stream);
cudaError_t launch_lossless_unpack(const void* mantissa, const void* exponents, const void* payload,
                                   const unsigned* metadata, float* out, long long count, cudaStream_t stream);
cudaError_t launch_l2_prefetch(const void* p, long long bytes, int blocks, int stride, int threads, int kind,
                               unsigned* sink, cudaStream_t stream);
}  // namespace klab
