// Internal declarations shared by the CUDA translation units of libklab_b200.
#pragma once
#include <cstddef>

#include <cuda_runtime.h>

#include "../../include/klab_b200.h"

namespace klab {
// Tensor-core projection for token tiles (kind 0: BF16 weights, 1: INT8 + per-row scale).
int tc_gemm_launch(int kind, const void* x, int ldx, const void* w, const float* scales, void* out, int ldo,
                   int out_f32, int m, int n, int k, int* status, cudaStream_t stream);
// Token tiles (M <= 16) of INT8 per-row (kind 0) or E2M1 + FP16 scale per 32 (kind 1) weights
// on the warp-level tensor cores (tile_mma.cu). KLAB_E_ALIGN / KLAB_E_UNSUPPORTED: not
// applicable, the caller uses the CUDA-core kernel. Workspace: [tickets][phase partials].
constexpr size_t kTileMmaTicketBytes = 16384 * 4;
int tile_mma_launch(int kind, int x_f16, const void* x, int ldx, const void* w, const void* scales, void* out,
                    int ldo, int out_f32, int m, int n, int k, void* ws, size_t ws_bytes, int sms, int* status,
                    bool pdl, cudaStream_t stream);
size_t tile_mma_workspace(int kind, int m, int n, int k);
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
