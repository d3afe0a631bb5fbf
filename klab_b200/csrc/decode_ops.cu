// Standalone decode elementwise kernels: residual add + RMSNorm and SiLU * up,
// BF16, with the reference kernels' arithmetic (decode_ops.cuh). Replace
// add_rmsnorm_bf16 / silu_mul_bf16 (research/l2-prefetch/src/decode_attn.cu:
// 471-527) behind decode_attn.add_rmsnorm / silu_mul (decode_attn.py:64-81).
#include <cuda_runtime.h>

#include "decode_ops.cuh"
#include "klab_kernels.h"

namespace klab {
namespace {

// One 256-thread block per row.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const unsigned* __restrict__ res,
                                                          const unsigned* __restrict__ y,
                                                          const unsigned* __restrict__ w, unsigned* __restrict__ x,
                                                          unsigned* __restrict__ xn, int d, float eps) {
  __shared__ float red[8];
  const long long row = static_cast<long long>(blockIdx.x) * (d / 2);
  const float inv = add_rmsnorm_inv(res + row, y + row, x + row, d, eps, red);
  for (int i = threadIdx.x; i < d / 2; i += blockDim.x)
    xn[row + i] = add_rmsnorm_pair(__ldg(res + row + i), __ldg(y + row + i), __ldg(w + i), inv);
}

// Pairs over all rows: gu row r = [gate (inter) | up (inter)], out row r = inter values.
__global__ void __launch_bounds__(256) silu_mul_kernel(const unsigned* __restrict__ gu, unsigned* __restrict__ out,
                                                       int inter, long long pairs) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= pairs) return;
  const int per_row = inter / 2;
  const long long row = i / per_row;
  const int j = static_cast<int>(i - row * per_row);
  const unsigned* g = gu + row * inter;  // inter values = inter / 2 words of gate, then up
  out[i] = silu_mul_pair(__ldg(g + j), __ldg(g + per_row + j));
}

}  // namespace

cudaError_t launch_add_rmsnorm(const void* res, const void* y, const void* w, void* x, void* xn, int m, int d,
                               float eps, cudaStream_t stream) {
  add_rmsnorm_kernel<<<m, 256, 0, stream>>>(static_cast<const unsigned*>(res), static_cast<const unsigned*>(y),
                                            static_cast<const unsigned*>(w), static_cast<unsigned*>(x),
                                            static_cast<unsigned*>(xn), d, eps);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* gu, void* out, int m, int inter, cudaStream_t stream) {
  const long long pairs = static_cast<long long>(m) * inter / 2;
  const long long blocks = (pairs + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  silu_mul_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<const unsigned*>(gu),
                                                                     static_cast<unsigned*>(out), inter, pairs);
  return cudaGetLastError();
}

}  // namespace klab
