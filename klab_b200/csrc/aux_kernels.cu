// Bit-exact decode kernels behind the unpack / dequantize APIs.
//
//   cbf16_unpack_kernel   lossless BF16 codec v1 -> original uint16 bits, any K
//                         (compressed_kernels.cu:181-200 / compressed_bf16.unpack_weights)
//   int8_dequant_kernel   code * scale in FP32 (int8_weights.py:15-17), per-64 or per-row
//   fp4_dequant_kernel    E2M1 * scale (fp4.py:21-27 for the E4M3/16 + global format;
//                         the FP16/32 format multiplies by the FP16 scale)
#include <cstdint>

#include "common.cuh"
#include "lossless_f32.cuh"
#include "klab_kernels.h"

namespace klab {

// One thread per output weight; only integer operations.
__global__ void __launch_bounds__(256) cbf16_unpack_kernel(const unsigned char* __restrict__ payload,
                                                          const unsigned* __restrict__ metadata,
                                                          unsigned short* __restrict__ out, int n,
                                                          int k) {
  const long long index = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  const long long total = static_cast<long long>(n) * k;
  if (index >= total) return;
  const long long row = index / k;
  const int col = static_cast<int>(index - row * k);
  const long long blocks_per_row = (k + 63) / 64;
  const unsigned meta = metadata[row * blocks_per_row + (col >> 6)];
  const unsigned char* block = payload + (static_cast<size_t>(meta & 0x7fffffu) << 5);
  const unsigned j = col & 63;
  unsigned bits;
  if (meta >> 31) {
    bits = block[2 * j] | (static_cast<unsigned>(block[2 * j + 1]) << 8);
  } else {
    // Code j starts at bit 12*j of the block, least significant bits first.
    const unsigned byte = (3 * j) >> 1, shift = (j & 1) ? 4 : 0;
    const unsigned pair = block[byte] | (static_cast<unsigned>(block[byte + 1]) << 8);
    const unsigned code = (pair >> shift) & 0xfffu;
    const unsigned exponent = ((meta >> 23) & 0xffu) + (code >> 8);
    bits = (code & 0x7fu) | ((code & 0x80u) << 8) | (exponent << 7);
  }
  out[index] = static_cast<unsigned short>(bits);
}

// group == 64: scales [N, K/64]; group == 0: scales [N] (one per row).
__global__ void __launch_bounds__(256) int8_dequant_kernel(const signed char* __restrict__ codes,
                                                          const float* __restrict__ scales, int group,
                                                          float* __restrict__ out, int n, int k) {
  const long long index = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  const long long total = static_cast<long long>(n) * k;
  if (index >= total) return;
  const long long row = index / k;
  const int col = static_cast<int>(index - row * k);
  const float scale = group ? scales[row * (k / 64) + col / 64] : scales[row];
  out[index] = mul_rn(static_cast<float>(codes[index]), scale);
}

// E2M1 magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 as exact FP32; bit 3 is the sign.
__device__ __forceinline__ float e2m1_value(unsigned code) {
  const unsigned m = code & 7u;
  const unsigned bits = m < 2u ? m * 0x3f000000u : 0x3f000000u + (m << 22);
  return __uint_as_float(bits | ((code & 8u) << 28));
}

// E4M3 (fn) byte -> FP32: bias 7, subnormals, 0x7f/0xff NaN, no infinities.
__device__ __forceinline__ float e4m3_value(unsigned byte) {
  const unsigned e = (byte >> 3) & 15u, m = byte & 7u;
  float v;
  if ((byte & 0x7fu) == 0x7fu) {
    v = __uint_as_float(0x7fc00000u);
  } else if (e == 0) {
    v = static_cast<float>(m) * 0.001953125f;  // m * 2^-9, exact
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  }
  return (byte & 0x80u) ? -v : v;
}

// kind KLAB_FP4_E4M3_G16: scales [N, K/16] E4M3 bytes, w = e2m1 * (scale * global);
// kind KLAB_FP4_F16_G32: scales [N, K/32] FP16, w = e2m1 * scale.
__global__ void __launch_bounds__(256) fp4_dequant_kernel(const unsigned char* __restrict__ packed,
                                                         const void* __restrict__ scales, int kind,
                                                         const float* __restrict__ gscale,
                                                         float* __restrict__ out, int n, int k) {
  const long long index = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  const long long total = static_cast<long long>(n) * k;
  if (index >= total) return;
  const long long row = index / k;
  const int col = static_cast<int>(index - row * k);
  const unsigned byte = packed[row * (k / 2) + col / 2];
  const float e = e2m1_value((col & 1) ? (byte >> 4) : (byte & 15u));
  float scale;
  if (kind == KLAB_FP4_E4M3_G16) {
    const unsigned s = static_cast<const unsigned char*>(scales)[row * (k / 16) + col / 16];
    scale = mul_rn(e4m3_value(s), *gscale);
  } else {
    scale = f16_to_f32(static_cast<const unsigned short*>(scales)[row * (k / 32) + col / 32]);
  }
  out[index] = mul_rn(e, scale);
}

// Lossless FP32 formats -> FP32, four weights per thread (exact bits).
__global__ void __launch_bounds__(256) lossless_unpack_kernel(const unsigned char* __restrict__ mantissa,
                                                              const unsigned char* __restrict__ exponents,
                                                              const unsigned* __restrict__ payload,
                                                              const unsigned* __restrict__ metadata,
                                                              float* __restrict__ out, long long count) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (idx >= count) return;
  const float4 v = mantissa ? lf32_load4(mantissa, exponents, metadata, idx) : fp28_load4(payload, metadata, idx);
  *reinterpret_cast<float4*>(out + idx) = v;
}

cudaError_t launch_lossless_unpack(const void* mantissa, const void* exponents, const void* payload,
                                   const unsigned* metadata, float* out, long long count, cudaStream_t stream) {
  const long long blocks = (count / 4 + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  lossless_unpack_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const unsigned char*>(mantissa), static_cast<const unsigned char*>(exponents),
      static_cast<const unsigned*>(payload), metadata, out, count);
  return cudaGetLastError();
}

cudaError_t launch_cbf16_unpack(const void* payload, const unsigned* metadata, void* out, int n, int k,
                                cudaStream_t stream) {
  const long long total = static_cast<long long>(n) * k;
  const long long blocks = (total + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  cbf16_unpack_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const unsigned char*>(payload), metadata, static_cast<unsigned short*>(out), n, k);
  return cudaGetLastError();
}

cudaError_t launch_int8_dequant(const void* codes, const float* scales, int group, float* out, int n, int k,
                                cudaStream_t stream) {
  const long long total = static_cast<long long>(n) * k;
  const long long blocks = (total + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  int8_dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const signed char*>(codes), scales, group, out, n, k);
  return cudaGetLastError();
}

cudaError_t launch_fp4_dequant(const void* packed, const void* scales, int kind, const float* gscale, float* out,
                               int n, int k, cudaStream_t stream) {
  const long long total = static_cast<long long>(n) * k;
  const long long blocks = (total + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  fp4_dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const unsigned char*>(packed), scales, kind, gscale, out, n, k);
  return cudaGetLastError();
}

// y[r, :] = ((x + residual)[r, :] * rsqrt(mean((x + residual)[r, :]^2) + eps)) * weight
// for FP32 rows of K <= 8192: one CTA of 256 threads per row, the summed row kept
// in registers (thread t holds columns t, t + 256, ...). Reduction order: per
// thread in column order, a butterfly within each warp, then the eight warp sums
// in warp order; one rsqrtf. Same contract as kernels.cu:168-222.
constexpr int kRmsThreads = 256;
constexpr int kRmsMaxK = 8192;
__global__ void __launch_bounds__(kRmsThreads) residual_rmsnorm_kernel(const float* __restrict__ x,
                                                                       const float* __restrict__ residual,
                                                                       const float* __restrict__ weight,
                                                                       float* __restrict__ y, int k, float eps) {
  constexpr int VALUES = kRmsMaxK / kRmsThreads;
  constexpr int WARPS = kRmsThreads / 32;
  __shared__ float partial[WARPS];
  const long long base = static_cast<long long>(blockIdx.x) * k;
  float v[VALUES];
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < VALUES; ++i) {
    const int col = threadIdx.x + i * kRmsThreads;
    v[i] = col < k ? __fadd_rn(__ldg(x + base + col), __ldg(residual + base + col)) : 0.0f;
    sum = __fmaf_rn(v[i], v[i], sum);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = sum;
  __syncthreads();
  float total = partial[0];
#pragma unroll
  for (int w = 1; w < WARPS; ++w) total = __fadd_rn(total, partial[w]);
  const float inv_rms = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(k)), eps));
#pragma unroll
  for (int i = 0; i < VALUES; ++i) {
    const int col = threadIdx.x + i * kRmsThreads;
    if (col < k) y[base + col] = __fmul_rn(__fmul_rn(v[i], inv_rms), __ldg(weight + col));
  }
}

cudaError_t launch_residual_rmsnorm(const float* x, const float* residual, const float* weight, float* y, int m,
                                    int k, float eps, cudaStream_t stream) {
  if (k > kRmsMaxK) return cudaErrorInvalidValue;
  residual_rmsnorm_kernel<<<m, kRmsThreads, 0, stream>>>(x, residual, weight, y, k, eps);
  return cudaGetLastError();
}

}  // namespace klab
