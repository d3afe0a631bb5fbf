// Decode-step elementwise ops that surround the projections, with the
// arithmetic of the reference's fused kernels (research/l2-prefetch/src/
// decode_attn.cu:471-527): residual add + RMSNorm (BF16 in, BF16 x and x_norm
// out) and SiLU(gate) * up (BF16). Used by the standalone kernels in
// decode_ops.cu and by the projection kernel's x staging when the op is fused
// into the next projection, so both give the same bits.
#pragma once
#include <cuda_runtime.h>

namespace klab {

__device__ __forceinline__ float bf16_value(unsigned b) { return __uint_as_float((b & 0xffffu) << 16); }

// Round to nearest even by the bit formula the reference uses (NaN payloads
// follow the same formula).
__device__ __forceinline__ unsigned bf16_rne_bits(float f) {
  const unsigned u = __float_as_uint(f);
  return (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
}

// x = RNE(res + y) for one pair of BF16 values (two per 32-bit word).
__device__ __forceinline__ unsigned add_pair(unsigned a, unsigned b) {
  const float x0 = __fadd_rn(bf16_value(a), bf16_value(b));
  const float x1 = __fadd_rn(bf16_value(a >> 16), bf16_value(b >> 16));
  return bf16_rne_bits(x0) | (bf16_rne_bits(x1) << 16);
}

// 1 / RMS of one row of d BF16 values (d even) in the reference's order: thread t
// of the first 256 threads takes pairs t, t + 256, ...; per pair the FMA chain
// adds x1^2 then x0^2; a butterfly sums each warp; the eight warp sums are
// added from zero in warp order; inv = rsqrtf(ss / d + eps). When x_out2 is
// not null, the first 256 threads also store x = RNE(res + y). Every thread of
// the block must call it (it holds one barrier); `red` is 8 shared floats, and
// the caller separates two calls with a barrier of its own.
__device__ __forceinline__ float add_rmsnorm_inv(const unsigned* res2, const unsigned* y2, unsigned* x_out2, int d,
                                                 float eps, float* red) {
  const int tid = threadIdx.x;
  float ss = 0.0f;
  if (tid < 256) {
    for (int i = tid; i < d / 2; i += 256) {
      const unsigned x = add_pair(__ldg(res2 + i), __ldg(y2 + i));
      if (x_out2) x_out2[i] = x;
      const float x0 = bf16_value(x), x1 = bf16_value(x >> 16);
      ss = __fmaf_rn(x0, x0, __fmaf_rn(x1, x1, ss));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if ((tid & 31) == 0) red[tid >> 5] = ss;
  }
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) total = __fadd_rn(total, red[w]);
  return rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(d)), eps));
}

// x_norm pair i = RNE((x * inv) * w) with x = RNE(res + y).
__device__ __forceinline__ unsigned add_rmsnorm_pair(unsigned res_pair, unsigned y_pair, unsigned w_pair, float inv) {
  const unsigned x = add_pair(res_pair, y_pair);
  const float o0 = __fmul_rn(__fmul_rn(bf16_value(x), inv), bf16_value(w_pair));
  const float o1 = __fmul_rn(__fmul_rn(bf16_value(x >> 16), inv), bf16_value(w_pair >> 16));
  return bf16_rne_bits(o0) | (bf16_rne_bits(o1) << 16);
}

// SiLU(gate) * up for one pair: g / (1 + exp(-g)) * u in FP32 (the fast exp
// intrinsic, an IEEE division), one RNE to BF16.
__device__ __forceinline__ unsigned silu_mul_pair(unsigned g, unsigned u) {
  const float g0 = bf16_value(g), g1 = bf16_value(g >> 16);
  const float o0 = __fmul_rn(__fdiv_rn(g0, __fadd_rn(1.0f, __expf(-g0))), bf16_value(u));
  const float o1 = __fmul_rn(__fdiv_rn(g1, __fadd_rn(1.0f, __expf(-g1))), bf16_value(u >> 16));
  return bf16_rne_bits(o0) | (bf16_rne_bits(o1) << 16);
}

}  // namespace klab
