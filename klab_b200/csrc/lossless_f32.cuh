// Decoders of the two lossless FP32 weight formats (every weight keeps its exact
// IEEE-754 bits). Used by the projection kernel's slot fill and by the unpack
// kernels. Both formats cut the row-major [N, K] matrix (K % 64 == 0) into blocks
// of 64 consecutive weights; a block's exponents are stored as 4-bit deltas from
// the block's minimum exponent when they all fit, otherwise as the original bits.
//
// Lossless FP32 v1 (lossless_weights.py:38-75, lossless_kernels.cu:4-29):
//   mantissa  u8 [N, 3K]: weight i's 23 mantissa bits and its sign (at bit 23),
//             little-endian in bytes 3i..3i+2;
//   exponents u8 stream: per block 32 bytes of deltas (byte j = delta[2j] |
//             delta[2j+1] << 4) or 64 raw exponent bytes ("wide"), blocks in order;
//   metadata  i32 [N, K/64]: (offset / 32) << 9 | base << 1 | wide, offset = the
//             block's first byte in the exponent stream.
//
// Packed FP32 "fp28" (packed_fp32.py:35-67, adaptive_kernels.cu:41-75):
//   payload   i32 stream: per block either 56 words holding 64 28-bit codes
//             (code = significand | sign << 23 | delta << 24, code j at bit 28j of
//             the block, least significant bit first) or 64 words of original
//             bits ("wide");
//   metadata  i32 [N, K/64]: (offset / 8) << 9 | base << 1 | wide, offset = the
//             block's first payload word.
#pragma once
#include <cstdint>

namespace klab {

__device__ __forceinline__ float lossless_value(unsigned sig24, unsigned exponent) {
  return __uint_as_float((sig24 & 0x7fffffu) | ((sig24 & 0x800000u) << 8) | (exponent << 23));
}

// Four consecutive weights starting at flat index idx (idx % 4 == 0).
__device__ __forceinline__ float4 lf32_load4(const unsigned char* mantissa, const unsigned char* exponents,
                                             const unsigned* metadata, long long idx) {
  const unsigned* mw = reinterpret_cast<const unsigned*>(mantissa + idx * 3);
  const unsigned a = __ldg(mw), b = __ldg(mw + 1), c = __ldg(mw + 2);
  const unsigned sig[4] = {a & 0xffffffu, (a >> 24) | ((b & 0xffffu) << 8), (b >> 16) | ((c & 0xffu) << 16),
                           c >> 8};
  const unsigned meta = __ldg(metadata + (idx >> 6));
  const int local = static_cast<int>(idx & 63);
  const unsigned char* block = exponents + ((meta >> 9) << 5);
  float v[4];
  if (meta & 1u) {
    const unsigned e4 = __ldg(reinterpret_cast<const unsigned*>(block + local));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = lossless_value(sig[i], (e4 >> (8 * i)) & 0xffu);
  } else {
    const unsigned d4 = __ldg(reinterpret_cast<const unsigned short*>(block + local / 2));
    const unsigned base = (meta >> 1) & 0xffu;
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = lossless_value(sig[i], base + ((d4 >> (4 * i)) & 0xfu));
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Code j (0..63) of a compact fp28 block.
__device__ __forceinline__ unsigned fp28_code(const unsigned* block, int j) {
  const int bit = 28 * j;
  const int w = bit >> 5, s = bit & 31;
  unsigned long long pair = __ldg(block + w);
  if (s > 4) pair |= static_cast<unsigned long long>(__ldg(block + w + 1)) << 32;
  return static_cast<unsigned>(pair >> s) & 0x0fffffffu;
}

__device__ __forceinline__ float4 fp28_load4(const unsigned* payload, const unsigned* metadata, long long idx) {
  const unsigned meta = __ldg(metadata + (idx >> 6));
  const int local = static_cast<int>(idx & 63);
  const unsigned* block = payload + (static_cast<unsigned long long>(meta >> 9) << 3);
  if (meta & 1u) {
    return make_float4(__uint_as_float(__ldg(block + local)), __uint_as_float(__ldg(block + local + 1)),
                       __uint_as_float(__ldg(block + local + 2)), __uint_as_float(__ldg(block + local + 3)));
  }
  const unsigned base = (meta >> 1) & 0xffu;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const unsigned code = fp28_code(block, local + i);
    v[i] = lossless_value(code & 0xffffffu, base + (code >> 24));
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

}  // namespace klab
