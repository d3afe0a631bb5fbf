// Host (CPU) side of the lossless BF16 codec v1: packing and validated
// unpacking, used at weight-preparation time (compressed_bf16.py:84-243,
// docs/bf16-format.md). Integer-only; every bit pattern round-trips.
#include <cstdint>
#include <cstring>

#include "../../include/klab_b200.h"

namespace {

constexpr int kBlock = 64;
constexpr uint32_t kCodedBytes = 96, kRawBytes = 128, kUnit = 32;
constexpr uint64_t kMaxPayload = 1ull << 28;

// Block b of row r, padded with the row's last weight past K.
inline void load_block(const uint16_t* row, int k, int b, uint16_t (&v)[kBlock]) {
  const int c0 = b * kBlock;
  for (int i = 0; i < kBlock; ++i) {
    const int c = c0 + i;
    v[i] = row[c < k ? c : k - 1];
  }
}

}  // namespace

extern "C" {

KLAB_API int klab_cbf16_pack_host(const uint16_t* bits, int n, int k, uint32_t* metadata, uint8_t* payload,
                                  size_t payload_capacity, size_t* payload_bytes) {
  if (!bits || !metadata || !payload_bytes || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (static_cast<long long>(n) * k >= (1ll << 31)) return KLAB_E_SHAPE;
  const int bpr = (k + kBlock - 1) / kBlock;
  uint64_t offset = 0;
  uint16_t v[kBlock];
  // Pass 1: bases, raw flags, canonical offsets.
  for (int r = 0; r < n; ++r) {
    const uint16_t* row = bits + static_cast<size_t>(r) * k;
    for (int b = 0; b < bpr; ++b) {
      load_block(row, k, b, v);
      unsigned lo = 255, hi = 0;
      for (int i = 0; i < kBlock; ++i) {
        const unsigned e = (v[i] >> 7) & 0xffu;
        lo = e < lo ? e : lo;
        hi = e > hi ? e : hi;
      }
      const bool raw = hi - lo > 15;
      metadata[static_cast<size_t>(r) * bpr + b] = static_cast<uint32_t>(offset / kUnit) |
                                                   (raw ? 0x80000000u : (static_cast<uint32_t>(lo) << 23));
      offset += raw ? kRawBytes : kCodedBytes;
    }
  }
  *payload_bytes = static_cast<size_t>(offset);
  if (offset > kMaxPayload) return KLAB_E_SHAPE;
  if (!payload) return 0;
  if (payload_capacity < offset) return KLAB_E_INVALID;
  // Pass 2: write the blocks.
  for (int r = 0; r < n; ++r) {
    const uint16_t* row = bits + static_cast<size_t>(r) * k;
    for (int b = 0; b < bpr; ++b) {
      load_block(row, k, b, v);
      const uint32_t meta = metadata[static_cast<size_t>(r) * bpr + b];
      uint8_t* dst = payload + static_cast<size_t>(meta & 0x7fffffu) * kUnit;
      if (meta >> 31) {
        for (int i = 0; i < kBlock; ++i) {
          dst[2 * i] = static_cast<uint8_t>(v[i] & 0xff);
          dst[2 * i + 1] = static_cast<uint8_t>(v[i] >> 8);
        }
      } else {
        const unsigned base = (meta >> 23) & 0xffu;
        for (int i = 0; i < kBlock; i += 2) {
          unsigned code[2];
          for (int h = 0; h < 2; ++h) {
            const unsigned u = v[i + h];
            code[h] = (u & 0x7fu) | ((u >> 8) & 0x80u) | ((((u >> 7) & 0xffu) - base) << 8);
          }
          uint8_t* p = dst + (i / 2) * 3;
          p[0] = static_cast<uint8_t>(code[0] & 0xff);
          p[1] = static_cast<uint8_t>(((code[0] >> 8) & 0xf) | ((code[1] & 0xf) << 4));
          p[2] = static_cast<uint8_t>((code[1] >> 4) & 0xff);
        }
      }
    }
  }
  return 0;
}

// Validates the canonical layout, exponent range and tail padding, and writes
// the original [N, K] bits. Returns KLAB_E_INVALID on any malformed input.
KLAB_API int klab_cbf16_unpack_host(const uint8_t* payload, size_t payload_bytes, const uint32_t* metadata, int n,
                                    int k, uint16_t* out) {
  if (!payload || !metadata || !out || n <= 0 || k <= 0) return KLAB_E_INVALID;
  if (static_cast<long long>(n) * k >= (1ll << 31) || payload_bytes > kMaxPayload) return KLAB_E_SHAPE;
  const int bpr = (k + kBlock - 1) / kBlock;
  uint64_t expect = 0;
  uint16_t v[kBlock];
  for (int r = 0; r < n; ++r) {
    for (int b = 0; b < bpr; ++b) {
      const uint32_t meta = metadata[static_cast<size_t>(r) * bpr + b];
      const bool raw = meta >> 31;
      const unsigned base = (meta >> 23) & 0xffu;
      if (raw && base) return KLAB_E_INVALID;
      if (static_cast<uint64_t>(meta & 0x7fffffu) * kUnit != expect) return KLAB_E_INVALID;
      const uint32_t size = raw ? kRawBytes : kCodedBytes;
      if (expect + size > payload_bytes) return KLAB_E_INVALID;
      const uint8_t* src = payload + expect;
      if (raw) {
        for (int i = 0; i < kBlock; ++i) v[i] = static_cast<uint16_t>(src[2 * i] | (src[2 * i + 1] << 8));
      } else {
        for (int i = 0; i < kBlock; i += 2) {
          const uint8_t* p = src + (i / 2) * 3;
          const unsigned code[2] = {p[0] | ((p[1] & 0xfu) << 8), (p[1] >> 4) | (static_cast<unsigned>(p[2]) << 4)};
          for (int h = 0; h < 2; ++h) {
            const unsigned e = base + (code[h] >> 8);
            if (e > 0xff) return KLAB_E_INVALID;
            v[i + h] = static_cast<uint16_t>((code[h] & 0x7fu) | ((code[h] & 0x80u) << 8) | (e << 7));
          }
        }
      }
      expect += size;
      uint16_t* row = out + static_cast<size_t>(r) * k;
      for (int i = 0; i < kBlock; ++i) {
        const int c = b * kBlock + i;
        if (c < k) {
          row[c] = v[i];
        } else if (v[i] != row[k - 1]) {
          return KLAB_E_INVALID;  // tail padding must repeat the row's last weight
        }
      }
    }
  }
  return expect == payload_bytes ? 0 : KLAB_E_INVALID;
}

}  // extern "C"
