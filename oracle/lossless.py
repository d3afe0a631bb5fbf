"""CPU restatement of the reference's two lossless FP32 weight formats.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU baseline, never by the product path.

Both formats keep every FP32 bit. The row-major [N, K] matrix (K % 64 == 0) is
cut into blocks of 64 consecutive weights; a block whose exponents all lie
within 15 of the block minimum stores 4-bit deltas, any other block ("wide")
stores the original exponents (v1) or the original words (fp28).

* v1 (lossless_weights.py:38-75): 3 bytes per weight (23 mantissa bits, sign at
  bit 23, little-endian), an exponent byte stream of 32 (nibble deltas) or 64
  (raw) bytes per block, metadata (offset/32) << 9 | base << 1 | wide.
* fp28 (packed_fp32.py:35-67): 28-bit codes significand | sign << 23 | delta << 24,
  eight codes in seven 32-bit words, least significant bit first, 56 words per
  block (or 64 original words when wide), metadata (offset/8) << 9 | base << 1 | wide.
"""

from __future__ import annotations

import numpy as np


def _blocks(w: np.ndarray):
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2 or w.shape[1] % 64:
        raise ValueError("expected FP32 [N, K] with K % 64 == 0")
    bits = w.view(np.uint32)
    exps = ((bits >> 23) & 0xFF).astype(np.int64).reshape(-1, 64)
    base = exps.min(axis=1)
    delta = exps - base[:, None]
    wide = delta.max(axis=1) > 15
    sig = ((bits & 0x7FFFFF) | ((bits >> 31) << 23)).astype(np.uint32)
    return bits, exps, base, delta, wide, sig


def lf32_pack(w: np.ndarray):
    """(mantissa u8 [N, 3K], exponents u8 [total], metadata i32 [N, K/64])."""
    bits, exps, base, delta, wide, sig = _blocks(w)
    n, k = w.shape
    mantissa = np.stack([sig & 0xFF, (sig >> 8) & 0xFF, (sig >> 16) & 0xFF], axis=-1).astype(np.uint8)
    mantissa = mantissa.reshape(n, 3 * k)
    chunks, offsets, off = [], [], 0
    for b in range(exps.shape[0]):
        if wide[b]:
            chunk = exps[b].astype(np.uint8)
        else:
            chunk = (delta[b, 0::2] | (delta[b, 1::2] << 4)).astype(np.uint8)
        offsets.append(off)
        chunks.append(chunk)
        off += chunk.size
    exponents = np.concatenate(chunks) if chunks else np.zeros(0, np.uint8)
    offsets = np.array(offsets, dtype=np.int64)
    meta = ((offsets >> 5) << 9) | (base << 1) | wide.astype(np.int64)
    return mantissa, exponents, meta.astype(np.uint32).view(np.int32).reshape(n, k // 64)


def lf32_unpack(mantissa: np.ndarray, exponents: np.ndarray, metadata: np.ndarray) -> np.ndarray:
    """Exact FP32 [N, K] from the v1 format."""
    n = metadata.shape[0]
    k = metadata.shape[1] * 64
    m = np.asarray(mantissa, np.uint32).reshape(n * k, 3)
    sig = m[:, 0] | (m[:, 1] << 8) | (m[:, 2] << 16)
    meta = np.asarray(metadata).view(np.uint32).reshape(-1).astype(np.int64)
    exps = np.empty(n * k, dtype=np.uint32)
    for b, word in enumerate(meta):
        off = (word >> 9) << 5
        if word & 1:
            exps[64 * b:64 * b + 64] = exponents[off:off + 64]
        else:
            packed = exponents[off:off + 32].astype(np.uint32)
            d = np.empty(64, dtype=np.uint32)
            d[0::2], d[1::2] = packed & 0xF, packed >> 4
            exps[64 * b:64 * b + 64] = ((word >> 1) & 0xFF) + d
    bits = (sig & 0x7FFFFF) | ((sig >> 23) << 31) | (exps << 23)
    return bits.astype(np.uint32).view(np.float32).reshape(n, k)


def fp28_pack(w: np.ndarray):
    """(payload i32 [total], metadata i32 [N, K/64])."""
    bits, exps, base, delta, wide, sig = _blocks(w)
    n, k = w.shape
    codes = (sig.reshape(-1, 64).astype(np.uint64) | (delta.astype(np.uint64) << 24))
    words, offsets, off = [], [], 0
    flat_bits = bits.reshape(-1, 64)
    for b in range(codes.shape[0]):
        if wide[b]:
            block = flat_bits[b].astype(np.uint32)
        else:
            acc, nacc, out = 0, 0, []
            for c in codes[b]:
                acc |= int(c & 0x0FFFFFFF) << nacc
                nacc += 28
                while nacc >= 32:
                    out.append(acc & 0xFFFFFFFF)
                    acc >>= 32
                    nacc -= 32
            assert nacc == 0 and len(out) == 56
            block = np.array(out, dtype=np.uint32)
        offsets.append(off)
        words.append(block)
        off += block.size
    payload = np.concatenate(words) if words else np.zeros(0, np.uint32)
    offsets = np.array(offsets, dtype=np.int64)
    meta = ((offsets >> 3) << 9) | (base << 1) | wide.astype(np.int64)
    return payload.view(np.int32), meta.astype(np.uint32).view(np.int32).reshape(n, k // 64)


def fp28_unpack(payload: np.ndarray, metadata: np.ndarray) -> np.ndarray:
    n = metadata.shape[0]
    k = metadata.shape[1] * 64
    words = np.asarray(payload).view(np.uint32)
    meta = np.asarray(metadata).view(np.uint32).reshape(-1).astype(np.int64)
    out = np.empty(n * k, dtype=np.uint32)
    for b, word in enumerate(meta):
        off = (word >> 9) << 3
        if word & 1:
            out[64 * b:64 * b + 64] = words[off:off + 64]
            continue
        stream = 0
        for i, v in enumerate(words[off:off + 56]):
            stream |= int(v) << (32 * i)
        base = (word >> 1) & 0xFF
        for j in range(64):
            code = (stream >> (28 * j)) & 0x0FFFFFFF
            out[64 * b + j] = (code & 0x7FFFFF) | (((code >> 23) & 1) << 31) | ((base + (code >> 24)) << 23)
    return out.view(np.float32).reshape(n, k)
