"""Lossless BF16 codec, format version 1 -- numpy restatement.

Test infrastructure only (see oracle/__init__.py). Format (docs/bf16-format.md:7-27,
compressed_bf16.py:84-151):

* [N, K] uint16 BF16 bits, row-major; each row is ceil(K/64) blocks of 64; a
  short last block is padded by repeating the row's last weight.
* per block one uint32 metadata word: bits 0-22 payload offset in 32-byte
  units, bits 23-30 base exponent, bit 31 raw flag; blocks are laid out
  sequentially (canonical layout), payload <= 256 MiB.
* coded block (max exponent - min exponent <= 15): base = min exponent, 64
  twelve-bit codes sm | (exponent - base) << 8 with sm = (u & 127) | ((u >> 8) & 128),
  packed LSB-first, 3 bytes per code pair, 96 bytes;
* raw block: the 64 original uint16 values, 128 bytes, base 0.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

BLOCK = 64
CODED_BYTES = 96
RAW_BYTES = 128
UNIT = 32
MAX_PAYLOAD_BYTES = 1 << 28
OFFSET_MASK = 0x7FFFFF
RAW_FLAG = 0x80000000


@dataclass(frozen=True)
class Packed:
    payload: np.ndarray   # uint8
    metadata: np.ndarray  # uint32
    n: int
    k: int
    source_sha256: str

    @property
    def storage_bytes(self) -> int:
        return int(self.payload.nbytes + self.metadata.nbytes)


def _blocks(bits: np.ndarray) -> np.ndarray:
    """[N, K] -> [N * ceil(K/64), 64], padding each row with its last weight."""
    n, k = bits.shape
    padded = ((k + BLOCK - 1) // BLOCK) * BLOCK
    if padded != k:
        bits = np.concatenate([bits, np.repeat(bits[:, -1:], padded - k, axis=1)], axis=1)
    return np.ascontiguousarray(bits).reshape(-1, BLOCK)


def pack_bits(bits: np.ndarray) -> Packed:
    """Encode BF16 bits (compressed_bf16.py:99-151). Every bit is preserved."""
    if not isinstance(bits, np.ndarray) or bits.dtype != np.uint16 or bits.ndim != 2:
        raise ValueError("Expected a two-dimensional uint16 array of BF16 bits")
    n, k = map(int, bits.shape)
    if min(n, k) <= 0 or n * k >= 2 ** 31:
        raise ValueError("N and K must be positive with N*K < 2^31")
    blocks = _blocks(bits.astype("<u2"))
    exponent = ((blocks >> 7) & 0xFF).astype(np.int32)
    lo, hi = exponent.min(axis=1), exponent.max(axis=1)
    raw = (hi - lo) > 15
    base = np.where(raw, 0, lo).astype(np.uint32)
    units = np.where(raw, RAW_BYTES // UNIT, CODED_BYTES // UNIT).astype(np.int64)
    start = np.cumsum(units) - units
    total = int(units.sum()) * UNIT
    if total > MAX_PAYLOAD_BYTES:
        raise ValueError("Payload exceeds the 256 MiB offset range")
    metadata = (start.astype(np.uint32) | (base << np.uint32(23)) |
                (raw.astype(np.uint32) << np.uint32(31))).astype(np.uint32)

    payload = np.zeros(total, dtype=np.uint8)
    byte_start = start * UNIT
    coded = ~raw
    if coded.any():
        b = blocks[coded].astype(np.uint32)
        sm = (b & 0x7F) | ((b >> 8) & 0x80)
        delta = ((b >> 7) & 0xFF) - base[coded][:, None]
        code = sm | (delta << 8)
        a, c = code[:, 0::2], code[:, 1::2]
        triple = np.stack([a & 0xFF, ((a >> 8) & 0xF) | ((c & 0xF) << 4), (c >> 4) & 0xFF], axis=-1)
        data = triple.reshape(-1, CODED_BYTES).astype(np.uint8)
        idx = byte_start[coded][:, None] + np.arange(CODED_BYTES)
        payload[idx] = data
    if raw.any():
        data = blocks[raw].astype("<u2").view(np.uint8).reshape(-1, RAW_BYTES)
        idx = byte_start[raw][:, None] + np.arange(RAW_BYTES)
        payload[idx] = data
    digest = hashlib.sha256(np.ascontiguousarray(bits, dtype="<u2").tobytes()).hexdigest()
    return Packed(payload, metadata, n, k, digest)


def _check_layout(payload: np.ndarray, metadata: np.ndarray, n: int, k: int):
    """Canonical-layout validation (compressed_bf16.py:162-200)."""
    if payload.dtype != np.uint8 or payload.ndim != 1:
        raise ValueError("Payload must be 1-D uint8")
    if metadata.dtype != np.uint32 or metadata.ndim != 1:
        raise ValueError("Metadata must be 1-D uint32")
    if min(n, k) <= 0 or n * k >= 2 ** 31:
        raise ValueError("N and K must be positive with N*K < 2^31")
    count = n * ((k + BLOCK - 1) // BLOCK)
    if metadata.size != count:
        raise ValueError("Metadata must hold one word per 64-weight block")
    if payload.size > MAX_PAYLOAD_BYTES:
        raise ValueError("Payload exceeds the version-1 offset range")
    raw = (metadata >> 31) != 0
    base = (metadata >> 23) & 0xFF
    if np.any(raw & (base != 0)):
        raise ValueError("Raw blocks must have base exponent zero")
    units = np.where(raw, RAW_BYTES // UNIT, CODED_BYTES // UNIT).astype(np.int64)
    start = np.cumsum(units) - units
    if not np.array_equal((metadata & OFFSET_MASK).astype(np.int64), start):
        raise ValueError("Block offsets are not the canonical sequential layout")
    if int(units.sum()) * UNIT != payload.size:
        raise ValueError("Payload length does not match its block metadata")
    return raw, base.astype(np.uint32), start * UNIT


def unpack_bits(packed: Packed) -> np.ndarray:
    """Decode to the original [N, K] bits after validation (compressed_bf16.py:232-243):
    exponent overflow, tail padding and the source SHA-256 are checked."""
    n, k = int(packed.n), int(packed.k)
    raw, base, byte_start = _check_layout(packed.payload, packed.metadata, n, k)
    count = raw.size
    out = np.empty((count, BLOCK), dtype=np.uint16)
    coded = ~raw
    if coded.any():
        idx = byte_start[coded][:, None] + np.arange(CODED_BYTES)
        t = packed.payload[idx].reshape(-1, BLOCK // 2, 3).astype(np.uint32)
        a = t[..., 0] | ((t[..., 1] & 0xF) << 8)
        c = (t[..., 1] >> 4) | (t[..., 2] << 4)
        code = np.stack([a, c], axis=-1).reshape(-1, BLOCK)
        exponent = base[coded][:, None] + (code >> 8)
        if np.any(exponent > 0xFF):
            raise ValueError("Decoded exponent overflows BF16")
        out[coded] = ((code & 0x7F) | ((code & 0x80) << 8) | (exponent << 7)).astype(np.uint16)
    if raw.any():
        idx = byte_start[raw][:, None] + np.arange(RAW_BYTES)
        out[raw] = packed.payload[idx].reshape(-1, RAW_BYTES).view("<u2")
    padded = ((k + BLOCK - 1) // BLOCK) * BLOCK
    rows = out.reshape(n, padded)
    if padded != k and np.any(rows[:, k:] != rows[:, k - 1:k]):
        raise ValueError("Tail padding must repeat each row's last weight")
    result = np.ascontiguousarray(rows[:, :k])
    if hashlib.sha256(result.astype("<u2").tobytes()).hexdigest() != packed.source_sha256:
        raise ValueError("Decoded bits do not match source_sha256")
    return result


def decode_bf16(payload: bytes, metadata: np.ndarray, n: int, k: int) -> np.ndarray:
    """Independent bit-stream decoder (bf16_reference.py:10-46): reads code i as
    bits [12i, 12i+12) of the block with np.unpackbits, no shift arithmetic."""
    if type(n) is not int or type(k) is not int or min(n, k) <= 0 or n * k >= 2 ** 31:
        raise ValueError("Expected positive N,K within signed 32-bit indexing")
    data = np.frombuffer(payload, dtype=np.uint8)
    raw, base, byte_start = _check_layout(data, np.asarray(metadata), n, k)
    out = np.empty((raw.size, BLOCK), dtype=np.uint16)
    weights = (1 << np.arange(12, dtype=np.uint32))
    coded = np.nonzero(~raw)[0]
    if coded.size:
        stream = np.unpackbits(data[byte_start[coded][:, None] + np.arange(CODED_BYTES)], axis=1,
                               bitorder="little").reshape(-1, BLOCK, 12)
        code = (stream.astype(np.uint32) * weights).sum(axis=2, dtype=np.uint32)
        exponent = base[coded][:, None] + (code >> 8)
        if np.any(exponent > 0xFF):
            raise ValueError("Decoded exponent overflows BF16")
        out[coded] = ((code & 0x7F) | ((code & 0x80) << 8) | (exponent << 7)).astype(np.uint16)
    rawi = np.nonzero(raw)[0]
    if rawi.size:
        out[rawi] = data[byte_start[rawi][:, None] + np.arange(RAW_BYTES)].copy().view("<u2").reshape(-1, BLOCK)
    return out.reshape(n, -1)[:, :k]
