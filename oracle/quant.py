"""INT8 and FP4 weight quantizers / dequantizers -- numpy restatement.

Test infrastructure only (see oracle/__init__.py). All arithmetic is IEEE FP32
with round-to-nearest-even, exactly as the reference's torch code computes it:

* Scalar divisors: the reference's quantizers run only on CUDA tensors, where
  torch divides a tensor by a Python number as a multiply by the FP32
  reciprocal (a * fl(1/b)); on CPU it is a true IEEE division. The two differ
  by one ulp in a few percent of groups. semantics="cuda" (default) reproduces
  the reference's device results; semantics="cpu" reproduces the same code run
  on CPU (how tests/golden/make_golden.py produced its fixtures).
* INT8, reference format (int8_weights.py:15-35): per 64-value group,
  scale = max|w|/127 (clamped to FP32 tiny; 1.0 for an all-zero group),
  code = clamp(round_half_even(w / scale), -127, 127); dequant = code * scale.
* INT8, per-row (benchmark config 2): one group per row, true IEEE division.
* FP4, reference format (fp4.py:21-60): global = max|W|/(448*6) (tiny-clamped,
  1.0 when W == 0); per 16 values an E4M3 scale = RNE_e4m3(min(max|g| / (6*global), 448));
  E2M1 codes by nearest value with ties to even (the bucketize + tie fix of
  fp4.py:53-58), sign bit from signbit(w / scale); low nibble = even k;
  dequant = e2m1 * (e4m3 * global).
* FP4, FP16 scale per 32 (benchmark config 3): scale = RNE_fp16(max|g| / 6)
  with a true IEEE division;
  codes as above against that scale; dequant = e2m1 * scale (exact in FP32).
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np

F32 = np.float32
TINY = np.finfo(np.float32).tiny
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
# Decision boundaries between neighbouring E2M1 magnitudes (fp4.py:53).
_E2M1_BOUNDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)


# ------------------------------------------------------------------ INT8

def scalar_divide(a, b: float, semantics: str) -> np.ndarray:
    """a / b for an FP32 array a and a Python number b, as torch computes it on
    `semantics` = "cuda" (a * fl32(1/b)) or "cpu" (IEEE division)."""
    a = np.asarray(a, dtype=F32)
    if semantics == "cuda":
        return (a * (F32(1) / F32(b))).astype(F32)
    if semantics == "cpu":
        return (a / F32(b)).astype(F32)
    raise ValueError("semantics must be 'cuda' or 'cpu'")


def _int8_quantize_groups(groups: np.ndarray, semantics: str):
    amax = np.abs(groups).max(axis=-1)
    scale = np.where(amax > 0, np.maximum(scalar_divide(amax, 127, semantics), TINY), F32(1)).astype(F32)
    codes = np.clip(np.rint(groups / scale[..., None]), -127, 127).astype(np.int8)
    return codes, scale


def _check_weights(w, multiple):
    if not isinstance(w, np.ndarray) or w.dtype != np.float32 or w.ndim != 2:
        raise ValueError("Expected FP32 weights [N, K]")
    n, k = w.shape
    if min(n, k) <= 0 or k % multiple:
        raise ValueError(f"Positive N and K divisible by {multiple} required")
    if not np.isfinite(w).all():
        raise ValueError("Finite weights required")
    return n, k


def int8_quantize_g64(w: np.ndarray, semantics: str = "cuda"):
    """Reference INT8 format (int8_weights.py:23-35): codes int8 [N,K], scales fp32 [N,K/64]."""
    n, k = _check_weights(w, 64)
    codes, scales = _int8_quantize_groups(w.reshape(n, k // 64, 64), semantics)
    return codes.reshape(n, k), scales


def int8_quantize_row(w: np.ndarray):
    """Per-row INT8 (benchmark config 2): codes int8 [N,K], scales fp32 [N]."""
    n, k = _check_weights(w, 1)
    codes, scales = _int8_quantize_groups(w.reshape(n, 1, k), "cpu")
    return codes.reshape(n, k), scales.reshape(n)


def int8_dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """code * scale in FP32 (int8_weights.py:15-17); scales [N,K/64] or [N]."""
    n, k = codes.shape
    if scales.ndim == 1:
        return (codes.astype(F32) * scales[:, None]).astype(F32)
    g = k // scales.shape[1]
    return (codes.astype(F32).reshape(n, -1, g) * scales[..., None]).reshape(n, k).astype(F32)


# ------------------------------------------------------------------ FP8 / FP4 primitives

@lru_cache(maxsize=1)
def _e4m3_grid():
    """Non-negative E4M3 (fn) values 0x00..0x7E plus a virtual 480 -> NaN code."""
    codes = np.arange(0x7F, dtype=np.uint8)
    values = e4m3_to_f32(codes).astype(np.float64)
    return np.concatenate([values, [480.0]]), np.concatenate([codes, [0x7F]]).astype(np.uint8)


def e4m3_to_f32(codes) -> np.ndarray:
    """E4M3 (fn) bytes -> FP32: bias 7, subnormals m * 2^-9, 0x7F / 0xFF NaN."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.uint32)
    e, m = (c >> 3) & 15, c & 7
    mag = np.where(e == 0, m.astype(np.float64) * 2.0 ** -9,
                   (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7.0))
    mag = np.where((c & 0x7F) == 0x7F, np.nan, mag)
    return np.where(c & 0x80, -mag, mag).astype(F32)


def f32_to_e4m3(values) -> np.ndarray:
    """FP32 -> E4M3 (fn) bytes, round to nearest even, |x| >= 464 -> NaN (0x7F)
    (torch's float8_e4m3fn conversion, used at fp4.py:50)."""
    v = np.asarray(values, dtype=F32).astype(np.float64)
    grid, codes = _e4m3_grid()
    mag = np.abs(v)
    hi = np.searchsorted(grid, mag).clip(1, len(grid) - 1)
    lo = hi - 1
    d_lo, d_hi = mag - grid[lo], grid[hi] - mag
    take_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((codes[hi] & 1) == 0))
    out = np.where(take_hi, codes[hi], codes[lo]).astype(np.uint8)
    out = np.where(mag == 0, 0, out).astype(np.uint8)
    out = np.where(np.isnan(v) | (mag >= 480.0), 0x7F, out).astype(np.uint8)
    return (out | np.where(np.signbit(v), 0x80, 0).astype(np.uint8)).astype(np.uint8)


def e2m1_codes(normalized: np.ndarray) -> np.ndarray:
    """Nearest E2M1 code, ties to the even mantissa, sign from signbit (fp4.py:52-59)."""
    mag = np.abs(normalized)
    code = np.searchsorted(_E2M1_BOUNDS, mag, side="left").astype(np.uint8)
    for lower, bound in ((1, 0.75), (3, 1.75), (5, 3.5)):
        code = np.where(mag == F32(bound), lower + 1, code).astype(np.uint8)
    return (code | (np.signbit(normalized).astype(np.uint8) << 3)).astype(np.uint8)


def e2m1_to_f32(codes) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8)
    v = E2M1_VALUES[c & 7]
    return np.where(c & 8, -v, v).astype(F32)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """[N, K] 4-bit codes -> [N, K/2] bytes, low nibble = even k (fp4.py:59)."""
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    n, half = packed.shape
    return np.stack([packed & 15, packed >> 4], axis=-1).reshape(n, 2 * half).astype(np.uint8)


# ------------------------------------------------------------------ FP4 formats

def fp4_quantize_e4m3(w: np.ndarray, semantics: str = "cuda"):
    """Reference FP4 format (fp4.py:33-60): packed uint8 [N,K/2], E4M3 scale bytes
    [N,K/16], global scale fp32 (shape ())."""
    n, k = _check_weights(w, 16)
    blocks = w.reshape(n, k // 16, 16)
    amax = np.abs(w).max()
    glob = F32(max(scalar_divide(amax, 448.0 * 6.0, semantics), TINY)) if amax > 0 else F32(1)
    block_scale = np.minimum(np.abs(blocks).max(axis=-1) / (F32(6.0) * glob), F32(448)).astype(F32)
    scales = f32_to_e4m3(block_scale)
    decoded = (e4m3_to_f32(scales) * glob).astype(F32)
    normalized = (blocks / np.maximum(decoded, TINY)[..., None]).astype(F32)
    codes = e2m1_codes(normalized).reshape(n, k)
    return pack_nibbles(codes), scales, np.array(glob, dtype=F32)


def fp4_dequantize_e4m3(packed, scales, glob) -> np.ndarray:
    """e2m1 * (e4m3 * global) in FP32 (fp4.py:21-27)."""
    n = packed.shape[0]
    values = e2m1_to_f32(unpack_nibbles(packed))
    scale = (e4m3_to_f32(scales) * F32(glob)).astype(F32)
    return (values.reshape(n, -1, 16) * scale[..., None]).reshape(n, -1).astype(F32)


def fp4_quantize_f16(w: np.ndarray):
    """FP4 with an FP16 scale per 32 (benchmark config 3): packed [N,K/2],
    scales float16 [N,K/32]."""
    n, k = _check_weights(w, 32)
    blocks = w.reshape(n, k // 32, 32)
    scale16 = (np.abs(blocks).max(axis=-1) / F32(6.0)).astype(F32).astype(np.float16)
    decoded = scale16.astype(F32)
    normalized = (blocks / np.maximum(decoded, TINY)[..., None]).astype(F32)
    return pack_nibbles(e2m1_codes(normalized).reshape(n, k)), scale16


def fp4_dequantize_f16(packed, scales16) -> np.ndarray:
    n = packed.shape[0]
    values = e2m1_to_f32(unpack_nibbles(packed))
    return (values.reshape(n, -1, 32) * scales16.astype(F32)[..., None]).reshape(n, -1).astype(F32)
