"""BF16 bit helpers, FP64 -> BF16 rounding and the output tolerance check.

Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np

# projection_accuracy.py:13-14
ATOL = 1e-5
RTOL = 1e-4


def bf16_values(bits) -> np.ndarray:
    """uint16 BF16 bit patterns -> exact float64 values (bits << 16 as FP32)."""
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32).astype(np.float64)


def f32_to_bf16_bits(values) -> np.ndarray:
    """FP32 -> BF16 bits, round to nearest even, NaN -> 0x7FC0 (torch's
    .to(torch.bfloat16) conversion)."""
    f = np.ascontiguousarray(values, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)
    return np.where(np.isnan(f), 0x7FC0, rounded).astype(np.uint16)


@lru_cache(maxsize=1)
def _finite_grid():
    """Sorted finite BF16 values with their bit codes, plus virtual +-2^128
    neighbours so that overflow rounds at the IEEE midpoint
    (projection_accuracy.py:21-30)."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    bits = bits[(bits & 0x7F80) != 0x7F80]
    values = bf16_values(bits)
    values = np.concatenate((values, np.array([-(2.0 ** 128), 2.0 ** 128])))
    bits = np.concatenate((bits, np.array([0xFF80, 0x7F80], dtype=np.uint16)))
    order = np.argsort(values, kind="stable")
    return values[order], bits[order]


def round_bf16_bits(reference64) -> np.ndarray:
    """FP64 -> nearest BF16 bits, ties to even, no intermediate FP32 rounding;
    a result of zero keeps the sign of the input (projection_accuracy.py:33-59)."""
    ref = np.asarray(reference64, dtype=np.float64)
    if not np.isfinite(ref).all():
        raise ValueError("round_bf16_bits expects finite values")
    grid, codes = _finite_grid()
    hi = np.searchsorted(grid, ref).clip(1, len(grid) - 1)
    lo = hi - 1
    d_lo, d_hi = ref - grid[lo], grid[hi] - ref
    take_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((codes[hi] & 1) == 0))
    out = np.where(take_hi, codes[hi], codes[lo]).astype(np.uint16)
    zero = (out & 0x7FFF) == 0
    return np.where(zero, np.where(np.signbit(ref), 0x8000, 0), out).astype(np.uint16)


def _as64(value) -> np.ndarray:
    if isinstance(value, np.ndarray):
        return value.astype(np.float64, copy=False)
    if hasattr(value, "detach"):
        return value.detach().cpu().double().numpy()
    return np.asarray(value, dtype=np.float64)


def _order(bits) -> np.ndarray:
    """Monotone integer rank of BF16 bit patterns (for ULP distances)."""
    b = np.asarray(bits, dtype=np.int64)
    return np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + b)


def check_outputs(reference64, output, *, output_dtype) -> dict:
    """Tolerance check of projection outputs against an FP64 reference
    (projection_accuracy.py:62-101): every element finite; FP32 outputs within
    atol + rtol*|ref|; BF16 outputs representable in BF16 and inside the BF16
    rounding of [ref - tol, ref + tol]. Reports ULP diagnostics for BF16."""
    name = str(output_dtype).removeprefix("torch.")
    name = {"bfloat16": "bf16", "float32": "fp32"}.get(name, name)
    if name not in ("bf16", "fp32"):
        raise ValueError("Expected bf16 or fp32 output contract")
    ref, act = _as64(reference64), _as64(output)
    if ref.shape != act.shape or ref.size == 0:
        raise ValueError("Reference and output shapes must be equal and nonempty")
    finite = np.isfinite(ref) & np.isfinite(act)
    if not finite.all():
        bad = int(np.count_nonzero(~finite))
        return {"passed": False, "elements_checked": int(ref.size), "nonfinite": bad, "violations": bad}
    tol = ATOL + RTOL * np.abs(ref)
    delta = np.abs(act - ref)
    extra = {}
    if name == "bf16":
        act_bits = round_bf16_bits(act)
        if not np.array_equal(bf16_values(act_bits), act):
            raise ValueError("Output is not representable in BF16")
        low = bf16_values(round_bf16_bits(ref - tol))
        high = bf16_values(round_bf16_bits(ref + tol))
        ok = (act >= low) & (act <= high)
        ref_bits = round_bf16_bits(ref)
        ulps = np.abs(_order(act_bits) - _order(ref_bits))
        extra = {"exact_rounding_fraction": float(np.mean(act == bf16_values(ref_bits))),
                 "within_one_ulp_fraction": float(np.mean(ulps <= 1)),
                 "max_ulp_error": int(ulps.max())}
    else:
        ok = delta <= tol
    norm = np.linalg.norm(ref.reshape(-1))
    return {"passed": bool(ok.all()), "elements_checked": int(ref.size),
            "violations": int(np.count_nonzero(~ok)), "nonfinite": 0,
            "max_abs_error": float(delta.max()),
            "relative_l2_error": float(np.linalg.norm(delta.reshape(-1)) / norm) if norm else None,
            "atol": ATOL, "rtol": RTOL, **extra}
