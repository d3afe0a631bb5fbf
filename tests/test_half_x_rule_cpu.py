"""The FP16 staging rule of the INT8 / E2M1 projections, checked on the CPU.

The kernels stage a BF16 token t as FP16 after multiplying it by 2^s_t,
s_t = 142 - (largest exponent field of its nonzero values), when its nonzero
values have exponent fields in [39, 200] spanning at most 32 binades. These
tests restate that rule in numpy and check the two facts the kernels rely on:
inside the rule every scaled value is exact in FP16 (so the FP16 path multiplies
the same numbers as the FP32 path), and just outside it exactness fails, so the
rule is not looser than it must be."""

import numpy as np
import pytest


def bf16_values(sign, field, mant):
    """BF16 values from sign bits, exponent fields (1..254) and 7-bit mantissas."""
    bits = (sign.astype(np.uint32) << 15) | (field.astype(np.uint32) << 7) | mant.astype(np.uint32)
    return (bits << 16).astype(np.uint32).view(np.float32).astype(np.float64)


def rule(fields):
    fmin, fmax = int(fields.min()), int(fields.max())
    return fmin >= 39 and fmax <= 200 and fmax - fmin <= 32, 142 - fmax


def exact_in_f16(values):
    return np.array_equal(values.astype(np.float16).astype(np.float64), values)


@pytest.mark.parametrize("seed", range(40))
def test_tokens_inside_the_rule_are_exact_in_fp16(seed):
    rng = np.random.default_rng(seed)
    lo = int(rng.integers(39, 169))
    hi = int(min(200, lo + rng.integers(0, 33)))
    n = 4096
    fields = rng.integers(lo, hi + 1, n)
    fields[:2] = (lo, hi)
    x = bf16_values(rng.integers(0, 2, n), fields, rng.integers(0, 128, n))
    ok, s = rule(fields)
    assert ok
    scaled = x * 2.0 ** s
    assert exact_in_f16(scaled)
    assert np.abs(scaled).max() <= 65504.0
    # Unscaling by 2^-s gives the BF16 values back exactly.
    assert np.array_equal(scaled * 2.0 ** -s, x)


def test_range_just_outside_the_rule_loses_bits():
    # 33 binades: with s chosen for the largest value, the smallest value with a
    # full mantissa falls below FP16's 2^-24 resolution.
    fields = np.array([100, 133])
    ok, s = rule(fields)
    assert not ok
    x = bf16_values(np.array([0, 0]), fields, np.array([127, 127]))
    assert not exact_in_f16(x * 2.0 ** s)


def test_largest_value_stays_below_fp16_overflow():
    # The largest BF16 mantissa at the largest exponent scales to 65280 <= 65504.
    x = bf16_values(np.array([1]), np.array([200]), np.array([127]))
    _, s = rule(np.array([200]))
    assert x[0] * 2.0 ** s == -65280.0
    assert exact_in_f16(x * 2.0 ** s)


def test_field_limits_guard_fp32_range():
    # emin >= 39: the smallest product with an E2M1 weight (0.5) and an FP16
    # group scale (>= 2^-24) stays a normal FP32 number in the unscaled sums.
    smallest_x = 2.0 ** (39 - 127)
    assert smallest_x * 2.0 ** -7 * 0.5 * 2.0 ** -24 >= np.finfo(np.float32).tiny
    # emax <= 200: a full-range sum of K = 65536 products with |w| <= 127 stays finite.
    largest_x = 2.0 ** (200 - 127 + 1)
    assert largest_x * 127 * 65536 < np.finfo(np.float32).max
