"""Seeded synthetic inputs and FP64 reference projections.

Test infrastructure only (see oracle/__init__.py). The reference's accuracy
contract compares every projection output with x . W^T evaluated in FP64 over
the exact input values (projection_accuracy.py:1-10, verify_compressed.py
values64), then rounds once to BF16 (round_bf16_bits) or checks FP32 outputs
within atol + rtol*|ref| (check_outputs). Quantized weights enter as their
dequantized FP32 values (bench_int8.py:29-31, bench_fp4.py:38-43).
"""

from __future__ import annotations

import numpy as np

from .bf16 import bf16_values, f32_to_bf16_bits


def normal_f32(seed: int, shape, std: float = 1.0) -> np.ndarray:
    """Seeded N(0, std^2) FP32 values."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def normal_bf16_bits(seed: int, shape, std: float = 1.0) -> np.ndarray:
    """Seeded N(0, std^2) values rounded to BF16 (RNE); returns uint16 bits."""
    return f32_to_bf16_bits(normal_f32(seed, shape, std))


def projection64(x64: np.ndarray, w64: np.ndarray) -> np.ndarray:
    """FP64 x[M,K] . W[N,K]^T."""
    return np.asarray(x64, dtype=np.float64) @ np.asarray(w64, dtype=np.float64).T


def bf16_projection64(x_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """FP64 reference of a BF16 x BF16 projection (the exact values of both)."""
    return projection64(bf16_values(x_bits), bf16_values(w_bits))


def chain_reference_bf16(x_bits: np.ndarray, layers) -> np.ndarray:
    """Reference for a projection chain whose every output is rounded once to
    BF16: layers is a list of (w_bits, gather) stages applied in order, each
    stage y = round_bf16(x . W^T). Used for small chain parity cases."""
    from .bf16 import round_bf16_bits

    h = x_bits
    for w_bits in layers:
        h = round_bf16_bits(bf16_projection64(h, w_bits))
    return h


def residual_rmsnorm64(x: np.ndarray, residual: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """FP64 restatement of the reference's fused residual RMSNorm
    (kernels.cu:168-222, KernelLab.residual_rmsnorm kernel_lab.py:281-294):
    v = x + residual, y = (v / sqrt(mean(v^2, row) + eps)) * weight."""
    v = np.asarray(x, dtype=np.float64) + np.asarray(residual, dtype=np.float64)
    inv = 1.0 / np.sqrt(np.mean(v * v, axis=1, keepdims=True) + float(eps))
    return (v * inv) * np.asarray(weight, dtype=np.float64)[None, :]


def add_rmsnorm_ref(res_bits: np.ndarray, y_bits: np.ndarray, w_bits: np.ndarray, eps: float):
    """The reference's add_rmsnorm (research/l2-prefetch/src/decode_attn.cu:471-511):
    x = RNE_bf16(fp32(res) + fp32(y)) exactly (bits), and xn in FP64 from that x:
    x / sqrt(mean(x^2) + eps) * w (the kernel rounds xn once to BF16)."""
    from .bf16 import bf16_values, round_bf16_bits

    s32 = (bf16_values(res_bits).astype(np.float32) + bf16_values(y_bits).astype(np.float32))
    x_bits = round_bf16_bits(s32.astype(np.float64))
    x = bf16_values(x_bits)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + float(eps))
    return x_bits, (x * inv) * bf16_values(w_bits)[None, :]


def silu_mul64(gu_bits: np.ndarray) -> np.ndarray:
    """silu(gate) * up in FP64 for gu = [gate | up] (decode_attn.cu:513-527)."""
    from .bf16 import bf16_values

    g, u = np.split(bf16_values(gu_bits), 2, axis=1)
    return g / (1.0 + np.exp(-g)) * u
