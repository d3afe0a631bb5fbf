"""Lossless FP32 weights, format v1 (drop-in for lossless_weights.py).

Every weight keeps its exact IEEE-754 bits: 3 bytes of sign and mantissa per
weight, per 64-weight block either 32 bytes of 4-bit exponent deltas or the 64
raw exponent bytes, one 32-bit metadata word per block (lossless_weights.py:38-75;
the format is documented in klab_b200/csrc/lossless_f32.cuh). The projection
decodes each 4 KiB item into shared memory and then uses the FP32 projection's
arithmetic, so its results equal klab_f32_linear on the unpacked weights bit
for bit.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from ._module import get_module

THREADS = (32, 64, 128, 256)


@dataclass(frozen=True)
class LosslessWeights:
    mantissa: torch.Tensor   # uint8 [N, 3K]
    exponents: torch.Tensor  # uint8 [total]
    metadata: torch.Tensor   # int32 [N, K/64]

    @property
    def shape(self):
        return self.mantissa.shape[0], self.mantissa.shape[1] // 3

    @property
    def storage_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.mantissa, self.exponents, self.metadata))

    def unpack(self):
        """The original FP32 [N, K] (exact bits)."""
        n, k = self.shape
        out = torch.empty(n, k, device=self.mantissa.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(self.mantissa.device)
        with torch.cuda.device(self.mantissa.device):
            rc = _native.lib().klab_lossless_f32_unpack(self.mantissa.data_ptr(), self.exponents.data_ptr(),
                                                        self.metadata.data_ptr(), out.data_ptr(), n * k,
                                                        stream.cuda_stream)
        _native.check(rc, "klab_lossless_f32_unpack")
        _native.record(stream, self.mantissa, self.exponents, self.metadata, out)
        return out

    def linear(self, x, threads=128):
        return lossless_linear(x, self.mantissa, self.exponents, self.metadata, threads)


def _blocks(w):
    """Exponents per 64-block, their minimum, deltas and the wide flags."""
    bits = w.view(torch.int32)
    exps = ((bits >> 23) & 0xFF).reshape(-1, 64)
    lo = exps.amin(dim=1)
    delta = exps - lo[:, None]
    return bits, exps, lo, delta, delta.amax(dim=1) > 15


def _scatter_blocks(rows, sizes, dtype, device):
    """Concatenate the first sizes[b] entries of rows[b] for every block b."""
    offsets = torch.cumsum(sizes, 0) - sizes
    total = int(sizes.sum().item())  # setup-time sizing
    out = torch.empty(total, dtype=dtype, device=device)
    col = torch.arange(rows.shape[1], device=device)
    keep = col[None, :] < sizes[:, None]
    out[(offsets[:, None] + col[None, :])[keep]] = rows[keep].to(dtype)
    return out, offsets, total


def pack_weights(w):
    """Pack CUDA FP32 [N, K] (K % 64 == 0) without losing a bit."""
    if w.device.type != "cuda" or w.dtype != torch.float32 or w.ndim != 2 or not w.is_contiguous():
        raise ValueError("Expected contiguous CUDA FP32 [N,K]")
    if w.requires_grad or min(w.shape) <= 0 or w.shape[1] % 64 or w.numel() * 3 >= 2 ** 31:
        raise ValueError("Inference-only, K divisible by 64, positive 32-bit-addressable storage required")
    n, k = w.shape
    bits, exps, lo, delta, wide = _blocks(w)
    sign_mant = (bits & 0x7FFFFF) | ((bits >> 8) & 0x800000)
    mantissa = torch.stack([(sign_mant >> s) & 0xFF for s in (0, 8, 16)], dim=-1).to(torch.uint8).reshape(n, 3 * k)
    nibbles = delta[:, 0::2] | (delta[:, 1::2] << 4)
    rows = torch.where(wide[:, None], exps, torch.nn.functional.pad(nibbles, (0, 32)))
    sizes = torch.where(wide, 64, 32).to(torch.int64)
    exponents, offsets, total = _scatter_blocks(rows, sizes, torch.uint8, w.device)
    if total >= 2 ** 28:
        raise ValueError("Exponent payload exceeds this experimental metadata format's 256 MiB limit")
    meta = ((offsets >> 5) << 9) | (lo.to(torch.int64) << 1) | wide.to(torch.int64)
    return LosslessWeights(mantissa.contiguous(), exponents, meta.to(torch.int32).reshape(n, k // 64).contiguous())


def fused_linear(x, packed, threads=128, out=None):
    """out[M, N] = x[M, K] @ W.T in FP32 with W decoded exactly
    (validation as lossless_weights.py:78-105)."""
    tensors = (x, packed.mantissa, packed.exponents, packed.metadata)
    for tensor in tensors:
        if tensor.device.type != "cuda" or tensor.device != x.device or not tensor.is_contiguous() \
                or tensor.requires_grad:
            raise ValueError("Inference-only contiguous tensors on the current CUDA device required")
    if x.dtype != torch.float32 or x.ndim != 2:
        raise ValueError("FP32 activations required")
    n, k = packed.shape
    if min(x.shape[0], n, k) <= 0 or x.shape[1] != k or k % 64:
        raise ValueError("Invalid dimensions")
    if max(x.numel(), n * k * 3, x.shape[0] * n) >= 2 ** 31 or x.data_ptr() % 16 or packed.mantissa.data_ptr() % 4:
        raise ValueError("Require 32-bit indexing and aligned FP32 input")
    if threads not in THREADS:
        raise ValueError("Unsupported block size")
    if packed.metadata.shape != (n, k // 64):
        raise ValueError("Invalid metadata dimensions")
    if any(v.dtype != torch.uint8 for v in (packed.mantissa, packed.exponents)):
        raise ValueError("Expected byte payloads")
    if packed.metadata.dtype != torch.int32 or packed.exponents.ndim != 1:
        raise ValueError("Invalid exponent offsets")
    m = x.shape[0]
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=torch.float32)
    else:
        if out.dtype != torch.float32 or out.device != x.device or not out.is_contiguous() or out.requires_grad:
            raise ValueError("Only contiguous FP32 output tensors are supported")
        if out.shape != (m, n):
            raise ValueError("Output shape mismatch")
    if any(out.untyped_storage().data_ptr() == v.untyped_storage().data_ptr() for v in tensors):
        raise ValueError("Output cannot alias inputs")
    get_module(x.device)
    stream = torch.cuda.current_stream(x.device)
    ws_ptr, ws_bytes = _native.workspace_for(_native.W_LF32, m, n, k, x.device.index, stream)
    with torch.cuda.device(x.device):
        rc = _native.lib().klab_lossless_f32_linear(x.data_ptr(), packed.mantissa.data_ptr(),
                                                    packed.exponents.data_ptr(), packed.metadata.data_ptr(),
                                                    out.data_ptr(), m, n, k, ws_ptr, ws_bytes, stream.cuda_stream)
    _native.check(rc, "klab_lossless_f32_linear")
    _native.record(stream, *tensors, out)
    return out


@torch.library.custom_op("kernel_lab::lossless_linear", mutates_args=(), device_types="cuda")
def lossless_linear(x: torch.Tensor, mantissa: torch.Tensor, exponents: torch.Tensor, metadata: torch.Tensor,
                    threads: int = 128) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return fused_linear(x, LosslessWeights(mantissa, exponents, metadata), threads)


@lossless_linear.register_fake
def _lossless_fake(x, mantissa, exponents, metadata, threads=128):
    return x.new_empty((x.shape[0], mantissa.shape[0]))
