"""Signed INT8 weight-only projections on B200 (drop-in for int8_weights.py).

Two scale layouts share one kernel family:
* the reference format, an FP32 scale per 64 values (scales [N, K/64],
  int8_weights.py:23-35), x FP16/FP32 (the reference) or BF16, FP32 output;
* per-row FP32 scales (scales [N], benchmark config 2), x BF16, BF16 or FP32 output.
Codes are decoded to exact FP32 in registers; the product with the scale is
one FP32 multiply per 64-value group (per row for per-row scales).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from ._module import get_module

THREADS = (32, 64, 128, 256)
_XDT = {torch.bfloat16: _native.DT_BF16, torch.float16: _native.DT_F16, torch.float32: _native.DT_F32}
_ODT = {torch.bfloat16: _native.DT_BF16, torch.float32: _native.DT_F32}


@dataclass(frozen=True)
class Int8Weights:
    codes: torch.Tensor   # int8 [N, K]
    scales: torch.Tensor  # fp32 [N, K/64] (reference) or [N] (per row)

    def dequantize(self):
        """code * scale in FP32 (int8_weights.py:15-17); bit-exact on CUDA and CPU."""
        n, k = self.codes.shape
        if self.codes.is_cuda:
            out = torch.empty((n, k), dtype=torch.float32, device=self.codes.device)
            group = 0 if self.scales.ndim == 1 else 64
            stream = torch.cuda.current_stream(self.codes.device)
            with torch.cuda.device(self.codes.device):
                rc = _native.lib().klab_int8_dequantize(self.codes.data_ptr(), self.scales.data_ptr(), group,
                                                        out.data_ptr(), n, k, stream.cuda_stream)
            _native.check(rc, "klab_int8_dequantize")
            _native.record(stream, self.codes, self.scales, out)
            return out
        if self.scales.ndim == 1:
            return self.codes.float() * self.scales[:, None]
        return (self.codes.float().reshape(n, k // 64, 64) * self.scales.unsqueeze(-1)).reshape(n, k)

    def linear(self, x, threads=128, output_dtype=torch.float32):
        if self.scales.ndim == 1 or x.dtype == torch.bfloat16 or output_dtype != torch.float32:
            return fused_linear(x, self.codes, self.scales, threads, output_dtype=output_dtype)
        return int8_linear(x, self.codes, self.scales, threads)


def _quantize_groups(blocks, ieee_division=False):
    """ieee_division=False divides by the Python number 127 as the reference does
    (on CUDA: a multiply by fl32(1/127)); True divides by a device tensor (IEEE)."""
    amax = blocks.abs().amax(-1)
    tiny = torch.finfo(torch.float32).tiny
    divisor = amax.new_tensor(127.0) if ieee_division else 127
    scale = torch.where(amax > 0, (amax / divisor).clamp_min(tiny), torch.ones_like(amax))
    codes = torch.round(blocks / scale.unsqueeze(-1)).clamp_(-127, 127).to(torch.int8)
    return codes, scale


def _check_source(w, multiple):
    if w.device.type != "cuda" or w.dtype != torch.float32 or w.ndim != 2 or not w.is_contiguous():
        raise ValueError("Expected contiguous CUDA FP32 weights [N,K]")
    if w.requires_grad or min(w.shape) <= 0 or w.shape[1] % multiple:
        raise ValueError(f"Inference only; positive N and K divisible by {multiple} required")
    if not torch.isfinite(w).all():
        raise ValueError("Finite weights required")


def quantize_weights(w):
    """Reference format: scale per 64 = max|w|/127 (tiny-clamped, 1.0 for zero
    groups), code = clamp(round_half_even(w/scale), +-127) (int8_weights.py:23-35)."""
    _check_source(w, 64)
    n, k = w.shape
    codes, scale = _quantize_groups(w.reshape(n, k // 64, 64))
    return Int8Weights(codes.reshape(n, k).contiguous(), scale.contiguous())


def quantize_weights_per_row(w):
    """Per-row scale = max|row|/127 with an IEEE division (benchmark config 2),
    otherwise the reference's rounding rules."""
    _check_source(w, 1)
    n, k = w.shape
    codes, scale = _quantize_groups(w.reshape(n, 1, k), ieee_division=True)
    return Int8Weights(codes.reshape(n, k).contiguous(), scale.reshape(n).contiguous())


def fused_linear(x, codes, scales, threads=128, out=None, *, output_dtype=torch.float32):
    """out[M,N] = x[M,K] @ dequant(codes).T with FP32 accumulation."""
    for tensor in (x, codes, scales):
        if not isinstance(tensor, torch.Tensor) or tensor.device.type != "cuda" or not tensor.is_contiguous() \
                or tensor.requires_grad:
            raise ValueError("Inference-only contiguous tensors on the current CUDA device required")
    if x.device != codes.device or x.device != scales.device:
        raise ValueError("Inference-only contiguous tensors on the current CUDA device required")
    if x.dtype not in _XDT or x.ndim != 2:
        raise ValueError("Expected FP16/FP32/BF16 activations [M,K]")
    if codes.dtype != torch.int8 or codes.ndim != 2 or scales.dtype != torch.float32:
        raise ValueError("Expected INT8 codes and FP32 scales")
    if output_dtype not in _ODT:
        raise ValueError("output_dtype must be torch.float32 or torch.bfloat16")
    m, k = x.shape
    n = codes.shape[0]
    per_row = scales.ndim == 1
    if min(m, n, k) <= 0 or codes.shape[1] != k:
        raise ValueError("Invalid 64-value group dimensions")
    if per_row:
        if scales.shape != (n,):
            raise ValueError("Per-row scales must be [N]")
    elif k % 64 or scales.shape != (n, k // 64):
        raise ValueError("Invalid 64-value group dimensions")
    if max(m * k, n * k, m * n) >= 2 ** 31 or codes.data_ptr() % 4:
        raise ValueError("Require 32-bit indices and aligned codes")
    if threads not in THREADS:
        raise ValueError("Unsupported block size")
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=output_dtype)
    else:
        if out.dtype != output_dtype or out.device != x.device or not out.is_contiguous() or out.requires_grad:
            raise ValueError("Only contiguous output tensors of the requested dtype are supported")
        if out.shape != (m, n):
            raise ValueError("Output shape mismatch")
    if any(out.untyped_storage().data_ptr() == v.untyped_storage().data_ptr() for v in (x, codes, scales)):
        raise ValueError("Output may not alias inputs")
    get_module(x.device)
    wfmt = _native.W_I8_ROW if per_row else _native.W_I8_G64
    return _native.gemv(wfmt, _XDT[x.dtype], x, codes, scales, None, out, _ODT[output_dtype], m, n, k)


@torch.library.custom_op("kernel_lab::int8_linear", mutates_args=(), device_types="cuda")
def int8_linear(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, threads: int = 128) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return fused_linear(x, codes, scales, threads)


@int8_linear.register_fake
def _int8_fake(x, codes, scales, threads=128):
    return torch.empty((x.shape[0], codes.shape[0]), device=x.device, dtype=torch.float32)
