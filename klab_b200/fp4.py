"""FP4 (E2M1) weight projections on B200 (drop-in for fp4.py).

Two scale layouts share one kernel family:
* the reference format (fp4.py:33-60): an E4M3 scale per 16 values and one
  FP32 global scale, x FP16/FP32 (reference) or BF16, FP32 output;
* an FP16 scale per 32 values (benchmark config 3), x BF16, BF16 or FP32 output.
Two codes per byte, low nibble = even k. E2M1 codes are converted with the
hardware cvt.rn.f16x2.e2m1x2 and widened to FP32 in registers; each scale is
applied once per group to the group's FP32 partial sum.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from ._module import get_module

THREADS = (32, 64, 128, 256)
_XDT = {torch.bfloat16: _native.DT_BF16, torch.float16: _native.DT_F16, torch.float32: _native.DT_F32}
_ODT = {torch.bfloat16: _native.DT_BF16, torch.float32: _native.DT_F32}
_MAGNITUDES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _dequantize_native(packed, scales, kind, global_scale):
    n, half_k = packed.shape
    out = torch.empty((n, 2 * half_k), dtype=torch.float32, device=packed.device)
    stream = torch.cuda.current_stream(packed.device)
    with torch.cuda.device(packed.device):
        rc = _native.lib().klab_fp4_dequantize(packed.data_ptr(), scales.data_ptr(), kind,
                                               None if global_scale is None else global_scale.data_ptr(),
                                               out.data_ptr(), n, 2 * half_k, stream.cuda_stream)
    _native.check(rc, "klab_fp4_dequantize")
    _native.record(stream, packed, scales, global_scale, out)
    return out


def _e2m1_values(packed):
    n, half_k = packed.shape
    codes = torch.stack((packed & 15, packed >> 4), dim=-1).reshape(n, 2 * half_k)
    table = torch.tensor(_MAGNITUDES, device=packed.device)
    return table[(codes & 7).long()] * torch.where((codes & 8) != 0, -1.0, 1.0)


@dataclass(frozen=True)
class FP4Weights:
    """Reference format: packed [N,K/2] uint8, E4M3 scale bytes [N,K/16], FP32 global scale."""

    packed: torch.Tensor
    scales: torch.Tensor
    global_scale: torch.Tensor

    def dequantize(self):
        """e2m1 * (e4m3 * global) in FP32 (fp4.py:21-27)."""
        if self.packed.is_cuda:
            return _dequantize_native(self.packed, self.scales, _native.FP4_E4M3_G16, self.global_scale)
        n = self.packed.shape[0]
        scale = self.scales.view(torch.float8_e4m3fn).float() * self.global_scale
        return (_e2m1_values(self.packed).reshape(n, -1, 16) * scale.unsqueeze(-1)).reshape(n, -1)

    def linear(self, x, threads=128, output_dtype=torch.float32):
        if x.dtype == torch.bfloat16 or output_dtype != torch.float32:
            return fused_linear(x, self.packed, self.scales, self.global_scale, threads, output_dtype=output_dtype)
        return fp4_linear(x, self.packed, self.scales, self.global_scale, threads)


@dataclass(frozen=True)
class FP4F16Weights:
    """Benchmark format: packed [N,K/2] uint8, FP16 scales [N,K/32]."""

    packed: torch.Tensor
    scales: torch.Tensor

    def dequantize(self):
        """e2m1 * scale in FP32 (exact)."""
        if self.packed.is_cuda:
            return _dequantize_native(self.packed, self.scales, _native.FP4_F16_G32, None)
        n = self.packed.shape[0]
        return (_e2m1_values(self.packed).reshape(n, -1, 32) * self.scales.float().unsqueeze(-1)).reshape(n, -1)

    def linear(self, x, threads=128, output_dtype=torch.bfloat16):
        return fused_linear(x, self.packed, self.scales, None, threads, output_dtype=output_dtype)


def _check_source(w, multiple):
    if w.device.type != "cuda" or w.dtype != torch.float32 or w.ndim != 2 or not w.is_contiguous():
        raise ValueError("Weights must be contiguous CUDA FP32 [N,K]")
    if w.requires_grad or min(w.shape) <= 0 or w.shape[1] % multiple:
        raise ValueError(f"Inference only; positive N and K divisible by {multiple} required")
    if not torch.isfinite(w).all():
        raise ValueError("Quantization requires finite weights")


def _e2m1_codes(normalized):
    """Nearest E2M1 magnitude with ties to the even code, sign from signbit."""
    magnitude = normalized.abs().contiguous()
    bounds = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=normalized.device)
    codes = torch.bucketize(magnitude, bounds).to(torch.uint8)
    # bucketize puts an exact boundary in the lower bin; at the ties whose lower
    # neighbour has an odd mantissa the even neighbour is the upper one.
    for lower, bound in ((1, 0.75), (3, 1.75), (5, 3.5)):
        codes = torch.where(magnitude == bound, lower + 1, codes)
    return codes | (torch.signbit(normalized).to(torch.uint8) << 3)


def _pack(codes):
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()


def quantize_weights(w):
    """Reference format (fp4.py:33-60): global = max|W|/(448*6) (tiny-clamped,
    1.0 for W == 0); per 16 an E4M3 scale of min(max|g|/(6*global), 448);
    nearest-even E2M1 codes against the decoded scale."""
    _check_source(w, 16)
    n, k = w.shape
    blocks = w.reshape(n, k // 16, 16)
    tiny = torch.finfo(torch.float32).tiny
    amax = w.abs().amax()
    global_scale = torch.where(amax > 0, (amax / (448.0 * 6.0)).clamp_min(tiny), torch.ones_like(amax))
    scales = (blocks.abs().amax(-1) / (6.0 * global_scale)).clamp(max=448).to(torch.float8_e4m3fn)
    decoded = scales.float() * global_scale
    codes = _e2m1_codes(blocks / decoded.clamp_min(tiny).unsqueeze(-1)).reshape(n, k)
    return FP4Weights(_pack(codes), scales.view(torch.uint8).contiguous(), global_scale.contiguous())


def quantize_weights_f16(w):
    """Benchmark format: per 32 values an FP16 scale = max|g|/6 (IEEE division, RNE to FP16),
    nearest-even E2M1 codes against that scale."""
    _check_source(w, 32)
    n, k = w.shape
    blocks = w.reshape(n, k // 32, 32)
    amax = blocks.abs().amax(-1)
    scales = (amax / amax.new_tensor(6.0)).to(torch.float16)  # IEEE division
    tiny = torch.finfo(torch.float32).tiny
    codes = _e2m1_codes(blocks / scales.float().clamp_min(tiny).unsqueeze(-1)).reshape(n, k)
    return FP4F16Weights(_pack(codes), scales.contiguous())


def fused_linear(x, packed, scales, global_scale, threads=128, out=None, *, output_dtype=torch.float32):
    """out[M,N] = x[M,K] @ dequant(W).T with FP32 accumulation. global_scale
    None selects the FP16-per-32 scale format."""
    f16_format = global_scale is None
    tensors = (x, packed, scales) + (() if f16_format else (global_scale,))
    for tensor in tensors:
        if not isinstance(tensor, torch.Tensor) or tensor.device.type != "cuda" or tensor.device != x.device \
                or not tensor.is_contiguous():
            raise ValueError("All tensors must be contiguous on the current CUDA device")
        if tensor.requires_grad:
            raise ValueError("Inference only")
    if x.dtype not in _XDT or x.ndim != 2:
        raise ValueError("Expected FP16, FP32 or BF16 activations [M,K]")
    if packed.dtype != torch.uint8 or packed.ndim != 2:
        raise ValueError("Packed weights and FP8 scale bytes must be uint8")
    if output_dtype not in _ODT:
        raise ValueError("output_dtype must be torch.float32 or torch.bfloat16")
    m, k = x.shape
    n = packed.shape[0]
    group = 32 if f16_format else 16
    if f16_format:
        if scales.dtype != torch.float16:
            raise ValueError("FP16-per-32 scales must be float16")
    elif scales.dtype != torch.uint8:
        raise ValueError("Packed weights and FP8 scale bytes must be uint8")
    if min(m, n, k) <= 0 or k % group or packed.shape[1] != k // 2 or scales.shape != (n, k // group):
        raise ValueError(f"Invalid {group}-value block dimensions")
    if max(m * k, n * k, m * n) >= 2 ** 31:
        raise ValueError("Dimensions exceed signed 32-bit indexing")
    if not f16_format and (global_scale.dtype != torch.float32 or global_scale.numel() != 1):
        raise ValueError("Expected one FP32 global scale")
    if packed.data_ptr() % 4 or threads not in THREADS:
        raise ValueError("Packed weights require 4-byte alignment and supported block size")
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=output_dtype)
    else:
        if out.dtype != output_dtype or out.device != x.device or not out.is_contiguous() or out.requires_grad:
            raise ValueError("Only contiguous output tensors of the requested dtype are supported")
        if out.shape != (m, n):
            raise ValueError("Output shape mismatch")
    if any(out.untyped_storage().data_ptr() == v.untyped_storage().data_ptr() for v in tensors):
        raise ValueError("Output may not share input storage")
    get_module(x.device)
    wfmt = _native.W_FP4_G32H if f16_format else _native.W_FP4_G16E
    return _native.gemv(wfmt, _XDT[x.dtype], x, packed, scales, global_scale, out, _ODT[output_dtype], m, n, k)


@torch.library.custom_op("kernel_lab::fp4_linear", mutates_args=(), device_types="cuda")
def fp4_linear(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
               global_scale: torch.Tensor, threads: int = 128) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return fused_linear(x, packed, scales, global_scale, threads)


@fp4_linear.register_fake
def _fp4_fake(x, packed, scales, global_scale, threads=128):
    return torch.empty((x.shape[0], packed.shape[0]), device=x.device, dtype=torch.float32)
