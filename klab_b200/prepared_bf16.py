"""Prepared BF16 projections (drop-in for prepared_bf16.py).

PreparedBF16Projection validates and prepares once, before capture, and then
each call is one launch. The reference routes this object to the vendor matmul
until its custom kernels pass a held-out dispatch cohort (prepared_bf16.py:1-15,
64-100). Here the route is the B200 prepared plan (stream_gemv_kernel, parity
pinned bit for bit against the CPU oracle) unless a compressed-projection
report is supplied, in which case projection_policy's vendor decision is
honoured exactly as in the reference. vendor_callable / vendor_out_callable are
the reference's vendor bindings (torch.mm with the requested output dtype).
"""

from __future__ import annotations

import time
from functools import partial

import torch

from . import _native
from .prepared import PreparedPlan
from .projection_policy import compressed_vendor_fallback


def vendor_callable(w, output_dtype):
    """torch.mm over immutable BF16 weights with the requested output dtype."""
    if output_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("Expected BF16 or FP32 output")
    if not isinstance(w, torch.Tensor) or w.ndim != 2 or min(w.shape) <= 0 or w.dtype != torch.bfloat16 \
            or w.requires_grad:
        raise ValueError("Expected nonempty inference-only BF16 weights [N,K]")
    w_t = w.T
    if output_dtype == torch.bfloat16:
        return lambda x: torch.mm(x, w_t)
    return lambda x: torch.mm(x, w_t, out_dtype=torch.float32)


def vendor_out_callable(w, output_dtype):
    vendor_callable(w, output_dtype)
    return partial(_vendor_linear, w.T, output_dtype)


def _check_out(out, x, n, dtype):
    if not isinstance(out, torch.Tensor) or out.dtype != dtype or out.device != x.device or out.ndim != 2 \
            or tuple(out.shape) != (x.shape[0], n) or not out.is_contiguous() or out.requires_grad:
        raise RuntimeError("out must be a contiguous inference tensor of the expected dtype, device and shape")


def _vendor_linear(w_t, output_dtype, x, *, out=None):
    if out is not None:
        _check_out(out, x, w_t.shape[1], output_dtype)
        if torch._C._overlaps(out, x) or torch._C._overlaps(out, w_t):
            raise ValueError("out must not overlap the input or prepared weights")
    if output_dtype == torch.float32:
        return torch.mm(x, w_t, out_dtype=torch.float32, out=out)
    return torch.mm(x, w_t, out=out)


class PreparedBF16Projection:
    def __init__(self, w, tokens=1, profile=None, *, output_dtype=torch.float32):
        started = time.perf_counter()
        if not isinstance(w, torch.Tensor) or w.device.type != "cuda" or w.ndim != 2 or min(w.shape) <= 0 \
                or not w.is_contiguous() or w.requires_grad or w.dtype != torch.bfloat16:
            raise ValueError("Expected nonempty contiguous inference-only BF16 CUDA weights [N,K]")
        if isinstance(tokens, bool) or not isinstance(tokens, int) or tokens <= 0:
            raise ValueError("Expected a positive integer token count")
        if output_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("Expected BF16 or FP32 output")
        with torch.cuda.device(w.device):
            if torch.cuda.is_current_stream_capturing():
                raise ValueError("Prepare weights before CUDA graph capture")
            self.w = w
            self.dtype = w.dtype
            self.output_dtype = output_dtype
            self.precision_flags = {
                "allow_tf32": torch.backends.cuda.matmul.allow_tf32,
                "allow_bf16_reduced_precision_reduction":
                    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction}
            if any(self.precision_flags.values()):
                raise ValueError("Set allow_tf32 and allow_bf16_reduced_precision_reduction to False before "
                                 "preparing this FP32-accumulation contract")
            self.m, self.n, self.k = tokens, *w.shape
            self.shape_mnk = (tokens, *w.shape)
            name = "bf16" if output_dtype == torch.bfloat16 else "fp32"
            self.packed = None
            self.packing_seconds = 0.0
            if profile is not None:
                self.plan = compressed_vendor_fallback(profile, self.shape_mnk, name)
                self.strategy = self.plan["config"]
                self.linear = vendor_callable(w, output_dtype)
                self.linear_out = vendor_out_callable(w, output_dtype)
                self.native = None
            else:
                self.native = PreparedPlan(_native.W_BF16, torch.bfloat16, output_dtype, tokens, *w.shape, w.device)
                self.plan = {"backend": "custom", "config": "b200_stream_gemv",
                             "reason": "B200 prepared plan; parity pinned against the CPU oracle",
                             "requires_packing": False, "custom_win_validated": False,
                             "accepted_10pct_target": False, "dispatch_overhead_validated": False,
                             "launch": self.native.info}
                self.strategy = self.plan["config"]
                self.linear = self._native_linear
                self.linear_out = self._native_linear_out
            warmup = torch.zeros((tokens, self.k), device=w.device, dtype=w.dtype)
            self.linear(warmup)
        self.setup_seconds = time.perf_counter() - started

    def _native_linear(self, x):
        return self.native.launch(x, self.w)

    def _native_linear_out(self, x, *, out):
        _check_out(out, x, self.n, self.output_dtype)
        if torch._C._overlaps(out, x) or torch._C._overlaps(out, self.w):
            raise ValueError("out must not overlap the input or prepared weights")
        return self.native.launch(x, self.w, out=out)

    def __call__(self, x, out=None):
        return self.linear(x) if out is None else self.linear_out(x, out=out)
