"""Decode-step elementwise ops around the projections, and their fusion into the
next projection's x staging.

add_rmsnorm(res, y, w) and silu_mul(gu) keep the reference's signatures, BF16
contract and arithmetic (research/l2-prefetch/src/decode_attn.py:64-81 over
decode_attn.cu:471-527): x = RNE(res + y), xn = RNE(x * rsqrt(mean(x^2) + eps) * w)
summed in the reference kernel's order; silu_mul = RNE(g / (1 + exp(-g)) * u).
They accept any even width (the reference's kernel stops at 2048).

add_rmsnorm_linear and silu_mul_linear compute the same x inside the BF16
projection kernel while it stages x, so they return exactly what the
standalone op followed by compressed_bf16.raw_linear returns, without the
intermediate tensor and its launch.
"""

from __future__ import annotations

import torch

from . import _native
from ._module import get_module


def _check_bf16(*tensors):
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda" or t.dtype != torch.bfloat16:
            raise ValueError("Expected BF16 CUDA tensors")
        if not t.is_contiguous():
            raise ValueError("Expected contiguous tensors")
        if t.device != tensors[0].device:
            raise ValueError("All tensors must be on one device")


def add_rmsnorm(res, y, w, eps=1e-6):
    """Returns (x, xn) with x = res + y and xn = rms_norm(x) * w, both BF16 [M, d]."""
    _check_bf16(res, y, w)
    if res.ndim != 2 or y.shape != res.shape or w.shape != (res.shape[1],):
        raise ValueError("Unsupported add_rmsnorm shape")
    m, d = res.shape
    if d % 2 or m <= 0 or d <= 0 or not eps > 0:
        raise ValueError("Unsupported add_rmsnorm shape")
    get_module(res.device)
    x, xn = torch.empty_like(res), torch.empty_like(res)
    stream = torch.cuda.current_stream(res.device)
    with torch.cuda.device(res.device):
        rc = _native.lib().klab_add_rmsnorm(res.data_ptr(), y.data_ptr(), w.data_ptr(), x.data_ptr(), xn.data_ptr(),
                                            m, d, float(eps), stream.cuda_stream)
    _native.check(rc, "klab_add_rmsnorm")
    _native.record(stream, res, y, w, x, xn)
    return x, xn


def silu_mul(gu):
    """gu [M, 2*inter] BF16 -> silu(gate) * up [M, inter]."""
    _check_bf16(gu)
    if gu.ndim != 2 or gu.shape[1] % 4:
        raise ValueError("Unsupported silu_mul shape")
    m, two = gu.shape
    inter = two // 2
    get_module(gu.device)
    out = torch.empty(m, inter, device=gu.device, dtype=gu.dtype)
    stream = torch.cuda.current_stream(gu.device)
    with torch.cuda.device(gu.device):
        rc = _native.lib().klab_silu_mul(gu.data_ptr(), out.data_ptr(), m, inter, stream.cuda_stream)
    _native.check(rc, "klab_silu_mul")
    _native.record(stream, gu, out)
    return out


def _overlap(a, b):
    """True when two tensors' storage byte ranges intersect."""
    pa, pb = a.data_ptr(), b.data_ptr()
    return pa < pb + b.numel() * b.element_size() and pb < pa + a.numel() * a.element_size()


def _projection_out(out, m, n, like):
    if out is None:
        return torch.empty((m, n), device=like.device, dtype=torch.bfloat16)
    _check_bf16(out)
    if tuple(out.shape) != (m, n):
        raise ValueError("Output shape mismatch")
    return out


def add_rmsnorm_linear(res, y, norm_weight, w, eps=1e-6, out=None, x_out=None):
    """(x, out) with x = res + y and out = (rms_norm(x) * norm_weight) @ w.T in one launch;
    w BF16 [N, K]; K % 8 == 0. x_out=False skips writing x."""
    _check_bf16(res, y, norm_weight, w)
    if res.ndim != 2 or y.shape != res.shape or norm_weight.shape != (res.shape[1],) or w.ndim != 2 \
            or w.shape[1] != res.shape[1]:
        raise ValueError("Expected res/y=[M,K], norm_weight=[K], w=[N,K]")
    m, k = res.shape
    n = w.shape[0]
    if k % 8 or not eps > 0:
        raise ValueError("K must be a multiple of 8 and eps positive")
    get_module(res.device)
    out = _projection_out(out, m, n, res)
    if x_out is None:
        x_out = torch.empty_like(res)
    elif x_out is not False:
        _check_bf16(x_out)
        if x_out.shape != res.shape:
            raise ValueError("x_out shape mismatch")
    # Every CTA re-reads res and y while it stages x and one column of CTAs writes x_out, so an
    # in-place residual update (x_out aliasing res or y) would feed updated values to later CTAs.
    written = [out] + ([] if x_out is False else [x_out])
    for dst in written:
        if any(_overlap(dst, src) for src in (res, y, norm_weight)):
            raise ValueError("x_out and out must not overlap res, y or norm_weight")
    if x_out is not False and _overlap(x_out, out):
        raise ValueError("x_out and out must not overlap")
    stream = torch.cuda.current_stream(res.device)
    ws_ptr, ws_bytes = _native.workspace_for(_native.W_BF16, m, n, k, res.device.index, stream)
    with torch.cuda.device(res.device):
        rc = _native.lib().klab_add_rmsnorm_linear(res.data_ptr(), y.data_ptr(), norm_weight.data_ptr(), float(eps),
                                                   w.data_ptr(), out.data_ptr(),
                                                   None if x_out is False else x_out.data_ptr(), m, n, k, ws_ptr,
                                                   ws_bytes, stream.cuda_stream)
    _native.check(rc, "klab_add_rmsnorm_linear")
    _native.record(stream, res, y, norm_weight, w, out, None if x_out is False else x_out)
    return (None if x_out is False else x_out), out


def silu_mul_linear(gu, w, out=None):
    """silu_mul(gu) @ w.T in one launch; gu BF16 [M, 2*inter], w BF16 [N, inter], inter % 8 == 0."""
    _check_bf16(gu, w)
    if gu.ndim != 2 or w.ndim != 2 or gu.shape[1] != 2 * w.shape[1]:
        raise ValueError("Expected gu=[M,2*inter], w=[N,inter]")
    m = gu.shape[0]
    n, inter = w.shape
    if inter % 8:
        raise ValueError("inter must be a multiple of 8")
    get_module(gu.device)
    out = _projection_out(out, m, n, gu)
    if _overlap(out, gu):
        raise ValueError("out must not overlap gu")
    stream = torch.cuda.current_stream(gu.device)
    ws_ptr, ws_bytes = _native.workspace_for(_native.W_BF16, m, n, inter, gu.device.index, stream)
    with torch.cuda.device(gu.device):
        rc = _native.lib().klab_silu_mul_linear(gu.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, inter, ws_ptr,
                                                ws_bytes, stream.cuda_stream)
    _native.check(rc, "klab_silu_mul_linear")
    _native.record(stream, gu, w, out)
    return out
