"""Fused multi-output projections: several weight matrices that read the same x
in one launch (drop-in for examples/kv_pair_projection.py:13-36).

prepare_pair_graph(wk, wv) keeps the reference's validation, call signature and
FP32 joint output with K and V views, but instead of concatenating the weights
and calling torch.mm it runs the B200 streaming kernel over both matrices in
one launch (two segments: no concatenated copy, one x staging, one stream of
both weights). Each output element is bit-identical to the same weight
projected alone. prepare_fused_projection generalizes to any number of BF16
matrices sharing K (QKV, gate/up), with FP32 or BF16 output.
"""

from __future__ import annotations

import torch

from . import _native
from ._module import get_module

_OUT = {torch.float32: _native.DT_F32, torch.bfloat16: _native.DT_BF16}


def prepare_fused_projection(weights, out_dtype=torch.float32):
    """Prepare once; return fn(x [M, K], out [M, sum N_i]) -> views of out per weight."""
    if not weights or len(weights) > 8:
        raise ValueError("Expected one to eight weight matrices")
    w0 = weights[0]
    for w in weights:
        if (w.device.type != "cuda" or w.device != w0.device or w.dtype != torch.bfloat16 or w.ndim != 2
                or w.shape[1] != w0.shape[1] or not w.is_contiguous() or w.requires_grad):
            raise ValueError("Require contiguous inference BF16 CUDA weights sharing K")
    if out_dtype not in _OUT:
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    if torch.cuda.is_current_stream_capturing():
        raise ValueError("Prepare before graph capture")
    get_module(w0.device)
    width = w0.shape[1]
    rows = [w.shape[0] for w in weights]
    n = sum(rows)
    starts = [sum(rows[:i]) for i in range(len(rows))]

    def fused(x, out):
        m = x.shape[0] if x.ndim == 2 else 0
        if (x.ndim != 2 or x.shape[1] != width or m < 1 or x.device != w0.device or x.dtype != torch.bfloat16
                or not x.is_contiguous() or x.requires_grad):
            raise ValueError("Require a contiguous BF16 input [M, K] on the prepared device")
        if (tuple(out.shape) != (m, n) or out.device != x.device or out.dtype != out_dtype
                or not out.is_contiguous() or out.requires_grad):
            raise ValueError("Require a contiguous joint output [M, sum N] of the prepared dtype")
        if torch._C._overlaps(out, x) or any(torch._C._overlaps(out, w) for w in weights):
            raise ValueError("Output must not overlap input or prepared weights")
        segments = [(w, None, out[:, s:], n, r) for w, s, r in zip(weights, starts, rows)]
        _native.gemv_multi(_native.W_BF16, _native.DT_BF16, x, segments, None, _OUT[out_dtype], m, width)
        return tuple(out[:, s:s + r] for s, r in zip(starts, rows))

    return fused


def prepare_pair_graph(wk, wv):
    """Prepare once; return graph callable(x, joint_out)->(k_view, v_view)."""
    if (wk.device.type != "cuda" or wv.device != wk.device or wk.dtype != torch.bfloat16
            or wv.dtype != wk.dtype or wk.ndim != 2 or wv.ndim != 2 or wk.shape[1] != wv.shape[1]
            or not wk.is_contiguous() or not wv.is_contiguous() or wk.requires_grad or wv.requires_grad):
        raise ValueError("Require original contiguous inference BF16 CUDA K/V weights")
    if torch.backends.cuda.matmul.allow_tf32 or torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction:
        raise ValueError("Disable TF32 and BF16 reduced-precision reductions for this contract")
    if torch.cuda.is_current_stream_capturing():
        raise ValueError("Prepare concatenated weights before graph capture")
    fused = prepare_fused_projection([wk, wv], torch.float32)
    width, n = wk.shape[1], wk.shape[0] + wv.shape[0]

    def pair_graph(x, out):
        if (tuple(x.shape) != (1, width) or x.device != wk.device or x.dtype != wk.dtype
                or tuple(out.shape) != (1, n) or out.device != x.device or out.dtype != torch.float32
                or not out.is_contiguous() or x.requires_grad or out.requires_grad):
            raise ValueError("Require M1 input and contiguous FP32 joint output on the prepared device")
        return fused(x, out)

    return pair_graph
