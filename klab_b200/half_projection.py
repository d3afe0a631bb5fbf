"""FP16/BF16-input projection with FP32 output (drop-in for half_projection.py).

x[M,K] and w[N,K] share one 16-bit dtype; values are widened exactly and
accumulated in FP32 (half_projection.py:1-6). Runs the sm_100a streaming kernel.
"""

from __future__ import annotations

import torch

from . import _native
from ._module import get_module

SUFFIX = {torch.float16: "f16", torch.bfloat16: "bf16"}
THREADS = (32, 64, 128, 256)
VECTORS = (2, 8)


def kernel_names():
    """The reference's kernel name set (half_kernels.cu:63-80)."""
    return [f"half_warp_{s}_t{t}{'_v8' if v == 8 else ''}"
            for s in ("f16", "bf16") for v in VECTORS for t in THREADS]


def fused_linear(x, w, threads=32, out=None, vector=2):
    for tensor in (x, w):
        if not isinstance(tensor, torch.Tensor) or tensor.device.type != "cuda" or not tensor.is_contiguous() \
                or tensor.requires_grad:
            raise ValueError("Inference-only contiguous tensors on the current CUDA device required")
    if x.device != w.device:
        raise ValueError("Inference-only contiguous tensors on the current CUDA device required")
    if x.dtype not in SUFFIX or w.dtype != x.dtype:
        raise ValueError("x and w must both be FP16 or both BF16")
    if x.ndim != 2 or w.ndim != 2 or x.shape[1] != w.shape[1]:
        raise ValueError("Expected x=[M,K], w=[N,K]")
    m, k = x.shape
    n = w.shape[0]
    if min(m, n, k) <= 0 or m > 65535 or max(m * k, n * k, m * n) >= 2 ** 31:
        raise ValueError("Dimensions must be positive, M<=65535, and fit signed 32-bit indexing")
    if threads not in THREADS or vector not in VECTORS:
        raise ValueError("Unsupported launch configuration")
    align = 2 * vector
    if k % vector or x.data_ptr() % align or w.data_ptr() % align:
        raise ValueError(f"Require K divisible by {vector} and {align}-byte aligned inputs")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    else:
        if out.dtype != torch.float32 or out.device != x.device or not out.is_contiguous() or out.requires_grad:
            raise ValueError("Only contiguous FP32 tensors are supported")
        if tuple(out.shape) != (m, n):
            raise ValueError("Output shape mismatch")
        if any(out.untyped_storage().data_ptr() == t.untyped_storage().data_ptr() for t in (x, w)):
            raise ValueError("Output must not share storage with inputs")
    get_module(x.device)
    dt = _native.DT_BF16 if x.dtype == torch.bfloat16 else _native.DT_F16
    wfmt = _native.W_BF16 if x.dtype == torch.bfloat16 else _native.W_F16
    return _native.gemv(wfmt, dt, x, w, None, None, out, _native.DT_F32, m, n, k)


@torch.library.custom_op("kernel_lab::half_linear", mutates_args=(), device_types="cuda")
def linear(x: torch.Tensor, w: torch.Tensor, threads: int = 32, vector: int = 2) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return fused_linear(x, w, threads, vector=vector)


@linear.register_fake
def _linear_fake(x, w, threads=32, vector=2):
    if x.dtype not in SUFFIX or w.dtype != x.dtype or x.ndim != 2 or w.ndim != 2 or x.shape[1] != w.shape[1]:
        raise ValueError("Expected same-dtype FP16/BF16 x=[M,K], w=[N,K]")
    return x.new_empty((x.shape[0], w.shape[0]), dtype=torch.float32)
