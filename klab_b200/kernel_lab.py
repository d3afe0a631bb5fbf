"""FP32 projections behind the reference's KernelLab surface (kernel_lab.py).

KernelLab.matmul / warp_matmul / tiled_matmul / tiny_matmul keep their
signatures, validation and FP32 contract; on B200 all of them run the sm_100a
streaming kernel (FP32 weights and activations, FP32 accumulate and output),
so their launch-configuration arguments are validated hints. residual_rmsnorm
(kernel_lab.py:281-294) runs klab_residual_rmsnorm. The registered ops
kernel_lab::matmul, kernel_lab::warp_matmul and kernel_lab::residual_rmsnorm
keep their schemas.
"""

from __future__ import annotations

import torch

from . import _native
from ._module import get_module


class KernelLab:
    """Single-device FP32 projection handle with explicit close()."""

    def __init__(self):
        self.device = torch.cuda.current_device()
        self.module = get_module(self.device)
        self._closed = False

    def validate(self, *tensors):
        if self._closed:
            raise RuntimeError("Kernel module is closed")
        for tensor in tensors:
            if tensor.device != torch.device("cuda", self.device):
                raise ValueError("All tensors must be on this KernelLab's CUDA device")
            if tensor.dtype != torch.float32 or not tensor.is_contiguous():
                raise ValueError("Only contiguous FP32 tensors are supported")
            if tensor.requires_grad:
                raise ValueError("This experiment supports inference only")

    def output(self, out, shape, *inputs):
        if out is None:
            return torch.empty(shape, device=inputs[0].device, dtype=torch.float32)
        self.validate(out)
        if tuple(out.shape) != tuple(shape):
            raise ValueError("Output shape mismatch")
        if any(out.untyped_storage().data_ptr() == x.untyped_storage().data_ptr() for x in inputs):
            raise ValueError("Output must not share storage with inputs")
        return out

    def _shapes(self, x, w):
        self.validate(x, w)
        if x.ndim != 2 or w.ndim != 2 or x.shape[1] != w.shape[1]:
            raise ValueError("Expected x=[M,K], w=[N,K]")
        m, k = x.shape
        n = w.shape[0]
        if min(m, n, k) <= 0 or max(m * k, n * k, m * n) >= 2 ** 31:
            raise ValueError("Dimensions must be positive and fit signed 32-bit indexing")
        return m, n, k

    def _run(self, x, w, out):
        m, k = x.shape
        n = w.shape[0]
        return _native.gemv(_native.W_F32, _native.DT_F32, x, w, None, None, out, _native.DT_F32, m, n, k)

    def matmul(self, x, w, rows=4, threads=128, out=None, serial=False):
        """Compute x @ w.T, where x=[tokens,K] and w=[outputs,K] (kernel_lab.py:271-294)."""
        m, n, k = self._shapes(x, w)
        if rows not in (1, 2, 4, 8) or threads not in (64, 128, 256):
            raise ValueError("Unsupported launch configuration")
        if serial and m != 1:
            raise ValueError("Serial starting kernel supports one token")
        return self._run(x, w, self.output(out, (m, n), x, w))

    def warp_matmul(self, x, w, threads=128, vector=4, out=None):
        m, n, k = self._shapes(x, w)
        if threads not in (32, 64, 128, 256) or vector not in (1, 4):
            raise ValueError("Unsupported warp configuration")
        if vector == 4 and (k % 4 or x.data_ptr() % 16 or w.data_ptr() % 16):
            raise ValueError("Vector loads require K divisible by 4 and 16-byte aligned inputs")
        return self._run(x, w, self.output(out, (m, n), x, w))

    def tiled_matmul(self, x, w, tile="m32_n32", out=None):
        m, n, k = self._shapes(x, w)
        if tile not in ("m8_n32", "m16_n64", "m32_n32"):
            raise ValueError("Unsupported GEMM tile")
        return self._run(x, w, self.output(out, (m, n), x, w))

    def tiny_matmul(self, x, w, threads=32, vector=1, out=None):
        m, n, k = self._shapes(x, w)
        if k not in (64, 128, 256, 512, 1024):
            raise ValueError("Unsupported fixed-K shape or signed 32-bit indexing")
        if threads not in (32, 64, 128, 256) or vector not in (1, 4):
            raise ValueError("Unsupported fixed-K configuration")
        if vector == 4 and (x.data_ptr() % 16 or w.data_ptr() % 16):
            raise ValueError("Vector loads require 16-byte alignment")
        return self._run(x, w, self.output(out, (m, n), x, w))

    def residual_rmsnorm(self, x, residual, weight, eps=1e-6, threads=256, out=None):
        """((x + residual) * rsqrt(mean((x + residual)^2) + eps)) * weight per row, FP32
        (kernel_lab.py:281-294, kernels.cu:168-222); `threads` is a validated hint."""
        self.validate(x, residual, weight)
        if x.ndim != 2 or x.shape != residual.shape or weight.shape != (x.shape[1],):
            raise ValueError("Expected x/residual=[M,K], weight=[K]")
        m, k = x.shape
        if not (m > 0 and 0 < k <= 8192 and m * k < 2 ** 31 and eps > 0):
            raise ValueError("Require M>0, 1<=K<=8192, FP32 indexing, eps>0")
        if threads not in (128, 256):
            raise ValueError("threads must be 128 or 256")
        out = self.output(out, x.shape, x, residual, weight)
        stream = torch.cuda.current_stream(x.device)
        rc = _native.lib().klab_residual_rmsnorm(x.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                                                 out.data_ptr(), m, k, float(eps), stream.cuda_stream)
        _native.check(rc, "klab_residual_rmsnorm")
        _native.record(stream, x, residual, weight, out)
        return out

    def close(self):
        if not self._closed:
            torch.cuda.synchronize(self.device)
            self._closed = True


_modules: dict[int, KernelLab] = {}


def default_lab() -> KernelLab:
    device = torch.cuda.current_device()
    if device not in _modules or _modules[device]._closed:
        _modules[device] = KernelLab()
    return _modules[device]


@torch.library.custom_op("kernel_lab::matmul", mutates_args=(), device_types="cuda")
def matmul(x: torch.Tensor, w: torch.Tensor, rows: int = 4, threads: int = 128) -> torch.Tensor:
    with torch.cuda.device(x.device):
        lab = default_lab()
        if x.shape[0] > 1:
            return lab.tiled_matmul(x, w)
        return lab.matmul(x, w, rows=rows, threads=threads)


@matmul.register_fake
def _matmul_fake(x, w, rows=4, threads=128):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op("kernel_lab::warp_matmul", mutates_args=(), device_types="cuda")
def warp_matmul(x: torch.Tensor, w: torch.Tensor, threads: int = 128, vector: int = 4) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return default_lab().warp_matmul(x, w, threads, vector)


@warp_matmul.register_fake
def _warp_matmul_fake(x, w, threads=128, vector=4):
    return x.new_empty((x.shape[0], w.shape[0]))


@torch.library.custom_op("kernel_lab::residual_rmsnorm", mutates_args=(), device_types="cuda")
def residual_rmsnorm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6
) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return default_lab().residual_rmsnorm(x, residual, weight, eps=eps)


@residual_rmsnorm.register_fake
def _rmsnorm_fake(x, residual, weight, eps=1e-6):
    return torch.empty_like(x)
