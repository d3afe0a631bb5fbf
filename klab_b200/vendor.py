"""Vendor-library projections on the caller's tensors and stream: the baselines the
reference's dynamic_vendor operator routes to (dynamic_projection.py:21-46 over
cublas_baseline.py), kept for its operator surface and for the benchmark's vendor
columns. Not the product path.

`vendor_call(x, w, config, out=None)` computes out[M, N] = x . W^T (FP32 output) with
`config` one of the reference's names:

  torch_mm, torch_mv, torch_mm_out_fp32      torch.mm / torch.mv (cuBLAS through torch)
  cublas_mm, cublas_mv                       cublasSgemm / cublasSgemv, FP32, W [N, K]
  cublas_packed_mm, cublas_packed_mv         the same on W^T stored [K, N] ("packed")
  cublas_compute32, cublas_packed_compute32  cublasGemmEx with x, W in their 16-bit type
                                             (or FP32), CUBLAS_COMPUTE_32F, FP32 output

cuBLAS computes column-major: out^T[N, M] = op(A) . x^T with A = W viewed column-major
[K, N] (op = T) or W^T stored [K, N] viewed column-major [N, K] (op = N).
"""

from __future__ import annotations

import ctypes as ct
import threading
from pathlib import Path

import torch

CONFIGS = ("torch_mm", "torch_mv", "torch_mm_out_fp32", "cublas_mm", "cublas_mv", "cublas_packed_mm",
           "cublas_packed_mv", "cublas_compute32", "cublas_packed_compute32")
_OP_N, _OP_T = 0, 1
_R_32F, _R_16F, _R_16BF = 0, 2, 14
_COMPUTE_32F = 68
_TYPE = {torch.float32: _R_32F, torch.float16: _R_16F, torch.bfloat16: _R_16BF}


def _load(name):
    import nvidia.cublas

    base = Path(next(iter(nvidia.cublas.__path__))) / "lib"
    return ct.CDLL(str(base / name))


class Blas:
    """One cuBLAS handle on one device; every call runs on torch's current stream."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.lib = lib = _load("libcublas.so.12")
        P, I = ct.c_void_p, ct.c_int
        lib.cublasCreate_v2.argtypes = [ct.POINTER(P)]
        lib.cublasDestroy_v2.argtypes = [P]
        lib.cublasSetStream_v2.argtypes = [P, P]
        lib.cublasSetMathMode.argtypes = [P, I]
        lib.cublasSgemm_v2.argtypes = [P, I, I, I, I, I, P, P, I, P, I, P, P, I]
        lib.cublasSgemv_v2.argtypes = [P, I, I, I, P, P, I, P, I, P, P, I]
        lib.cublasGemmEx.argtypes = [P, I, I, I, I, I, P, P, I, I, P, I, I, P, P, I, I, I, I]
        self.handle = P()
        with torch.cuda.device(self.device):
            self._ok(lib.cublasCreate_v2(ct.byref(self.handle)), "cublasCreate")
        self._ok(lib.cublasSetMathMode(self.handle, 0), "cublasSetMathMode")   # default math, no TF32
        self.one, self.zero = ct.c_float(1.0), ct.c_float(0.0)

    @staticmethod
    def _ok(status, what):
        if status:
            raise RuntimeError(f"{what} failed with cuBLAS status {status}")

    def _stream(self):
        self._ok(self.lib.cublasSetStream_v2(self.handle, ct.c_void_p(torch.cuda.current_stream(self.device)
                                                                      .cuda_stream)), "cublasSetStream")

    def gemm(self, x, w, out, packed, compute32=False):
        """out = x . W^T; W [N, K] (packed: W^T [K, N]). FP32 Sgemm, or GemmEx with
        x/W in their own type and FP32 compute and output (compute32)."""
        m, k = x.shape
        n = w.shape[1] if packed else w.shape[0]
        op, lda = (_OP_N, n) if packed else (_OP_T, k)
        self._stream()
        args = (self.handle, op, _OP_N, n, m, k, ct.byref(self.one), ct.c_void_p(w.data_ptr()))
        if compute32 or x.dtype != torch.float32:
            self._ok(self.lib.cublasGemmEx(*args, _TYPE[w.dtype], lda, ct.c_void_p(x.data_ptr()), _TYPE[x.dtype], k,
                                           ct.byref(self.zero), ct.c_void_p(out.data_ptr()), _R_32F, n,
                                           _COMPUTE_32F, -1), "cublasGemmEx")
        else:
            self._ok(self.lib.cublasSgemm_v2(*args, lda, ct.c_void_p(x.data_ptr()), k, ct.byref(self.zero),
                                             ct.c_void_p(out.data_ptr()), n), "cublasSgemm")
        return out

    def gemv(self, x, w, out, packed):
        """out[1, N] = x[1, K] . W^T in FP32 (packed: W^T [K, N])."""
        if x.shape[0] != 1:
            raise ValueError("GEMV requires one input vector")
        k = x.shape[1]
        n = w.shape[1] if packed else w.shape[0]
        self._stream()
        if packed:   # W^T [K, N] is column-major [N, K]: y = A . x
            dims = (_OP_N, n, k, ct.byref(self.one), ct.c_void_p(w.data_ptr()), n)
        else:        # W [N, K] is column-major [K, N]: y = A^T . x
            dims = (_OP_T, k, n, ct.byref(self.one), ct.c_void_p(w.data_ptr()), k)
        self._ok(self.lib.cublasSgemv_v2(self.handle, *dims, ct.c_void_p(x.data_ptr()), 1, ct.byref(self.zero),
                                         ct.c_void_p(out.data_ptr()), 1), "cublasSgemv")
        return out

    def close(self):
        if self.handle:
            torch.cuda.synchronize(self.device)
            self._ok(self.lib.cublasDestroy_v2(self.handle), "cublasDestroy")
            self.handle = ct.c_void_p()


_blas = {}
_lock = threading.Lock()


def blas(device) -> Blas:
    index = torch.device(device).index
    with _lock:
        if index not in _blas:
            _blas[index] = Blas(torch.device("cuda", index))
        return _blas[index]


def vendor_call(x, w, config, out=None):
    """out[M, N] (FP32) = x . W^T by the vendor route `config` (see the module docstring);
    validation and errors as the reference's vendor_call."""
    if config not in CONFIGS:
        raise ValueError(f"config must be one of {CONFIGS}")
    for t in (x, w):
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda" or not t.is_contiguous() or t.requires_grad:
            raise ValueError("Inference-only contiguous same-device tensors required")
    if x.device != w.device:
        raise ValueError("Inference-only contiguous same-device tensors required")
    if x.dtype != w.dtype or x.dtype not in _TYPE:
        raise ValueError("Projection input dtypes differ or are unsupported")
    packed = "packed" in config
    if x.ndim != 2 or w.ndim != 2 or x.shape[1] != (w.shape[0] if packed else w.shape[1]):
        raise ValueError("Projection dimensions differ")
    n = w.shape[1] if packed else w.shape[0]
    shape = (x.shape[0], n)
    if out is None:
        out = torch.empty(shape, device=x.device, dtype=torch.float32)
    elif out.device != x.device or out.dtype != torch.float32 or not out.is_contiguous() or tuple(out.shape) != shape:
        raise ValueError("Output must be a contiguous FP32 CUDA tensor of shape [M, N]")
    elif any(out.untyped_storage().data_ptr() == t.untyped_storage().data_ptr() for t in (x, w)):
        raise ValueError("Output must not share storage with inputs")
    with torch.cuda.device(x.device):
        if config in ("torch_mm", "torch_mm_out_fp32"):
            if x.dtype == torch.float32:
                return torch.mm(x, w.T, out=out)
            return torch.mm(x, w.T, out_dtype=torch.float32, out=out)
        if config == "torch_mv":
            if x.shape[0] != 1:
                raise ValueError("GEMV requires one input vector")
            if x.dtype == torch.float32:
                return torch.mv(w, x[0], out=out[0]).view(1, n)
            out.copy_(torch.mm(x, w.T, out_dtype=torch.float32))
            return out
        b = blas(x.device)
        if config.endswith("compute32"):
            return b.gemm(x, w, out, packed, compute32=True)
        if x.dtype != torch.float32:
            raise ValueError(f"{config} takes FP32 tensors")
        if config.endswith("_mv"):
            return b.gemv(x, w, out, packed)
        return b.gemm(x, w, out, packed)
