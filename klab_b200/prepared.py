"""Prepared projection plans over the native plan ABI (klab_plan_*).

A plan validates one (weight format, x dtype, output dtype, M, N, K) case once,
outside CUDA graph capture, and freezes its launch (token tile, x staging, grid,
split-K and the split-K workspace, which the plan owns). Launching binds only
the x / weight / side-data / output pointers, so the host cost per call is one
ctypes call and one kernel launch. The reference's equivalent is the native
plan registry of native/prepared.cpp:155-413 with the Python candidates of
native_prepared.py:398-565 and prepared_kernels.py:178-320.
"""

from __future__ import annotations

import json
import threading

import torch

from . import _native
from ._module import get_module

_DT = {torch.bfloat16: _native.DT_BF16, torch.float16: _native.DT_F16, torch.float32: _native.DT_F32}
_OUT = {"bf16": torch.bfloat16, "fp32": torch.float32}


def output_name(value):
    """'bf16' | 'fp32' from a dtype or a name (prepared_kernels.py _output_name)."""
    for name, dtype in _OUT.items():
        if value is dtype or (isinstance(value, str) and value == name):
            return name
    raise ValueError("output_dtype must be 'bf16'/torch.bfloat16 or 'fp32'/torch.float32")


class PreparedPlan:
    """One frozen launch on one device. Keep it alive for every CUDA graph that
    captured its launches; launches of one plan must not overlap on the GPU."""

    def __init__(self, wfmt, x_dtype, output_dtype, m, n, k, device):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("Prepared plans are bound to a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if x_dtype not in _DT:
            raise ValueError("x dtype must be BF16, FP16 or FP32")
        self.wfmt, self.x_dtype = wfmt, x_dtype
        self.output_dtype = _OUT[output_name(output_dtype)]
        self.m, self.n, self.k = m, n, k
        with torch.cuda.device(self.device):
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Prepare plans before CUDA graph capture")
            get_module(self.device)
            self.handle = _native.plan_create(wfmt, _DT[x_dtype], _DT[self.output_dtype], m, n, k)
        self.info = json.loads(_native.plan_info(self.handle))
        self._lock = threading.Lock()

    def launch(self, x, w, aux=None, aux2=None, gscale=None, out=None):
        """out[M, N] (allocated when None) on torch's current stream of x's device."""
        if self.handle is None:
            raise RuntimeError("Plan was retired")
        if x.device != self.device or x.dtype != self.x_dtype or tuple(x.shape) != (self.m, self.k) \
                or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous {self.x_dtype} [{self.m},{self.k}] tensor on {self.device}")
        if out is None:
            out = torch.empty((self.m, self.n), dtype=self.output_dtype, device=self.device)
        elif out.dtype != self.output_dtype or tuple(out.shape) != (self.m, self.n) or not out.is_contiguous() \
                or out.device != self.device:
            raise ValueError("out must be a contiguous tensor of the prepared output dtype and shape")
        stream = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            _native.plan_launch(self.handle, x, w, aux, aux2, gscale, out, stream)
        _native.record(stream, x, w, aux, aux2, gscale, out)
        return out

    def close(self):
        with self._lock:
            if self.handle is not None:
                torch.cuda.synchronize(self.device)
                _native.plan_destroy(self.handle)
                self.handle = None

    def __del__(self):
        try:
            if getattr(self, "handle", None) is not None and not torch.cuda.is_current_stream_capturing():
                _native.plan_destroy(self.handle)
        except Exception:  # interpreter shutdown
            pass
