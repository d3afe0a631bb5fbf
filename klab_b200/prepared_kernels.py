"""Prepared raw / coded BF16 projections as registered ops (drop-in for
prepared_kernels.py).

prepared_bf16::raw_r2 and prepared_bf16::coded_r2 keep the reference's schemas
(prepared_kernels.py:128-173): the prepared M, N, K and the launch hints
(threads, vector, validated but not used: the B200 launch is planned from the
case) are arguments, output allocation is the op's. Each op launches the
device's prepared plan for that case; plans are created by a candidate or by
preload_modules(...) + the first eager call, never during graph capture. Fake
kernels check the logical contract only, on CPU FakeTensors.
RawCandidate / CodedCandidate are device-bound prepared objects
(prepared_kernels.py:178-320).
"""

from __future__ import annotations

import threading
import time

import torch

from . import _native
from .prepared import PreparedPlan, output_name

_THREADS = (32, 64, 128, 256)
_VECTORS = (2, 8)
_MAX_M = 65535
_INDEX_LIMIT = 2 ** 31
_BLOCK, _CODED_BYTES, _RAW_BYTES = 64, 96, 128
_OUTPUTS = {"bf16": torch.bfloat16, "fp32": torch.float32}

_PLANS = {}          # (device, kind, m, n, k, output) -> PreparedPlan
_PLANS_LOCK = threading.Lock()
_PRELOADED = set()   # device indices


def _check_plan(m, n, k, threads, vector, coded):
    if any(isinstance(v, bool) or not isinstance(v, int) for v in (m, n, k, threads, vector)):
        raise ValueError("M, N, K, threads and vector must be integers")
    if threads not in _THREADS or vector not in _VECTORS:
        raise ValueError(f"Unsupported launch configuration; threads in {_THREADS}, vector in {_VECTORS}")
    if min(m, n, k) <= 0 or m > _MAX_M or max(m * k, n * k, m * n) >= _INDEX_LIMIT:
        raise ValueError(f"Dimensions must be positive, M<={_MAX_M}, and fit signed 32-bit indexing")
    if k % vector:
        raise ValueError(f"Require K divisible by {vector}")
    if coded and k % _BLOCK:
        raise ValueError(f"Coded projections require K divisible by {_BLOCK}")


def _check_operand(tensor, label, dtype, ndim, shape=None):
    if not isinstance(tensor, torch.Tensor) or tensor.dtype != dtype or tensor.ndim != ndim:
        raise ValueError(f"{label} must be a {ndim}-D {dtype} tensor")
    if not tensor.is_contiguous() or tensor.requires_grad:
        raise ValueError(f"{label} must be contiguous and inference-only (no requires_grad)")
    if shape is not None and tuple(tensor.shape) != shape:
        raise ValueError(f"{label} must have the prepared shape {list(shape)}")


def _check_coded_buffers(payload, metadata, n, k):
    blocks = n * (k // _BLOCK)
    if metadata.numel() != blocks or not _CODED_BYTES * blocks <= payload.numel() <= _RAW_BYTES * blocks:
        raise ValueError("Packed buffers do not match N,K")


def preload_modules(device):
    """Load this device's kernels outside capture (plans are then created on first use)."""
    from . import compressed_bf16 as cb

    index = cb._device_index(device)
    with torch.cuda.device(index):
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Preload modules before CUDA graph capture")
        module = cb.get_module(index)
    _PRELOADED.add(index)
    return (module, module)


def plan_for(device, kind, m, n, k, output):
    """The prepared plan of a case on a device (created outside capture only)."""
    index = device.index if isinstance(device, torch.device) else int(device)
    key = (index, kind, m, n, k, output)
    with _PLANS_LOCK:
        plan = _PLANS.get(key)
        if plan is not None and plan.handle is not None:
            return plan
        if index not in _PRELOADED:
            raise RuntimeError("Prepare a candidate or call preload_modules on this device outside capture first")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Prepare a candidate on this device outside capture first")
        wfmt = _native.W_CBF16 if kind == "coded" else _native.W_BF16
        plan = PreparedPlan(wfmt, torch.bfloat16, _OUTPUTS[output], m, n, k, torch.device("cuda", index))
        _PLANS[key] = plan
        return plan


def _retained(x, m, k):
    if not isinstance(x, torch.Tensor) or x.device.type != "cuda":
        raise ValueError("x must be a CUDA tensor")
    if x.ndim != 2 or tuple(x.shape) != (m, k):
        raise ValueError(f"x must have the prepared shape [M,K]=[{m},{k}]")


# ---------------------------------------------------------------- operators


@torch.library.custom_op("prepared_bf16::coded_r2", mutates_args=(), device_types="cuda")
def coded_r2(x: torch.Tensor, payload: torch.Tensor, metadata: torch.Tensor, m: int, n: int, k: int,
             threads: int, vector: int, output_dtype: str) -> torch.Tensor:
    output = output_name(output_dtype)
    _check_plan(m, n, k, threads, vector, coded=True)
    _retained(x, m, k)
    _check_operand(x, "x", torch.bfloat16, 2, (m, k))
    _check_operand(payload, "payload", torch.uint8, 1)
    _check_operand(metadata, "metadata", torch.int32, 1)
    if payload.device != x.device or metadata.device != x.device:
        raise ValueError("x, payload and metadata must share a device")
    _check_coded_buffers(payload, metadata, n, k)
    return plan_for(x.device, "coded", m, n, k, output).launch(x, payload, metadata)


@coded_r2.register_fake
def _coded_r2_fake(x, payload, metadata, m, n, k, threads, vector, output_dtype):
    dtype = _OUTPUTS[output_name(output_dtype)]
    _check_plan(m, n, k, threads, vector, coded=True)
    _check_operand(x, "x", torch.bfloat16, 2, (m, k))
    _check_operand(payload, "payload", torch.uint8, 1)
    _check_operand(metadata, "metadata", torch.int32, 1)
    if payload.device != x.device or metadata.device != x.device:
        raise ValueError("x, payload and metadata must share a device")
    _check_coded_buffers(payload, metadata, n, k)
    return x.new_empty((m, n), dtype=dtype)


@torch.library.custom_op("prepared_bf16::raw_r2", mutates_args=(), device_types="cuda")
def raw_r2(x: torch.Tensor, w: torch.Tensor, m: int, n: int, k: int, threads: int, vector: int,
           output_dtype: str) -> torch.Tensor:
    output = output_name(output_dtype)
    _check_plan(m, n, k, threads, vector, coded=False)
    _retained(x, m, k)
    _check_operand(x, "x", torch.bfloat16, 2, (m, k))
    if tuple(w.shape) != (n, k):
        raise ValueError(f"w must have the prepared shape [N,K]=[{n},{k}]")
    _check_operand(w, "w", torch.bfloat16, 2, (n, k))
    if w.device != x.device:
        raise ValueError("x and w must share a device")
    return plan_for(x.device, "raw", m, n, k, output).launch(x, w)


@raw_r2.register_fake
def _raw_r2_fake(x, w, m, n, k, threads, vector, output_dtype):
    dtype = _OUTPUTS[output_name(output_dtype)]
    _check_plan(m, n, k, threads, vector, coded=False)
    _check_operand(x, "x", torch.bfloat16, 2, (m, k))
    _check_operand(w, "w", torch.bfloat16, 2, (n, k))
    if w.device != x.device:
        raise ValueError("x and w must share a device")
    return x.new_empty((m, n), dtype=dtype)


_CODED_OP = torch.ops.prepared_bf16.coded_r2.default
_RAW_OP = torch.ops.prepared_bf16.raw_r2.default


# ---------------------------------------------------------------- candidates


class _Candidate(torch.nn.Module):
    """Shared preparation of one device-bound (M, N, K, output) case."""

    custom_win_validated = False  # a benchmark candidate, not a policy decision

    def _contract(self, kind, tokens, n, k, threads, vector, output_dtype):
        self.output_dtype = output_name(output_dtype)
        _check_plan(tokens, n, k, threads, vector, coded=kind == "coded")
        self.kind = kind
        self.m, self.n, self.k = tokens, n, k
        self.shape_mnk = (tokens, n, k)
        self.threads, self.vector = threads, vector

    def _bind(self, device):
        with torch.cuda.device(device):
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Prepare candidates before CUDA graph capture")
            self.precision_flags = {
                "allow_tf32": torch.backends.cuda.matmul.allow_tf32,
                "allow_bf16_reduced_precision_reduction":
                    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction}
            if any(self.precision_flags.values()):
                raise ValueError("Set allow_tf32 and allow_bf16_reduced_precision_reduction to False "
                                 "before preparing this FP32-accumulation contract")
            self._kernel_modules = preload_modules(device)
            self._plan = plan_for(device, self.kind, self.m, self.n, self.k, self.output_dtype)
        self.device = device
        return self._kernel_modules

    def _finish(self, started):
        from . import mtile_bf16 as mt

        self.config = {"revision": mt.REVISION, "threads": self.threads, "vector": self.vector,
                       "tile": self._plan.info["tile"], "launch": dict(self._plan.info),
                       "route": "B200 prepared plan (stream_gemv_kernel)"}
        with torch.cuda.device(self.device):
            self.implementation = mt.implementation_fingerprint(self.device)
            self.linear(torch.zeros((self.m, self.k), dtype=torch.bfloat16, device=self.device))
        self.setup_seconds = time.perf_counter() - started

    def _apply(self, fn, recurse=True):
        raise RuntimeError(f"{type(self).__name__} is a device-bound prepared plan; "
                           "reprepare it instead of moving or casting it")

    def forward(self, x):
        return self.linear(x)

    def describe(self):
        return {"kind": self.kind, "shape_mnk": list(self.shape_mnk), "config": dict(self.config),
                "output_dtype": self.output_dtype, "storage": dict(self.storage),
                "provenance": dict(self.provenance), "precision_flags": dict(self.precision_flags),
                "device": str(self.device), "setup_seconds": self.setup_seconds,
                "custom_win_validated": self.custom_win_validated}


class CodedCandidate(_Candidate):
    """Coded BF16 over a compressed_bf16.upload() result."""

    def __init__(self, packed, tokens=1, *, threads, vector, output_dtype):
        super().__init__()
        started = time.perf_counter()
        from . import compressed_bf16 as cb

        if not isinstance(packed, cb.PackedBF16):
            raise ValueError("packed must come from compressed_bf16.upload()")
        payload, metadata = packed.payload, packed.metadata
        for t, label, dtype in ((payload, "payload", torch.uint8), (metadata, "metadata", torch.int32)):
            if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
                raise ValueError(f"{label} must be a CUDA tensor")
            _check_operand(t, label, dtype, 1)
        if metadata.device != payload.device:
            raise ValueError("payload and metadata must share a device")
        if packed.format_version != cb.FORMAT_VERSION:
            raise ValueError(f"Unsupported packed format version; expected {cb.FORMAT_VERSION}")
        self._contract("coded", tokens, packed.n, packed.k, threads, vector, output_dtype)
        _check_coded_buffers(payload, metadata, self.n, self.k)
        self._bind(payload.device)
        self.register_buffer("payload", payload, persistent=False)
        self.register_buffer("metadata", metadata, persistent=False)
        self._packed = packed
        self.storage = {"format": f"compressed_bf16_v{packed.format_version}", "bytes": packed.storage_bytes,
                        "raw_bf16_bytes": 2 * self.n * self.k}
        self.provenance = {"source_sha256": packed.source_sha256, "format_version": packed.format_version}
        self._finish(started)

    def linear(self, x):
        return _CODED_OP(x, self.payload, self.metadata, self.m, self.n, self.k, self.threads, self.vector,
                         self.output_dtype)

    def linear_out(self, x, *, out):
        from . import mtile_bf16 as mt

        _retained(x, self.m, self.k)
        if not isinstance(out, torch.Tensor):
            raise ValueError("out must be a tensor; use linear(x) to allocate")
        with torch.cuda.device(x.device):
            return mt.fused_linear(x, self._packed, threads=self.threads, vector=self.vector,
                                   output_dtype=self.output_dtype, out=out)


class RawCandidate(_Candidate):
    """Raw BF16 over the caller's original weight [N, K] (not copied)."""

    def __init__(self, w, tokens=1, *, threads, vector, output_dtype):
        super().__init__()
        started = time.perf_counter()
        if not isinstance(w, torch.Tensor) or w.device.type != "cuda":
            raise ValueError("w must be a CUDA tensor")
        _check_operand(w, "w", torch.bfloat16, 2)
        self._contract("raw", tokens, *w.shape, threads, vector, output_dtype)
        self._bind(w.device)
        self.register_buffer("w", w, persistent=False)
        self.storage = {"format": "raw_bf16", "bytes": 2 * self.n * self.k}
        self.provenance = {"weights": "caller's original tensor; not copied or hashed"}
        self._finish(started)

    def linear(self, x):
        return _RAW_OP(x, self.w, self.m, self.n, self.k, self.threads, self.vector, self.output_dtype)

    def linear_out(self, x, *, out):
        from . import mtile_bf16 as mt

        _retained(x, self.m, self.k)
        if not isinstance(out, torch.Tensor):
            raise ValueError("out must be a tensor; use linear(x) to allocate")
        with torch.cuda.device(x.device):
            return mt.raw_linear(x, self.w, threads=self.threads, vector=self.vector,
                                 output_dtype=self.output_dtype, out=out)
