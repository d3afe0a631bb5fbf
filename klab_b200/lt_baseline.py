"""Frozen cuBLASLt plans: the strongest vendor route for out = x . W^T, as a baseline.

The role of the reference's cublaslt_baseline.py:117-165 (a 64-byte
cublasLtMatmulAlgo_t chosen once, frozen with the context it was chosen in, checked
and restored later, never re-searched on the hot path), for the synthetic benchmark
shapes: no checkpoint is needed.

    plan = tune_plan(x, w, torch.bfloat16)     # heuristic candidates, fastest kept
    record = plan.freeze()                     # JSON-able dict (format klab-lt-plan-v1)
    plan2 = LtPlan.restore(record, device)     # validate_frozen + cublasLtMatmulAlgoCheck
    plan2.run(x, w, out)

Computation: out[M, N] (row-major) = x[M, K] . W[N, K]^T, which column-major is
D[N, M] = op(A) . B with A = W viewed [K, N] (ld K, op = T), B = x viewed [K, M]
(ld K), D = out viewed [N, M] (ld N); CUBLAS_COMPUTE_32F, FP32 alpha = 1, beta = 0.
Inputs BF16 or FP16; output the input type or FP32. Plans run on torch's current
stream and use one per-device workspace allocated outside graph capture.

`validate_frozen` needs neither torch nor the library.
"""

from __future__ import annotations

import base64
import binascii
import ctypes as ct
import threading

FORMAT = "klab-lt-plan-v1"
COMPUTE_32F = 68
_R32F, _R16F, _R16BF = 0, 2, 14
_TYPES = {"bf16": _R16BF, "fp16": _R16F, "fp32": _R32F}
_DESC_TRANSA, _DESC_TRANSB = 3, 4
_PREF_MAX_WORKSPACE = 1
_OP_N, _OP_T = 0, 1
WORKSPACE_BYTES = 32 << 20
CONTEXT_FIELDS = ("library_version", "device_uuid", "input_dtype", "output_dtype", "shape_mnk")
_CONTRACTS = (("bf16", "bf16"), ("bf16", "fp32"), ("fp16", "fp16"), ("fp16", "fp32"))


class LtUnavailable(RuntimeError):
    """libcublasLt or a CUDA device could not be used."""


class _Algo(ct.Structure):
    _fields_ = [("data", ct.c_uint64 * 8)]


class _Result(ct.Structure):
    _fields_ = [("algo", _Algo), ("workspace", ct.c_size_t), ("state", ct.c_int), ("waves", ct.c_float),
                ("reserved", ct.c_int * 4)]


assert ct.sizeof(_Algo) == 64 and ct.sizeof(_Result) == 96


def validate_frozen(record, context):
    """The 64 algorithm bytes of `record`, after checking its format and that it was frozen
    in exactly `context` (every CONTEXT_FIELDS entry equal). Raises ValueError otherwise."""
    if not isinstance(record, dict) or record.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} record")
    need = CONTEXT_FIELDS + ("compute_type", "workspace_bytes", "algorithm_b64")
    missing = [f for f in need if f not in record]
    if missing:
        raise ValueError(f"frozen record lacks {missing}")
    if (record["input_dtype"], record["output_dtype"]) not in _CONTRACTS:
        raise ValueError(f"unsupported dtypes; expected one of {_CONTRACTS}")
    shape = record["shape_mnk"]
    if not (isinstance(shape, (list, tuple)) and len(shape) == 3 and
            all(isinstance(v, int) and not isinstance(v, bool) and 0 < v < 2 ** 31 for v in shape)):
        raise ValueError("shape_mnk must be three positive 32-bit integers")
    if record["compute_type"] != COMPUTE_32F:
        raise ValueError("compute_type must be CUBLAS_COMPUTE_32F (68)")
    ws = record["workspace_bytes"]
    if not (isinstance(ws, int) and 0 <= ws <= WORKSPACE_BYTES):
        raise ValueError(f"workspace_bytes must be in [0, {WORKSPACE_BYTES}]")
    try:
        algo = base64.b64decode(record["algorithm_b64"], validate=True)
    except (binascii.Error, ValueError, TypeError) as error:
        raise ValueError(f"algorithm_b64 is not base64: {error}") from None
    if len(algo) != 64:
        raise ValueError(f"a cublasLtMatmulAlgo_t is 64 bytes, got {len(algo)}")
    if not isinstance(context, dict) or any(f not in context for f in CONTEXT_FIELDS):
        raise ValueError(f"context must give {CONTEXT_FIELDS}")
    for field in CONTEXT_FIELDS:
        want, got = record[field], context[field]
        if (list(want) if isinstance(want, tuple) else want) != (list(got) if isinstance(got, tuple) else got):
            raise ValueError(f"frozen {field} {want!r} differs from the runtime's {got!r}")
    return algo


# ---------------------------------------------------------------- library

_lib_handle = None
_lock = threading.Lock()
_handles, _workspaces = {}, {}


def _lib():
    global _lib_handle
    if _lib_handle is not None:
        return _lib_handle
    try:
        from pathlib import Path

        import nvidia.cublas

        lib = ct.CDLL(str(Path(next(iter(nvidia.cublas.__path__))) / "lib" / "libcublasLt.so.12"))
    except Exception as error:  # noqa: BLE001
        raise LtUnavailable(f"libcublasLt.so.12 unavailable: {error}") from None
    P, I, S = ct.c_void_p, ct.c_int, ct.c_size_t
    sig = {
        "cublasLtCreate": [ct.POINTER(P)],
        "cublasLtMatmulDescCreate": [ct.POINTER(P), I, I],
        "cublasLtMatmulDescDestroy": [P],
        "cublasLtMatmulDescSetAttribute": [P, I, P, S],
        "cublasLtMatrixLayoutCreate": [ct.POINTER(P), I, ct.c_uint64, ct.c_uint64, ct.c_int64],
        "cublasLtMatrixLayoutDestroy": [P],
        "cublasLtMatmulPreferenceCreate": [ct.POINTER(P)],
        "cublasLtMatmulPreferenceDestroy": [P],
        "cublasLtMatmulPreferenceSetAttribute": [P, I, P, S],
        "cublasLtMatmulAlgoGetHeuristic": [P] * 7 + [I, ct.POINTER(_Result), ct.POINTER(I)],
        "cublasLtMatmulAlgoCheck": [P] * 6 + [ct.POINTER(_Algo), ct.POINTER(_Result)],
        "cublasLtMatmul": [P] * 12 + [ct.POINTER(_Algo), P, S, P],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, I
    lib.cublasLtGetVersion.argtypes, lib.cublasLtGetVersion.restype = [], ct.c_size_t
    _lib_handle = lib
    return lib


def _ok(status, what):
    if status:
        raise RuntimeError(f"{what} failed with cuBLASLt status {status}")


def _dtype_name(dtype):
    import torch

    names = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}
    if dtype not in names:
        raise ValueError(f"unsupported dtype {dtype}")
    return names[dtype]


def runtime_context(device, in_dtype, out_dtype, m, n, k):
    """The context a plan for this device, dtypes and shape is frozen in and checked against."""
    import torch

    device = torch.device(device)
    return {"library_version": int(_lib().cublasLtGetVersion()),
            "device_uuid": "GPU-" + str(torch.cuda.get_device_properties(device).uuid),
            "input_dtype": _dtype_name(in_dtype), "output_dtype": _dtype_name(out_dtype), "shape_mnk": [m, n, k]}


def _device_state(device):
    """(handle, workspace tensor) of a device, created once outside graph capture."""
    import torch

    index = torch.device(device).index
    with _lock:
        if index not in _handles:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("create cuBLASLt plans before CUDA graph capture")
            handle = ct.c_void_p()
            with torch.cuda.device(index):
                _ok(_lib().cublasLtCreate(ct.byref(handle)), "cublasLtCreate")
                _workspaces[index] = torch.empty(WORKSPACE_BYTES, dtype=torch.uint8, device=f"cuda:{index}")
            _handles[index] = handle
        return _handles[index], _workspaces[index]


class LtPlan:
    """One frozen cuBLASLt matmul out[M, N] = x[M, K] . W[N, K]^T."""

    def __init__(self, m, n, k, in_dtype, out_dtype, device, algo=None):
        import torch

        self.m, self.n, self.k = m, n, k
        self.in_dtype, self.out_dtype, self.device = in_dtype, out_dtype, torch.device(device)
        self.context = runtime_context(self.device, in_dtype, out_dtype, m, n, k)
        if (self.context["input_dtype"], self.context["output_dtype"]) not in _CONTRACTS:
            raise ValueError(f"unsupported dtypes; expected one of {_CONTRACTS}")
        self.handle, self.workspace = _device_state(self.device)
        lib = _lib()
        self.desc = ct.c_void_p()
        _ok(lib.cublasLtMatmulDescCreate(ct.byref(self.desc), COMPUTE_32F, _R32F), "cublasLtMatmulDescCreate")
        for attr, value in ((_DESC_TRANSA, _OP_T), (_DESC_TRANSB, _OP_N)):
            v = ct.c_int32(value)
            _ok(lib.cublasLtMatmulDescSetAttribute(self.desc, attr, ct.addressof(v), ct.sizeof(v)),
                "cublasLtMatmulDescSetAttribute")
        tin, tout = _TYPES[self.context["input_dtype"]], _TYPES[self.context["output_dtype"]]
        self.layouts = []
        for typ, rows, cols, ld in ((tin, k, n, k), (tin, k, m, k), (tout, n, m, n), (tout, n, m, n)):
            lay = ct.c_void_p()
            _ok(lib.cublasLtMatrixLayoutCreate(ct.byref(lay), typ, rows, cols, ld), "cublasLtMatrixLayoutCreate")
            self.layouts.append(lay)
        self.algo = _Algo()
        if algo is None:
            found = self.candidates(1)
            if not found:
                raise LtUnavailable("the cuBLASLt heuristic proposed no algorithm")
            algo = found[0]
        ct.memmove(ct.addressof(self.algo), bytes(algo), 64)
        check = _Result()
        _ok(lib.cublasLtMatmulAlgoCheck(self.handle, self.desc, *self.layouts, ct.byref(self.algo), ct.byref(check)),
            "cublasLtMatmulAlgoCheck")
        if check.workspace > WORKSPACE_BYTES:
            raise ValueError(f"algorithm needs {check.workspace} bytes of workspace")
        self.workspace_bytes = int(check.workspace)
        self.alpha, self.beta = ct.c_float(1.0), ct.c_float(0.0)

    def candidates(self, count=8):
        """Up to `count` algorithms the heuristic proposes (64 bytes each), best first."""
        lib = _lib()
        pref = ct.c_void_p()
        _ok(lib.cublasLtMatmulPreferenceCreate(ct.byref(pref)), "cublasLtMatmulPreferenceCreate")
        try:
            cap = ct.c_uint64(WORKSPACE_BYTES)
            _ok(lib.cublasLtMatmulPreferenceSetAttribute(pref, _PREF_MAX_WORKSPACE, ct.addressof(cap), 8),
                "cublasLtMatmulPreferenceSetAttribute")
            results = (_Result * count)()
            found = ct.c_int(0)
            _ok(lib.cublasLtMatmulAlgoGetHeuristic(self.handle, self.desc, *self.layouts, pref, count, results,
                                                   ct.byref(found)), "cublasLtMatmulAlgoGetHeuristic")
        finally:
            lib.cublasLtMatmulPreferenceDestroy(pref)
        return [bytes(ct.string_at(ct.addressof(results[i].algo), 64)) for i in range(found.value)
                if results[i].state == 0]

    def run(self, x, w, out):
        """out = x . W^T on torch's current stream (shapes and dtypes as planned)."""
        import torch

        if tuple(x.shape) != (self.m, self.k) or tuple(w.shape) != (self.n, self.k) or \
                tuple(out.shape) != (self.m, self.n) or x.dtype != self.in_dtype or w.dtype != self.in_dtype or \
                out.dtype != self.out_dtype or not (x.is_contiguous() and w.is_contiguous() and out.is_contiguous()):
            raise ValueError("tensors do not match the plan")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _ok(_lib().cublasLtMatmul(self.handle, self.desc, ct.addressof(self.alpha), w.data_ptr(), self.layouts[0],
                                  x.data_ptr(), self.layouts[1], ct.addressof(self.beta), out.data_ptr(),
                                  self.layouts[2], out.data_ptr(), self.layouts[3], ct.byref(self.algo),
                                  self.workspace.data_ptr(), WORKSPACE_BYTES, ct.c_void_p(stream)), "cublasLtMatmul")
        return out

    def freeze(self):
        return {"format": FORMAT, **self.context, "compute_type": COMPUTE_32F,
                "workspace_bytes": self.workspace_bytes,
                "algorithm_b64": base64.b64encode(ct.string_at(ct.addressof(self.algo), 64)).decode()}

    @classmethod
    def restore(cls, record, device):
        """A plan from a frozen record, checked against this runtime's context and by the library."""
        import torch

        dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
        shape = record.get("shape_mnk") if isinstance(record, dict) else None
        if not (isinstance(shape, (list, tuple)) and len(shape) == 3):
            raise ValueError("frozen record lacks shape_mnk")
        in_dtype, out_dtype = dt.get(record.get("input_dtype")), dt.get(record.get("output_dtype"))
        if in_dtype is None or out_dtype is None:
            raise ValueError("frozen record has unknown dtypes")
        context = runtime_context(device, in_dtype, out_dtype, *shape)
        algo = validate_frozen(record, context)
        return cls(*shape, in_dtype, out_dtype, device, algo)

    def close(self):
        lib = _lib()
        if self.desc:
            for lay in self.layouts:
                lib.cublasLtMatrixLayoutDestroy(lay)
            lib.cublasLtMatmulDescDestroy(self.desc)
            self.desc, self.layouts = ct.c_void_p(), []


def tune_plan(x, w, out_dtype, rounds=9, candidates=8):
    """The heuristic's candidates for out = x . W^T, each timed over `rounds` CUDA-graph
    replays of 8 calls on these tensors; the fastest becomes the plan."""
    import statistics

    import torch

    m, k = x.shape
    n = w.shape[0]
    probe = LtPlan(m, n, k, x.dtype, out_dtype, x.device)
    out = torch.empty((m, n), device=x.device, dtype=out_dtype)
    best, best_us = None, float("inf")
    stream = torch.cuda.Stream(x.device)
    for algo in probe.candidates(candidates):
        try:
            plan = LtPlan(m, n, k, x.dtype, out_dtype, x.device, algo)
        except (RuntimeError, ValueError):
            continue
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            plan.run(x, w, out)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(8):
                plan.run(x, w, out)
        times = []
        for _ in range(rounds):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b) * 1000.0 / 8)
        us = statistics.median(times)
        del graph
        if us < best_us:
            if best is not None:
                best.close()
            best, best_us = plan, us
        else:
            plan.close()
    probe.close()
    if best is None:
        raise LtUnavailable("no cuBLASLt algorithm ran for this shape")
    return best
