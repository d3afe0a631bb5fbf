"""Native prepared-plan registry under the reference's operator namespace
(drop-in for the klab_native_v1 library of native/prepared.cpp:417-440 and the
candidates of native_prepared.py:398-565).

Operators (schemas as in the reference):
  klab_native_v1::_register_plan(Tensor ptx_cpu_u8, int device, int m, int n, int k,
                                 int threads, int vector, str kind, str output_dtype,
                                 str ptx_sha256) -> int
  klab_native_v1::raw(Tensor x, Tensor w, int plan, int m, int n, int k, int threads,
                      int vector, str output_dtype) -> Tensor
  klab_native_v1::coded(Tensor x, Tensor payload, Tensor metadata, int plan, int m, int n,
                        int k, int threads, int vector, str output_dtype) -> Tensor
  klab_native_v1::_retire_plan(int plan) -> ()
  klab_native_v1::plan_info(int plan) -> str
The reference registers its own compiled image with each plan; here the image
bytes are only integrity-checked against ptx_sha256 (the launch runs the sm_100a
kernels of libklab_b200, planned by klab_plan_create), so any caller image or a
descriptor works. raw/coded check x and the operands against the registered case
and launch the plan; Fake kernels check the logical contract only.
"""

from __future__ import annotations

import hashlib
import itertools
import json
import re
import threading
import time

import torch

from . import _native
from . import prepared_kernels as pk
from .prepared import PreparedPlan, output_name

NAMESPACE = "klab_native_v1"
_REGISTRY = {}            # plan id -> (PreparedPlan, case dict)
_LOCK = threading.Lock()
_IDS = itertools.count(1)
_SHA256 = re.compile(r"[0-9a-f]{64}")

_LIB = torch.library.Library(NAMESPACE, "DEF")
_LIB.define("raw(Tensor x, Tensor w, int plan, int m, int n, int k, int threads, int vector, "
            "str output_dtype) -> Tensor")
_LIB.define("coded(Tensor x, Tensor payload, Tensor metadata, int plan, int m, int n, int k, int threads, "
            "int vector, str output_dtype) -> Tensor")
_LIB.define("_register_plan(Tensor ptx_cpu_u8, int device, int m, int n, int k, int threads, int vector, "
            "str kind, str output_dtype, str ptx_sha256) -> int")
_LIB.define("_retire_plan(int plan) -> ()")
_LIB.define("plan_info(int plan) -> str")


def _register_plan(ptx_cpu_u8, device, m, n, k, threads, vector, kind, output_dtype, ptx_sha256):
    t = ptx_cpu_u8
    if not isinstance(t, torch.Tensor) or t.device.type != "cpu" or t.dtype != torch.uint8 or t.ndim != 1 \
            or not t.is_contiguous() or t.numel() == 0:
        raise ValueError("ptx_cpu_u8 must be a nonempty contiguous 1-D CPU uint8 tensor")
    if not _SHA256.fullmatch(ptx_sha256):
        raise ValueError("ptx_sha256 must be a lowercase SHA-256 hex digest")
    image = t.numpy().tobytes()
    if b"\0" in image:
        raise ValueError("PTX bytes must not contain NUL characters")
    if hashlib.sha256(image).hexdigest() != ptx_sha256:
        raise ValueError("ptx_sha256 does not match the image bytes")
    if kind not in ("raw", "coded"):
        raise ValueError("kind must be 'raw' or 'coded'")
    output = output_name(output_dtype)
    pk._check_plan(m, n, k, threads, vector, coded=kind == "coded")
    if not 0 <= device < torch.cuda.device_count():
        raise ValueError(f"CUDA device {device} is not available")
    wfmt = _native.W_CBF16 if kind == "coded" else _native.W_BF16
    plan = PreparedPlan(wfmt, torch.bfloat16, output, m, n, k, torch.device("cuda", device))
    pid = next(_IDS)
    info = plan.info
    case = {"plan": pid, "kind": kind, "output_dtype": output, "device": device, "shape_mnk": [m, n, k],
            "threads": threads, "vector": vector, "tile": info["tile"], "route": "B200 prepared plan",
            "kernel": info["kernel"], "grid": info["grid"], "block": info["block"],
            "dynamic_shared_bytes": info["dynamic_shared_bytes"], "ptx_sha256": ptx_sha256, "launch": info}
    with _LOCK:
        _REGISTRY[pid] = (plan, case)
    return pid


def _lookup(plan, kind, m, n, k, threads, vector, output_dtype):
    with _LOCK:
        entry = _REGISTRY.get(plan)
    if entry is None:
        raise ValueError(f"Unknown or retired plan {plan}")
    prepared, case = entry
    if (case["kind"], case["shape_mnk"], case["threads"], case["vector"], case["output_dtype"]) != \
            (kind, [m, n, k], threads, vector, output_name(output_dtype)):
        raise ValueError("Arguments do not match the registered plan")
    return prepared


def _raw(x, w, plan, m, n, k, threads, vector, output_dtype):
    prepared = _lookup(plan, "raw", m, n, k, threads, vector, output_dtype)
    pk._check_operand(x, "x", torch.bfloat16, 2, (m, k))
    pk._check_operand(w, "w", torch.bfloat16, 2, (n, k))
    if x.device != prepared.device or w.device != x.device:
        raise ValueError("x and w must be on the plan's device")
    return prepared.launch(x, w)


def _coded(x, payload, metadata, plan, m, n, k, threads, vector, output_dtype):
    prepared = _lookup(plan, "coded", m, n, k, threads, vector, output_dtype)
    pk._check_operand(x, "x", torch.bfloat16, 2, (m, k))
    pk._check_operand(payload, "payload", torch.uint8, 1)
    pk._check_operand(metadata, "metadata", torch.int32, 1)
    if x.device != prepared.device or payload.device != x.device or metadata.device != x.device:
        raise ValueError("x, payload and metadata must be on the plan's device")
    pk._check_coded_buffers(payload, metadata, n, k)
    if payload.data_ptr() % 32 or metadata.data_ptr() % 16:
        raise ValueError("Packed buffers must keep their 32-byte payload alignment")
    return prepared.launch(x, payload, metadata)


def _retire(plan):
    with _LOCK:
        entry = _REGISTRY.pop(plan, None)
    if entry is None:
        raise ValueError(f"Unknown or retired plan {plan}")
    entry[0].close()


def _info(plan):
    with _LOCK:
        entry = _REGISTRY.get(plan)
    if entry is None:
        raise ValueError(f"Unknown or retired plan {plan}")
    return json.dumps(entry[1])


_LIB.impl("raw", _raw, "CUDA")
_LIB.impl("coded", _coded, "CUDA")
_LIB.impl("_register_plan", _register_plan, "CPU")
_LIB.impl("_retire_plan", _retire, "CompositeExplicitAutograd")
_LIB.impl("plan_info", _info, "CompositeExplicitAutograd")


@torch.library.register_fake(f"{NAMESPACE}::raw")
def _raw_fake(x, w, plan, m, n, k, threads, vector, output_dtype):
    dtype = {"bf16": torch.bfloat16, "fp32": torch.float32}[output_name(output_dtype)]
    pk._check_plan(m, n, k, threads, vector, coded=False)
    pk._check_operand(x, "x", torch.bfloat16, 2, (m, k))
    pk._check_operand(w, "w", torch.bfloat16, 2, (n, k))
    return x.new_empty((m, n), dtype=dtype)


@torch.library.register_fake(f"{NAMESPACE}::coded")
def _coded_fake(x, payload, metadata, plan, m, n, k, threads, vector, output_dtype):
    dtype = {"bf16": torch.bfloat16, "fp32": torch.float32}[output_name(output_dtype)]
    pk._check_plan(m, n, k, threads, vector, coded=True)
    pk._check_operand(x, "x", torch.bfloat16, 2, (m, k))
    pk._check_operand(payload, "payload", torch.uint8, 1)
    pk._check_operand(metadata, "metadata", torch.int32, 1)
    pk._check_coded_buffers(payload, metadata, n, k)
    return x.new_empty((m, n), dtype=dtype)


def _descriptor():
    """Bytes registered with each candidate's plan: the library version and kernel."""
    text = f"libklab_b200 {_native.lib().klab_version()} stream_gemv_kernel sm_100a".encode()
    return torch.frombuffer(bytearray(text), dtype=torch.uint8), hashlib.sha256(text).hexdigest()


class _NativeCandidate(torch.nn.Module):
    """One device-bound native (M, N, K, output) plan in the registry."""

    custom_win_validated = False
    eager_promoted = False

    def __init__(self):
        super().__init__()
        self.plan_id = None
        self.closed = False

    def _prepare(self, kind, tokens, n, k, threads, vector, output_dtype, device):
        self.output_dtype = output_name(output_dtype)
        pk._check_plan(tokens, n, k, threads, vector, coded=kind == "coded")
        self.kind, self.m, self.n, self.k = kind, tokens, n, k
        self.shape_mnk = (tokens, n, k)
        self.threads, self.vector = threads, vector
        index = device.index
        with torch.cuda.device(index):
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Prepare native candidates before CUDA graph capture")
            self.precision_flags = {
                "allow_tf32": torch.backends.cuda.matmul.allow_tf32,
                "allow_bf16_reduced_precision_reduction":
                    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction}
            if any(self.precision_flags.values()):
                raise ValueError("Set allow_tf32 and allow_bf16_reduced_precision_reduction to False "
                                 "before preparing this FP32-accumulation contract")
            image, digest = _descriptor()
            ops = getattr(torch.ops, NAMESPACE)
            self.plan_id = ops._register_plan(image, index, tokens, n, k, threads, vector, kind,
                                              self.output_dtype, digest)
            self.plan_info = json.loads(ops.plan_info(self.plan_id))
        self._op = getattr(getattr(torch.ops, NAMESPACE), kind).default
        self.device = torch.device("cuda", index)
        self.config = {"threads": threads, "vector": vector, "tile": self.plan_info["tile"],
                       "kernel": self.plan_info["kernel"], "grid": self.plan_info["grid"],
                       "dispatch": f"{NAMESPACE} operator over a klab_plan_create plan"}

    def _apply(self, fn, recurse=True):
        raise RuntimeError(f"{type(self).__name__} is a device-bound prepared plan; reprepare it instead")

    def forward(self, x):
        return self.linear(x)

    def close(self):
        """Retire the plan (after every graph that captured it is gone)."""
        if not self.closed and self.plan_id is not None:
            getattr(torch.ops, NAMESPACE)._retire_plan(self.plan_id)
            self.closed = True


class NativeRawCandidate(_NativeCandidate):
    def __init__(self, w, tokens=1, *, threads, vector, output_dtype):
        super().__init__()
        started = time.perf_counter()
        if not isinstance(w, torch.Tensor) or w.device.type != "cuda":
            raise ValueError("w must be a CUDA tensor")
        pk._check_operand(w, "w", torch.bfloat16, 2)
        self._prepare("raw", tokens, *w.shape, threads, vector, output_dtype, w.device)
        self.register_buffer("w", w, persistent=False)
        self.linear(torch.zeros((self.m, self.k), dtype=torch.bfloat16, device=self.device))
        self.setup_seconds = time.perf_counter() - started

    def linear(self, x):
        return self._op(x, self.w, self.plan_id, self.m, self.n, self.k, self.threads, self.vector,
                        self.output_dtype)


class NativeCodedCandidate(_NativeCandidate):
    def __init__(self, packed, tokens=1, *, threads, vector, output_dtype):
        super().__init__()
        started = time.perf_counter()
        from . import compressed_bf16 as cb

        if not isinstance(packed, cb.PackedBF16):
            raise ValueError("packed must come from compressed_bf16.upload()")
        self._prepare("coded", tokens, packed.n, packed.k, threads, vector, output_dtype, packed.payload.device)
        self.register_buffer("payload", packed.payload, persistent=False)
        self.register_buffer("metadata", packed.metadata, persistent=False)
        self.linear(torch.zeros((self.m, self.k), dtype=torch.bfloat16, device=self.device))
        self.setup_seconds = time.perf_counter() - started

    def linear(self, x):
        return self._op(x, self.payload, self.metadata, self.plan_id, self.m, self.n, self.k, self.threads,
                        self.vector, self.output_dtype)
