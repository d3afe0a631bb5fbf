"""Lossless BF16 block storage (format version 1) and BF16 projections on B200.

Drop-in for the reference's compressed_bf16 module (compressed_bf16.py): the
same codec, dataclasses, validation rules, error types and the registered op
compressed_bf16::compressed_linear. The codec runs on the host in C++
(klab_cbf16_pack_host / klab_cbf16_unpack_host); projections run the sm_100a
streaming kernel of libklab_b200.so, which decodes the 12-bit codes in
registers from shared memory filled by bulk copies.

`threads` and `vector` are accepted and validated exactly as the reference
does (they select launch configurations there); the B200 kernel plans its own
launch, so they do not change the arithmetic. Every raw/coded pair of the same
weights is bit-identical, and so is every M.
"""

from __future__ import annotations

import ctypes as ct
import hashlib
import json
from dataclasses import dataclass

import numpy as np
import torch

from . import _native
from ._module import NativeModule, device_index as _device_index, get_module as _get_module

FORMAT_VERSION = 1
BLOCK = 64
CODED_BYTES = 96
RAW_BYTES = 128
UNIT = 32
MAX_PAYLOAD_BYTES = 1 << 28
OFFSET_MASK = 0x7FFFFF
RAW_FLAG = 0x80000000

THREADS = (32, 64, 128, 256)
VECTORS = (2, 8)
OUTPUT_DTYPES = {"bf16": torch.bfloat16, "fp32": torch.float32}
UNPACK_THREADS = 256


@dataclass(frozen=True, eq=False)
class PackedCPU:
    payload: np.ndarray   # uint8, blocks in row-major block order
    metadata: np.ndarray  # uint32, one word per block
    n: int
    k: int
    source_sha256: str
    format_version: int = FORMAT_VERSION

    @property
    def storage_bytes(self):
        return int(self.payload.nbytes + self.metadata.nbytes)


# ---------------------------------------------------------------- CPU codec

def _sha256_bits(bits: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(bits, dtype="<u2").tobytes()).hexdigest()


def pack_bits(bits: np.ndarray) -> PackedCPU:
    """Pack a row-major [N,K] uint16 BF16 bit matrix. Every bit is preserved."""
    if not isinstance(bits, np.ndarray) or bits.dtype.kind != "u" or bits.dtype.itemsize != 2:
        raise ValueError("Expected a numpy uint16 array of BF16 bit patterns")
    if bits.ndim != 2:
        raise ValueError("Expected a two-dimensional [N,K] array")
    n, k = (int(size) for size in bits.shape)
    if min(n, k) <= 0 or n * k >= 2 ** 31:
        raise ValueError("N and K must be positive with N*K < 2^31")
    src = np.ascontiguousarray(bits, dtype="<u2")
    metadata = np.empty(n * ((k + BLOCK - 1) // BLOCK), dtype="<u4")
    size = ct.c_size_t(0)
    lib = _native.lib()
    rc = lib.klab_cbf16_pack_host(src.ctypes.data, n, k, metadata.ctypes.data, None, 0, ct.byref(size))
    if rc == _native.E_SHAPE:
        raise ValueError(f"Payload of {size.value} bytes exceeds the {MAX_PAYLOAD_BYTES}-byte offset range; "
                         "pack smaller tensors separately")
    _native.check(rc, "klab_cbf16_pack_host")
    payload = np.empty(size.value, dtype=np.uint8)
    _native.check(lib.klab_cbf16_pack_host(src.ctypes.data, n, k, metadata.ctypes.data, payload.ctypes.data,
                                           payload.nbytes, ct.byref(size)), "klab_cbf16_pack_host")
    return PackedCPU(payload, metadata, n, k, _sha256_bits(src), FORMAT_VERSION)


def _dimension(value, name):
    if isinstance(value, bool) or not isinstance(value, (int, np.integer)):
        raise ValueError(f"{name} must be an integer")
    return int(value)


def _layout(packed):
    """Type and size checks (compressed_bf16.py:162-200); the byte-level layout is
    checked by the native decoder."""
    if getattr(packed, "format_version", None) != FORMAT_VERSION:
        raise ValueError(f"Unsupported packed format version; expected {FORMAT_VERSION}")
    n, k = _dimension(packed.n, "n"), _dimension(packed.k, "k")
    if min(n, k) <= 0 or n * k >= 2 ** 31:
        raise ValueError("N and K must be positive with N*K < 2^31")
    digest = packed.source_sha256
    if not isinstance(digest, str) or len(digest) != 64 or any(c not in "0123456789abcdef" for c in digest):
        raise ValueError("source_sha256 must be a lowercase SHA-256 hex digest")
    payload, metadata = packed.payload, packed.metadata
    if not isinstance(payload, np.ndarray) or payload.dtype != np.uint8 or payload.ndim != 1:
        raise ValueError("Payload must be a one-dimensional numpy uint8 array")
    if not isinstance(metadata, np.ndarray) or metadata.dtype != np.dtype("<u4") or metadata.ndim != 1:
        raise ValueError("Metadata must be a one-dimensional little-endian uint32 array")
    if metadata.size != n * ((k + BLOCK - 1) // BLOCK):
        raise ValueError("Metadata must contain one word per 64-weight block")
    if payload.size > MAX_PAYLOAD_BYTES:
        raise ValueError("Payload exceeds the version-1 offset range")
    return n, k


def _decode(packed) -> np.ndarray:
    n, k = _layout(packed)
    out = np.empty((n, k), dtype=np.uint16)
    payload = np.ascontiguousarray(packed.payload)
    metadata = np.ascontiguousarray(packed.metadata)
    rc = _native.lib().klab_cbf16_unpack_host(payload.ctypes.data, payload.nbytes, metadata.ctypes.data, n, k,
                                              out.ctypes.data)
    if rc == _native.E_INVALID:
        raise ValueError("Malformed packed BF16 data: offsets, raw-block base, exponent range, "
                         "payload length or tail padding")
    _native.check(rc, "klab_cbf16_unpack_host")
    return out


def validate(packed: PackedCPU) -> None:
    """Fully decode and check layout, exponents, tail padding and the source digest."""
    if _sha256_bits(_decode(packed)) != packed.source_sha256:
        raise ValueError("Decoded bits do not match source_sha256")


def unpack_bits(packed: PackedCPU) -> np.ndarray:
    """Decode to the original [N,K] uint16 bits, after full validation."""
    out = _decode(packed)
    if _sha256_bits(out) != packed.source_sha256:
        raise ValueError("Decoded bits do not match source_sha256")
    return out


# ---------------------------------------------------------------- GPU module

def kernel_names():
    """The reference's kernel name set for this module (compressed_kernels.cu:156-200);
    on B200 all of them map onto the streaming kernel's planner."""
    names = [f"cbf16_{kind}_{output}_t{threads}_v{vector}"
             for kind in ("raw", "coded") for output in OUTPUT_DTYPES
             for vector in VECTORS for threads in THREADS]
    return tuple(names + ["cbf16_unpack"])


def get_module(device=None) -> NativeModule:
    """This device's module; load it outside capture."""
    return _get_module(device)


def _fingerprint(module):
    identity = {"format_version": FORMAT_VERSION, "implementation": "klab_b200.compressed_bf16",
                "kernel_names": list(kernel_names()), "module_fingerprint": module.fingerprint,
                "torch": torch.__version__, "torch_cuda": torch.version.cuda}
    text = json.dumps(identity, sort_keys=True, separators=(",", ":"))
    return {**identity, "fingerprint_sha256": hashlib.sha256(text.encode()).hexdigest()}


def implementation_fingerprint(device=None):
    return _fingerprint(get_module(device))


@dataclass(frozen=True, eq=False)
class PackedBF16:
    payload: torch.Tensor   # uint8 [bytes]
    metadata: torch.Tensor  # int32 [blocks], raw uint32 bits
    n: int
    k: int
    source_sha256: str
    format_version: int
    module: NativeModule

    @property
    def storage_bytes(self):
        return int(self.payload.numel() + 4 * self.metadata.numel())

    @property
    def implementation_fingerprint(self):
        return _fingerprint(self.module)

    def linear(self, x, *, threads, vector, output_dtype):
        """Registered custom op compressed_bf16::compressed_linear (torch.compile-safe)."""
        return compressed_linear(x, self.payload, self.metadata, self.n, self.k,
                                 threads, vector, _output_name(output_dtype))

    def unpack(self):
        return unpack_weights(self)


def upload(packed: PackedCPU, device) -> PackedBF16:
    """Validate a private snapshot of `packed`, load the module, then copy to `device`."""
    index = _device_index(device)
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("upload must run outside CUDA graph capture")
    _layout(packed)
    snapshot = PackedCPU(packed.payload.copy(), packed.metadata.copy(), int(packed.n), int(packed.k),
                         packed.source_sha256, packed.format_version)
    validate(snapshot)
    module = get_module(index)
    target = torch.device("cuda", index)
    payload = torch.from_numpy(snapshot.payload).to(target)
    metadata = torch.from_numpy(snapshot.metadata.view(np.int32)).to(target)
    return PackedBF16(payload, metadata, snapshot.n, snapshot.k, snapshot.source_sha256, FORMAT_VERSION, module)


# ---------------------------------------------------------------- projections

def _output_name(value):
    if isinstance(value, str):
        if value in OUTPUT_DTYPES:
            return value
    else:
        for name, dtype in OUTPUT_DTYPES.items():
            if value is dtype:
                return name
    raise ValueError("output_dtype must be torch.bfloat16/'bf16' or torch.float32/'fp32'")


def _check_tensor(tensor, label, dtype, device, ndim):
    if not isinstance(tensor, torch.Tensor):
        raise ValueError(f"{label} must be a tensor")
    if tensor.device != device or tensor.dtype != dtype or tensor.ndim != ndim:
        raise ValueError(f"{label} must be a {ndim}-D {dtype} tensor on {device}")
    if not tensor.is_contiguous() or tensor.requires_grad:
        raise ValueError(f"{label} must be contiguous and inference-only (no requires_grad)")


def _overlaps(a, b):
    if a.untyped_storage().data_ptr() == b.untyped_storage().data_ptr():
        return True
    a0, b0 = a.data_ptr(), b.data_ptr()
    return a0 < b0 + b.numel() * b.element_size() and b0 < a0 + a.numel() * a.element_size()


def _prepare(x, n, k, threads, vector, output_dtype, out, inputs, aligned=()):
    """Shared validation (compressed_bf16.py:391-418); returns (output name, device, out)."""
    name = _output_name(output_dtype)
    if isinstance(threads, bool) or threads not in THREADS or isinstance(vector, bool) or vector not in VECTORS:
        raise ValueError(f"Unsupported launch configuration; threads in {THREADS}, vector in {VECTORS}")
    if not isinstance(x, torch.Tensor) or x.device.type != "cuda":
        raise ValueError("x must be a CUDA tensor")
    device = x.device
    _check_tensor(x, "x", torch.bfloat16, device, 2)
    m = x.shape[0]
    if x.shape[1] != k:
        raise ValueError("Expected x=[M,K] matching the weights")
    if min(m, n, k) <= 0 or m > 65535 or max(m * k, n * k, m * n) >= 2 ** 31:
        raise ValueError("Dimensions must be positive, M<=65535, and fit signed 32-bit indexing")
    align = 2 * vector
    if k % vector or any(tensor.data_ptr() % align for tensor in (x, *aligned)):
        raise ValueError(f"Require K divisible by {vector} and {align}-byte aligned inputs")
    dtype = OUTPUT_DTYPES[name]
    if out is None:
        out = torch.empty((m, n), dtype=dtype, device=device)
    else:
        _check_tensor(out, "out", dtype, device, 2)
        if tuple(out.shape) != (m, n):
            raise ValueError("Output shape mismatch")
        if any(_overlaps(out, tensor) for tensor in (x, *inputs)):
            raise ValueError("Output must not share storage with x or the weights")
    return name, device, out


def _check_coded_buffers(x, payload, metadata, n, k):
    """compressed_bf16.py:421-437 buffer checks."""
    n, k = _dimension(n, "n"), _dimension(k, "k")
    if not isinstance(x, torch.Tensor):
        raise ValueError("x must be a CUDA tensor")
    _check_tensor(payload, "payload", torch.uint8, x.device, 1)
    _check_tensor(metadata, "metadata", torch.int32, x.device, 1)
    if k <= 0 or k % BLOCK:
        raise ValueError("Fused compressed projections require K divisible by 64; "
                         "use unpack_weights for ragged K")
    blocks = n * (k // BLOCK)
    if metadata.numel() != blocks or not (CODED_BYTES * blocks <= payload.numel() <= RAW_BYTES * blocks):
        raise ValueError("Packed buffers do not match N,K")
    if payload.data_ptr() % UNIT or metadata.data_ptr() % 4:
        raise ValueError("Packed buffers must keep their 32-byte payload alignment")
    return n, k


def _launch_coded(x, payload, metadata, n, k, name, out):
    get_module(x.device)
    dt = _native.DT_BF16 if name == "bf16" else _native.DT_F32
    return _native.gemv(_native.W_CBF16, _native.DT_BF16, x, payload, metadata, None, out, dt, x.shape[0], n, k)


def _coded(x, payload, metadata, n, k, threads, vector, output_dtype, out=None):
    n, k = _check_coded_buffers(x, payload, metadata, n, k)
    name, device, out = _prepare(x, n, k, threads, vector, output_dtype, out, (payload, metadata))
    return _launch_coded(x, payload, metadata, n, k, name, out)


def fused_linear(x, packed: PackedBF16, *, threads, vector, output_dtype, out=None):
    """out[M,N] = x[M,K] @ W.T, decoding exact weights in registers."""
    if not isinstance(packed, PackedBF16):
        raise ValueError("packed must come from upload()")
    return _coded(x, packed.payload, packed.metadata, packed.n, packed.k, threads, vector, output_dtype, out)


def _launch_raw(x, w, n, k, name, out):
    get_module(x.device)
    dt = _native.DT_BF16 if name == "bf16" else _native.DT_F32
    return _native.gemv(_native.W_BF16, _native.DT_BF16, x, w, None, None, out, dt, x.shape[0], n, k)


def raw_linear(x, w, *, threads, vector, output_dtype, out=None):
    """The same arithmetic as fused_linear over an uncompressed BF16 w[N,K]."""
    if not isinstance(x, torch.Tensor):
        raise ValueError("x must be a CUDA tensor")
    _check_tensor(w, "w", torch.bfloat16, x.device, 2)
    n, k = w.shape
    name, device, out = _prepare(x, n, k, threads, vector, output_dtype, out, (w,), aligned=(w,))
    return _launch_raw(x, w, n, k, name, out)


def unpack_weights(packed: PackedBF16) -> torch.Tensor:
    """Integer-only GPU decode to a BF16 [N,K] tensor, for bitwise validation."""
    if not isinstance(packed, PackedBF16):
        raise ValueError("packed must come from upload()")
    device = packed.payload.device
    out = torch.empty((packed.n, packed.k), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    with torch.cuda.device(device):
        rc = _native.lib().klab_cbf16_unpack(packed.payload.data_ptr(), packed.metadata.data_ptr(),
                                             out.data_ptr(), packed.n, packed.k, stream.cuda_stream)
    _native.check(rc, "klab_cbf16_unpack")
    _native.record(stream, packed.payload, packed.metadata, out)
    return out


@torch.library.custom_op("compressed_bf16::compressed_linear", mutates_args=(), device_types="cuda")
def compressed_linear(x: torch.Tensor, payload: torch.Tensor, metadata: torch.Tensor, n: int, k: int,
                      threads: int, vector: int, output_dtype: str) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return _coded(x, payload, metadata, n, k, threads, vector, output_dtype)


@compressed_linear.register_fake
def _compressed_linear_fake(x, payload, metadata, n, k, threads, vector, output_dtype):
    dtype = OUTPUT_DTYPES[_output_name(output_dtype)]
    if (x.dtype != torch.bfloat16 or x.ndim != 2 or payload.dtype != torch.uint8
            or metadata.dtype != torch.int32 or payload.ndim != 1 or metadata.ndim != 1):
        raise ValueError("Expected BF16 x=[M,K], uint8 payload and int32 metadata")
    if x.shape[1] != k or k % BLOCK or metadata.shape[0] != n * (k // BLOCK):
        raise ValueError("Packed buffers do not match x or N,K")
    return x.new_empty((x.shape[0], n), dtype=dtype)
