"""Per-device handle on the loaded native library (stands where the reference
keeps its NVRTC-compiled CudaModule, compressed_bf16.py:273-289): identity
and fingerprint of the sm_100a build, and the load-outside-capture rule."""

from __future__ import annotations

import copy
import hashlib
import json
import threading

from . import _native

_MODULES = {}
_LOCK = threading.Lock()
_LIB_SHA256 = None


def _library_sha256():
    global _LIB_SHA256
    if _LIB_SHA256 is None:
        _LIB_SHA256 = hashlib.sha256(_native.LIB_PATH.read_bytes()).hexdigest()
    return _LIB_SHA256


class NativeModule:
    """The sm_100a kernels of libklab_b200.so as seen from one CUDA device."""

    def __init__(self, device: int):
        import torch

        self.device = device
        _native.lib()
        major, minor = torch.cuda.get_device_capability(device)
        self._compilation = {"library": _native.LIB_PATH.name, "library_sha256": _library_sha256(),
                             "architecture": "sm_100a", "device_capability": f"{major}.{minor}",
                             "compiler": "nvcc (ahead of time)", "device": device,
                             "launch_abi": "klab_b200.h typed entry points"}
        text = json.dumps(self._compilation, sort_keys=True)
        self._fingerprint = {**self._compilation,
                             "fingerprint_sha256": hashlib.sha256(text.encode()).hexdigest()}
        self._closed = False

    @property
    def compilation(self):
        return copy.deepcopy(self._compilation)

    @property
    def fingerprint(self):
        return copy.deepcopy(self._fingerprint)

    @property
    def closed(self):
        return self._closed

    def close(self):
        self._closed = True


def device_index(device) -> int:
    import torch

    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, bool):
        raise ValueError("device must be a CUDA device")
    if isinstance(device, int):
        return device
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("device must be a CUDA device")
    return torch.cuda.current_device() if device.index is None else device.index


def get_module(device=None, *, require_sm100=True) -> NativeModule:
    """This device's module. Create it outside CUDA graph capture."""
    import torch

    index = device_index(device)
    with _LOCK:
        module = _MODULES.get(index)
        if module is not None and not module.closed:
            return module
        if not torch.cuda.is_available() or not 0 <= index < torch.cuda.device_count():
            raise ValueError(f"CUDA device {index} is not available")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Load the projection module (upload/get_module) before CUDA graph capture")
        if require_sm100 and torch.cuda.get_device_capability(index) != (10, 0):
            raise RuntimeError("klab_b200 kernels are built for sm_100a (B200) only")
        module = NativeModule(index)
        _MODULES[index] = module
        return module
