"""Kernel images launched by name through the driver ABI (drop-in for cuda_module.py).

The reference compiles .cu sources with NVRTC at run time and loads the PTX
through native/driver.cpp (cuda_module.py:99-246). On B200 the images are
cubins built ahead of time for sm_100a (klab_b200/_lib/*.cubin) and loaded with
the same lab_load_* / lab_get_kernel / lab_launch C ABI, re-exported by
libklab_b200.so. Launch semantics are the reference's: torch's current stream,
2-D grid, 1-D block, zero dynamic shared memory (lab_launch_ex adds both).
"""

from __future__ import annotations

import copy
import ctypes as ct
import hashlib
from pathlib import Path

from . import _native

MAX_BLOCK_THREADS = 1024
MAX_GRID = (2 ** 31 - 1, 65535)
IMAGES = {"prefetch_kernels": _native.PREFETCH_CUBIN}


def _resolve(source):
    name = Path(str(source)).stem
    if name in IMAGES:
        return IMAGES[name]
    path = Path(source)
    if path.suffix in (".cubin", ".fatbin", ".ptx") and path.is_file():
        return path
    raise FileNotFoundError(f"No prebuilt sm_100a image for {source!r}; known images: {sorted(IMAGES)}")


class CudaModule:
    """One device's kernel image, launched through the C ABI. close() waits for
    the device and unloads; never replay a graph that captured its kernels after that."""

    def __init__(self, sources, names, device: int):
        if isinstance(sources, (str, bytes)) or not sources:
            raise ValueError("Sources must be a nonempty sequence of image names")
        if isinstance(names, (str, bytes)):
            raise ValueError("names must be a sequence of kernel names")
        names = tuple(names)
        if not names or len(set(names)) != len(names) or not all(isinstance(n, str) and n.isidentifier() for n in names):
            raise ValueError("Kernel names must be distinct C identifiers")
        if isinstance(device, bool) or not isinstance(device, int) or device < 0:
            raise ValueError("device must be a nonnegative CUDA device index")
        import torch

        if not torch.cuda.is_available() or device >= torch.cuda.device_count():
            raise ValueError(f"CUDA device {device} is not available")
        if len(sources) != 1:
            raise ValueError("Exactly one prebuilt image per module")
        image = _resolve(sources[0])
        lib = _native.lib()
        self.device = device
        self._lib = lib
        self._module = ct.c_void_p()
        self._functions = {}
        with torch.cuda.device(device):
            torch.empty(1, device=torch.device("cuda", device))  # make the primary context current
            self._check(lib.lab_load_file(str(image).encode(), ct.byref(self._module)))
            try:
                for name in names:
                    fn = ct.c_void_p()
                    self._check(lib.lab_get_kernel(self._module, name.encode(), ct.byref(fn)))
                    self._functions[name] = fn
            except BaseException:
                lib.lab_unload(self._module)
                self._module = ct.c_void_p()
                raise
        digest = hashlib.sha256(Path(image).read_bytes()).hexdigest()
        self._compilation = {"image": Path(image).name, "image_sha256": digest, "architecture": "sm_100a",
                             "kernels": list(names), "device": device}
        self._fingerprint = {"sources": [Path(image).name], "source_sha256": {Path(image).name: digest},
                             "fingerprint_sha256": digest}

    @property
    def compilation(self):
        return copy.deepcopy(self._compilation)

    @property
    def fingerprint(self):
        return copy.deepcopy(self._fingerprint)

    @property
    def closed(self):
        return not self._module.value

    def _check(self, status):
        if status:
            raise RuntimeError(self._lib.lab_error_string(status).decode())

    def launch(self, name, grid, threads, *args, smem=0, pdl=False):
        """Enqueue `name` on the current stream; args are CUDA tensors or ctypes scalars."""
        import torch

        if self.closed:
            raise RuntimeError("CudaModule is closed")
        if name not in self._functions:
            raise ValueError(f"Kernel {name!r} was not loaded by this module")
        grid = tuple(grid)
        if len(grid) != 2:
            raise ValueError("grid must be (x, y)")
        for value, limit in ((grid[0], MAX_GRID[0]), (grid[1], MAX_GRID[1]), (threads, MAX_BLOCK_THREADS)):
            if isinstance(value, bool) or not isinstance(value, int) or not 1 <= value <= limit:
                raise ValueError("Grid/block dimensions must be positive integers within CUDA limits")
        device = torch.device("cuda", self.device)
        values = []
        for arg in args:
            if isinstance(arg, torch.Tensor):
                if arg.device != device:
                    raise ValueError("All tensors must be on this module's CUDA device")
                values.append(ct.c_void_p(arg.data_ptr()))
            elif isinstance(arg, ct._SimpleCData):
                values.append(arg)
            else:
                raise TypeError("Kernel arguments must be torch tensors or ctypes scalars")
        params = (ct.c_void_p * max(1, len(values)))(*[ct.cast(ct.byref(v), ct.c_void_p) for v in values])
        stream = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            if smem or pdl:
                rc = self._lib.lab_launch_ex(self._functions[name], grid[0], grid[1], threads, smem,
                                             1 if pdl else 0, ct.c_void_p(stream.cuda_stream), params)
            else:
                rc = self._lib.lab_launch(self._functions[name], grid[0], grid[1], threads,
                                          ct.c_void_p(stream.cuda_stream), params)
            self._check(rc)
        _native.record(stream, *[a for a in args if isinstance(a, torch.Tensor)])

    def close(self):
        if self._module.value:
            import torch

            with torch.cuda.device(self.device):
                torch.cuda.synchronize(self.device)
                self._check(self._lib.lab_unload(self._module))
            self._module = ct.c_void_p()
            self._functions.clear()

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()
