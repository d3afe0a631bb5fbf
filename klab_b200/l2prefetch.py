"""Side-stream L2 prefetch for chains of projections (drop-in for
research/l2-prefetch/src/l2prefetch.py).

prefetch() never writes the tensor it reads. ChainRunner runs op i on the
current stream while a side stream prefetches the tensors op i+distance reads
(l2prefetch.py:38-60); both are capturable in one CUDA graph. On B200 (126 MB
L2) a layer's weights are far larger than L2, so useful plans prefetch only the
head of the next weight (nbytes); the policy module decides from measurements.
"""

from __future__ import annotations

import ctypes as ct

import torch

from . import _native

KERNELS = ("l2_hint", "l2_load", "l2_hint_last", "l2_bulk")
_KIND = {"l2_hint": _native.L2_HINT, "l2_hint_last": _native.L2_HINT_LAST, "l2_load": _native.L2_LOAD,
         "l2_bulk": _native.L2_BULK}
_modules = {}
_sink = {}


def module(device=None):
    """The prefetch kernels as a name-launched module (the lab_* driver ABI path)."""
    from .cuda_module import CudaModule

    index = torch.cuda.current_device() if device is None else int(device)
    if index not in _modules or _modules[index].closed:
        _modules[index] = CudaModule(("prefetch_kernels",), KERNELS, index)
    return _modules[index]


def prefetch(tensor, blocks, kernel="l2_hint", stride=128, threads=256, nbytes=None):
    """Enqueue an L2 prefetch of `tensor`'s bytes (or its first `nbytes`) on the current stream.
    kernel "l2_bulk" (this library's own) hands `stride` bytes per request (16 B .. 64 KiB) to the
    bulk-copy engine, so a few threads cover the range."""
    if blocks <= 0:
        return
    if kernel not in _KIND:
        raise ValueError(f"kernel must be one of {KERNELS}")
    device = tensor.device
    if device not in _sink:
        _sink[device] = torch.zeros(1, dtype=torch.int32, device=device)
    total = tensor.numel() * tensor.element_size()
    size = total if nbytes is None else min(int(nbytes), total)
    stream = torch.cuda.current_stream(device)
    with torch.cuda.device(device):
        rc = _native.lib().klab_l2_prefetch(tensor.data_ptr(), ct.c_longlong(size), int(blocks), int(threads),
                                            int(stride), _KIND[kernel], _sink[device].data_ptr(),
                                            stream.cuda_stream)
    _native.check(rc, "klab_l2_prefetch")
    _native.record(stream, tensor)


class ChainRunner:
    """ops[i](y) -> y; reads[i] = tensors op i reads that are worth prefetching;
    plans[i] = prefetch kwargs or None (l2prefetch.py:38-60)."""

    def __init__(self, ops, reads, plans=None, distance=1):
        self.ops, self.reads, self.distance = ops, reads, distance
        self.plans = plans if plans is not None else [None] * len(ops)
        self.side = torch.cuda.Stream()

    def __call__(self, y):
        main = torch.cuda.current_stream()
        used = False
        for i, op in enumerate(self.ops):
            j = i + self.distance
            if j < len(self.ops) and self.plans[j]:
                self.side.wait_stream(main)  # starts when op i starts
                with torch.cuda.stream(self.side):
                    for t in self.reads[j]:
                        prefetch(t, **self.plans[j])
                used = True
            y = op(y)
        if used:
            main.wait_stream(self.side)
        return y
