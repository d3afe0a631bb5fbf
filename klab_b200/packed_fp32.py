"""Lossless FP32 weights as 28-bit codes (drop-in for packed_fp32.py).

Per 64-weight block: 64 codes of 28 bits (23 mantissa bits, the sign, a 4-bit
exponent delta from the block minimum) packed eight to seven 32-bit words, or
the 64 original words when a delta exceeds 15; one 32-bit metadata word per
block (packed_fp32.py:35-67; format in klab_b200/csrc/lossless_f32.cuh). The
projection decodes into shared memory and uses the FP32 projection's
arithmetic: results equal klab_f32_linear on the unpacked weights bit for bit.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from ._module import get_module
from .lossless_weights import _blocks, _scatter_blocks

THREADS = (32, 64, 128, 256)


@dataclass(frozen=True)
class PackedFP32Weights:
    payload: torch.Tensor   # int32 [total]
    metadata: torch.Tensor  # int32 [N, K/64]

    @property
    def shape(self):
        return self.metadata.shape[0], self.metadata.shape[1] * 64

    @property
    def storage_bytes(self):
        return (self.payload.numel() + self.metadata.numel()) * 4

    def unpack(self):
        """The original FP32 [N, K] (exact bits)."""
        n, k = self.shape
        out = torch.empty(n, k, dtype=torch.float32, device=self.payload.device)
        stream = torch.cuda.current_stream(self.payload.device)
        with torch.cuda.device(self.payload.device):
            rc = _native.lib().klab_fp28_unpack(self.payload.data_ptr(), self.metadata.data_ptr(), out.data_ptr(),
                                                n * k, stream.cuda_stream)
        _native.check(rc, "klab_fp28_unpack")
        _native.record(stream, self.payload, self.metadata, out)
        return out

    def linear(self, x, threads=128):
        return linear(x, self.payload, self.metadata, threads)


def _code_words(codes):
    """[B, 64] 28-bit codes -> [B, 56] words: the 1,792-bit string of each block
    (code j at bit 28j) cut into 32-bit words."""
    groups = codes.reshape(codes.shape[0], 8, 8)          # 8 codes = 224 bits = 7 words
    words = []
    for wi in range(7):
        first, shift = divmod(32 * wi, 28)
        low = groups[:, :, first] >> shift
        high = groups[:, :, first + 1] << (28 - shift)
        words.append((low | high) & 0xFFFFFFFF)
    return torch.stack(words, dim=-1).reshape(codes.shape[0], 56)


def pack_weights(w):
    """Pack CUDA FP32 [N, K] (K % 64 == 0) without losing a bit."""
    if w.device.type != "cuda" or w.dtype != torch.float32 or w.ndim != 2 or not w.is_contiguous():
        raise ValueError("Expected contiguous CUDA FP32 [N,K]")
    n, k = w.shape
    if w.requires_grad or min(n, k) <= 0 or k % 64 or w.numel() * 4 >= 2 ** 31:
        raise ValueError("Inference only; positive 32-bit-addressable sizes and K divisible by 64 required")
    bits, exps, lo, delta, wide = _blocks(w)
    sign_mant = ((bits & 0x7FFFFF) | ((bits >> 8) & 0x800000)).to(torch.int64).reshape(-1, 64)
    compact = _code_words(sign_mant | ((delta.to(torch.int64) & 0xF) << 24))
    rows = torch.where(wide[:, None], bits.reshape(-1, 64).to(torch.int64) & 0xFFFFFFFF,
                       torch.nn.functional.pad(compact, (0, 8)))
    sizes = torch.where(wide, 64, 56).to(torch.int64)
    words, offsets, total = _scatter_blocks(rows, sizes, torch.int64, w.device)
    if total * 4 >= 2 ** 28:
        raise ValueError("Payload exceeds experimental 256 MiB metadata limit")
    payload = (words - ((words >> 31) << 32)).to(torch.int32)  # two's complement view of each word
    meta = ((offsets >> 3) << 9) | (lo.to(torch.int64) << 1) | wide.to(torch.int64)
    return PackedFP32Weights(payload, meta.to(torch.int32).reshape(n, k // 64).contiguous())


def fused_linear(x, packed, threads=128, out=None):
    """out[M, N] = x[M, K] @ W.T in FP32 (validation as packed_fp32.py:70-84)."""
    if x.device.type != "cuda" or not x.is_contiguous() or x.requires_grad:
        raise ValueError("Inference-only contiguous tensors on the current CUDA device required")
    n, k = packed.shape
    for tensor in (packed.payload, packed.metadata):
        if tensor.device != x.device or not tensor.is_contiguous() or tensor.dtype != torch.int32:
            raise ValueError("Expected intact contiguous int32 packed buffers on the input device")
    if x.dtype != torch.float32:
        raise ValueError("FP32 activations required")
    if x.ndim != 2 or x.shape[1] != k or min(x.shape[0], n, k) <= 0 or k % 64:
        raise ValueError("Expected x=[M,K], matching packed weights")
    if max(x.numel(), n * k, x.shape[0] * n) >= 2 ** 31 or x.data_ptr() % 16 or packed.payload.ndim != 1:
        raise ValueError("Aligned input and positive signed 32-bit indexing required")
    if threads not in THREADS:
        raise ValueError("Unsupported block size")
    m = x.shape[0]
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=torch.float32)
    else:
        if out.dtype != torch.float32 or out.device != x.device or not out.is_contiguous() or out.requires_grad:
            raise ValueError("Only contiguous FP32 output tensors are supported")
        if out.shape != (m, n):
            raise ValueError("Output shape mismatch")
    if any(out.untyped_storage().data_ptr() == v.untyped_storage().data_ptr()
           for v in (x, packed.payload, packed.metadata)):
        raise ValueError("Output cannot alias inputs")
    get_module(x.device)
    return _native.gemv(_native.W_FP28, _native.DT_F32, x, packed.payload, packed.metadata, None, out,
                        _native.DT_F32, m, n, k)


@torch.library.custom_op("kernel_lab::packed_fp32_linear", mutates_args=(), device_types="cuda")
def linear(x: torch.Tensor, payload: torch.Tensor, metadata: torch.Tensor, threads: int = 128) -> torch.Tensor:
    with torch.cuda.device(x.device):
        return fused_linear(x, PackedFP32Weights(payload, metadata), threads)


@linear.register_fake
def _fake(x, payload, metadata, threads=128):
    return x.new_empty((x.shape[0], metadata.shape[0]))
