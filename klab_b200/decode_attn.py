"""Decode attention with the fused KV append (drop-in for
research/l2-prefetch/src/decode_attn.py:20-107), plus the decode elementwise
ops of the same module (add_rmsnorm, silu_mul; see decode_ops).

decode_attention(q, k_new, v_new, k_cache, v_cache, length) writes k_new/v_new
at position `length` of the caches and returns softmax(q K^T / 8) V over
length + 1 tokens (heads of 64, grouped-query: heads % kv_heads == 0, up to 16
query heads per kv head). The reference's `kernel` choices are accepted as hints
(with their validation); one B200 kernel serves all of them.
decode_attention_dynamic takes the length as a CUDA int32 tensor so a captured
graph stays valid while the caller advances it.
"""

from __future__ import annotations

import math

import torch

from . import _native
from ._module import get_module
from .decode_ops import add_rmsnorm, silu_mul  # noqa: F401  (same module surface as the reference)

HD = 64
CHUNK = 64
SOURCE = "klab_b200/csrc/decode_attn.cu"  # the reference names its NVRTC source here
_KERNELS = ("decode_attn_bf16", "decode_attn_v2_bf16", "decode_attn_v3_bf16", "decode_attn_v4_bf16",
            "decode_attn_v5_bf16")
_work = {}


def module():
    """The native module serving these kernels on the current device (the reference's module()
    returns its NVRTC-compiled CudaModule, decode_attn.py:12-17)."""
    return get_module()


def _workspace(device, stream, heads, kv_heads, max_len):
    """Scratch for heads * ceil(max_len / 64) split records (enough for any length) and the
    tickets, one set per (device, stream, shape): calls on different streams may overlap on
    the GPU, so they never share tickets or records. Calls on one stream run in order."""
    key = (device, stream.cuda_stream, heads, kv_heads, max_len)
    if key not in _work:
        _work[key] = (torch.empty(heads * -(-max_len // CHUNK) * (HD + 2), device=device, dtype=torch.float32),
                      torch.zeros(kv_heads, device=device, dtype=torch.int32))
    return _work[key]


def _launch(q, k_new, v_new, k_cache, v_cache, out, len_ptr, length):
    kv_heads, max_len, _ = k_cache.shape
    heads = q.numel() // HD
    get_module(q.device)
    stream = torch.cuda.current_stream(q.device)
    scratch, tickets = _workspace(q.device, stream, heads, kv_heads, max_len)
    with torch.cuda.device(q.device):
        rc = _native.lib().klab_decode_attention(q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(),
                                                 v_cache.data_ptr(), out.data_ptr(), scratch.data_ptr(),
                                                 scratch.numel(), tickets.data_ptr(), len_ptr, length, max_len, heads,
                                                 kv_heads, 1.0 / math.sqrt(HD), stream.cuda_stream)
    _native.check(rc, "klab_decode_attention")
    _native.record(stream, q, k_new, v_new, k_cache, v_cache, out, scratch, tickets)
    return out


def _check_tensors(*tensors):
    for t in tensors:
        if not t.is_contiguous() or t.data_ptr() % 16:
            raise ValueError("Tensors must be contiguous and 16-byte aligned")


def decode_attention(q, k_new, v_new, k_cache, v_cache, length, out=None, kernel="decode_attn_v4_bf16"):
    """q [heads*64], k_new/v_new [kv_heads*64], caches [kv_heads, max_len, 64] (BF16, contiguous).

    Writes k_new/v_new at position `length` and returns softmax(q K^T / 8) V over length+1 tokens.
    """
    kv_heads, max_len, hd = k_cache.shape
    heads = q.numel() // hd
    if (hd != HD or q.dtype != torch.bfloat16 or length + 1 > min(max_len, 4096) or heads % kv_heads
            or kernel not in _KERNELS or heads // kv_heads > 16):
        raise ValueError("Unsupported decode attention shape")
    _check_tensors(q, k_new, v_new, k_cache, v_cache)
    if kernel == "decode_attn_v5_bf16" and heads // kv_heads > 8:
        raise ValueError("v5 supports GQA groups up to 8")
    if out is None:
        out = torch.empty(heads * hd, device=q.device, dtype=torch.bfloat16)
    return _launch(q, k_new, v_new, k_cache, v_cache, out, None, int(length))


def decode_attention_dynamic(q, k_new, v_new, k_cache, v_cache, length, out=None):
    """Like decode_attention, but `length` is a CUDA int32 tensor holding the current cache length.

    The launch shape depends only on the cache capacity, so a captured CUDA graph stays valid while the caller
    increments `length` between replays (length + 1 must stay <= capacity).
    """
    kv_heads, max_len, hd = k_cache.shape
    heads = q.numel() // hd
    if (hd != HD or q.dtype != torch.bfloat16 or heads % kv_heads or length.dtype != torch.int32
            or length.numel() != 1 or heads // kv_heads > 16 or max_len > 65536):
        raise ValueError("Unsupported dynamic decode attention arguments")
    _check_tensors(q, k_new, v_new, k_cache, v_cache)
    if out is None:
        out = torch.empty(heads * hd, device=q.device, dtype=torch.bfloat16)
    return _launch(q, k_new, v_new, k_cache, v_cache, out, length.data_ptr(), 0)
