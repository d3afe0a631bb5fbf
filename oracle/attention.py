"""FP64 decode attention (test infrastructure only): the reference test's
reference() (research/l2-prefetch/tests/test_decode.py:16-21) restated in numpy.
Keys/values of the first L cached tokens plus the new token; head i uses kv head
i // (heads // kv_heads); scores scaled by 1/8 (head dimension 64)."""

from __future__ import annotations

import numpy as np

from .bf16 import bf16_values


def decode_attention64(q_bits, kn_bits, vn_bits, k_bits, v_bits, length: int, heads: int, kv_heads: int):
    hd = 64
    K = bf16_values(k_bits)[:, :length]
    V = bf16_values(v_bits)[:, :length]
    Kf = np.concatenate([K, bf16_values(kn_bits).reshape(kv_heads, 1, hd)], axis=1)
    Vf = np.concatenate([V, bf16_values(vn_bits).reshape(kv_heads, 1, hd)], axis=1)
    q = bf16_values(q_bits).reshape(heads, hd)
    g = heads // kv_heads
    out = np.empty((heads, hd))
    for i in range(heads):
        s = Kf[i // g] @ q[i] / 8.0
        p = np.exp(s - s.max())
        out[i] = (p / p.sum()) @ Vf[i // g]
    return out.reshape(-1)
