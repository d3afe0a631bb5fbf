"""The decode attention oracle against torch's float64 scaled_dot_product_attention
(grouped-query heads) on CPU, on the reference test's shapes
(research/l2-prefetch/tests/test_decode.py)."""

import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import gemv as og
from oracle.bf16 import bf16_values


@pytest.mark.parametrize("h,kvh,L,cap", [(9, 3, 0, 16), (14, 2, 7, 16), (32, 4, 300, 512), (16, 16, 63, 64)])
def test_oracle_matches_torch_sdpa(h, kvh, L, cap):
    q = og.normal_bf16_bits(1, (h * 64,))
    kn, vn = og.normal_bf16_bits(2, (kvh * 64,)), og.normal_bf16_bits(3, (kvh * 64,))
    K, V = og.normal_bf16_bits(4, (kvh, cap, 64)), og.normal_bf16_bits(5, (kvh, cap, 64))
    got = oa.decode_attention64(q, kn, vn, K, V, L, h, kvh)
    Kf = np.concatenate([bf16_values(K)[:, :L], bf16_values(kn).reshape(kvh, 1, 64)], axis=1)
    Vf = np.concatenate([bf16_values(V)[:, :L], bf16_values(vn).reshape(kvh, 1, 64)], axis=1)
    ref = torch.nn.functional.scaled_dot_product_attention(
        torch.from_numpy(bf16_values(q).reshape(1, h, 1, 64)), torch.from_numpy(Kf)[None],
        torch.from_numpy(Vf)[None], enable_gqa=True).reshape(-1).numpy()
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-12)


def test_single_token_returns_new_value():
    q, kn = og.normal_bf16_bits(1, (128,)), og.normal_bf16_bits(2, (64,))
    vn = og.normal_bf16_bits(3, (64,))
    K = V = np.zeros((1, 4, 64), dtype=np.uint16)
    got = oa.decode_attention64(q, kn, vn, K, V, 0, 2, 1)
    np.testing.assert_array_equal(got.reshape(2, 64), np.stack([bf16_values(vn)] * 2))


def test_decode_attn_module_surface():
    """The mirror keeps the reference module's public names (decode_attn.py:7-107)."""
    import klab_b200.decode_attn as d

    for name in ("module", "decode_attention", "decode_attention_dynamic", "add_rmsnorm", "silu_mul"):
        assert callable(getattr(d, name)), name
    assert d.SOURCE.endswith("decode_attn.cu")
