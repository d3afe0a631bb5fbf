"""Decode attention with the fused KV append against the FP64 oracle, on the
reference test's cases and tolerance (research/l2-prefetch/tests/test_decode.py:
1e-2 * max(1, max|ref|)), plus a tighter bound, the cache append, the dynamic
length under one captured graph, and the reference's argument validation."""

import numpy as np
import pytest
import torch

from oracle import attention as oa
from oracle import gemv as og

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native():
    from klab_b200 import _native

    _native.lib()
    yield _native
    assert _native.device_status(clear=True) == 0


def bits_of(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def case(h, kvh, cap, seed):
    def r(*shape, s):
        return torch.from_numpy(og.normal_bf16_bits(seed * 10 + s, shape, 1.0).view(np.int16)).view(
            torch.bfloat16).cuda()
    return r(h * 64, s=1), r(kvh * 64, s=2), r(kvh * 64, s=3), r(kvh, cap, 64, s=4), r(kvh, cap, 64, s=5)


def check(out, q, kn, vn, K, V, L, h, kvh):
    ref = oa.decode_attention64(bits_of(q), bits_of(kn), bits_of(vn), bits_of(K), bits_of(V), L, h, kvh)
    got = out.double().cpu().numpy()
    err = np.abs(got - ref).max()
    assert err < 1e-2 * max(1.0, np.abs(ref).max())           # the reference test's bound
    assert err <= 2.0 ** -7 * np.abs(ref).max() + 1e-3          # about one BF16 ulp of the largest output


@pytest.mark.parametrize("h,kvh,L,cap", [(9, 3, 0, 512), (14, 2, 7, 512), (32, 4, 300, 512),
                                         (32, 8, 4095, 4096), (16, 1, 63, 128), (16, 16, 64, 128),
                                         (32, 8, 700, 1024), (48, 4, 256, 512)])
def test_matches_oracle_and_appends(h, kvh, L, cap):
    from klab_b200.decode_attn import decode_attention

    q, kn, vn, K, V = case(h, kvh, cap, L + h)
    Kc, Vc = K.clone(), V.clone()
    out = decode_attention(q, kn, vn, Kc, Vc, L)
    check(out, q, kn, vn, K, V, L, h, kvh)
    assert torch.equal(Kc[:, L], kn.view(kvh, 64)) and torch.equal(Vc[:, L], vn.view(kvh, 64))
    assert torch.equal(Kc[:, :L], K[:, :L]) and torch.equal(Kc[:, L + 1:], K[:, L + 1:])


def test_dynamic_length_one_graph():
    from klab_b200.decode_attn import decode_attention_dynamic

    h, kvh = 9, 3
    q, kn, vn, K, V = case(h, kvh, 256, 7)
    Kref, Vref = K.clone(), V.clone()
    length = torch.zeros(1, device="cuda", dtype=torch.int32)
    out = torch.empty(h * 64, device="cuda", dtype=torch.bfloat16)
    decode_attention_dynamic(q, kn, vn, K.clone(), V.clone(), length, out=out)  # warm-up outside capture
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        decode_attention_dynamic(q, kn, vn, K, V, length, out=out)
    for L in (0, 1, 63, 64, 130, 254):
        length.fill_(L)
        graph.replay()
        torch.cuda.synchronize()
        check(out, q, kn, vn, Kref, Vref, L, h, kvh)
        Kref[:, L], Vref[:, L] = kn.view(kvh, 64), vn.view(kvh, 64)
        assert torch.equal(K[:, L], kn.view(kvh, 64))


@pytest.mark.parametrize("h,kvh,L,cap", [(32, 2, 16000, 16384), (16, 1, 9000, 65536), (64, 8, 3000, 4096)])
def test_dynamic_long_spans(h, kvh, L, cap):
    from klab_b200.decode_attn import decode_attention_dynamic

    q, kn, vn, K, V = case(h, kvh, cap, 11)
    Kc, Vc = K.clone(), V.clone()
    out = decode_attention_dynamic(q, kn, vn, Kc, Vc, torch.tensor([L], device="cuda", dtype=torch.int32))
    check(out, q, kn, vn, K, V, L, h, kvh)
    assert torch.equal(Kc[:, L], kn.view(kvh, 64)) and torch.equal(Vc[:, :L], V[:, :L])


def test_repeated_calls_reset_tickets():
    from klab_b200.decode_attn import decode_attention

    q, kn, vn, K, V = case(8, 2, 1024, 3)
    first = decode_attention(q, kn, vn, K.clone(), V.clone(), 700)
    for _ in range(3):
        again = decode_attention(q, kn, vn, K.clone(), V.clone(), 700)
        assert torch.equal(again, first)


def test_validation_matches_reference():
    from klab_b200.decode_attn import decode_attention, decode_attention_dynamic

    q, kn, vn, K, V = case(32, 2, 128, 1)
    with pytest.raises(ValueError):
        decode_attention(q, kn, vn, K, V, 128)                   # length + 1 > capacity
    with pytest.raises(ValueError):
        decode_attention(q, kn, vn, K, V, 3, kernel="decode_attn_v5_bf16")  # group 16 > 8
    q2, kn2, vn2, K2, V2 = case(9, 3, 64, 2)
    with pytest.raises(ValueError):
        decode_attention(q2.float(), kn2, vn2, K2, V2, 3)
    with pytest.raises(ValueError):
        decode_attention_dynamic(q2, kn2, vn2, K2, V2, torch.zeros(1, device="cuda", dtype=torch.int64))


def test_dynamic_length_out_of_range_is_reported(native):
    from klab_b200.decode_attn import decode_attention_dynamic

    q, kn, vn, K, V = case(4, 2, 100, 5)
    Kc, Vc = K.clone(), V.clone()
    out = torch.zeros(4 * 64, device="cuda", dtype=torch.bfloat16)
    assert native.device_status(clear=True) == 0
    for bad in (100, 127, -1):  # capacity 100 spans two chunks: 100..127 would land past the cache
        decode_attention_dynamic(q, kn, vn, Kc, Vc, torch.tensor([bad], device="cuda", dtype=torch.int32), out=out)
        torch.cuda.synchronize()
        assert native.device_status(clear=True) == 3
    assert torch.equal(Kc, K) and torch.equal(Vc, V) and not out.any()
    decode_attention_dynamic(q, kn, vn, Kc, Vc, torch.tensor([99], device="cuda", dtype=torch.int32), out=out)
    torch.cuda.synchronize()
    assert native.device_status(clear=True) == 0
    check(out, q, kn, vn, K, V, 99, 4, 2)
