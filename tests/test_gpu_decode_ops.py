"""Decode elementwise ops and their fusion into the next projection.

add_rmsnorm / silu_mul against the oracle (x bit-exact; xn and silu_mul inside the
check_outputs interval and within one BF16 ulp of FP64), the reference test's own
check (decode_attn tests, test_fused_elementwise: x == res + y), and the fused
projections bit-identical to the standalone op followed by raw_linear."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native():
    from klab_b200 import _native

    _native.lib()
    yield _native
    assert _native.device_status(clear=True) == 0


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def bits_of(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


@pytest.mark.parametrize("m,d", [(2, 576), (1, 2048), (3, 4096), (2, 14336), (1, 2)])
def test_add_rmsnorm_matches_oracle(m, d):
    from klab_b200 import decode_ops

    res = og.normal_bf16_bits(m + d, (m, d), 1.0)
    y = og.normal_bf16_bits(2 * m + d, (m, d), 1.0)
    w = ob.round_bf16_bits(0.5 + np.random.default_rng(d).random(d))
    x, xn = decode_ops.add_rmsnorm(dev_bf16(res), dev_bf16(y), dev_bf16(w))
    x_ref, xn_ref = og.add_rmsnorm_ref(res, y, w, 1e-6)
    np.testing.assert_array_equal(bits_of(x), x_ref)
    assert torch.equal(x, dev_bf16(res) + dev_bf16(y))  # the reference test's check
    report = ob.check_outputs(xn_ref, xn.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


@pytest.mark.parametrize("m,inter", [(2, 1536), (1, 14336), (3, 4)])
def test_silu_mul_matches_oracle(m, inter):
    from klab_b200 import decode_ops

    gu = og.normal_bf16_bits(m + inter, (m, 2 * inter), 2.0)
    out = decode_ops.silu_mul(dev_bf16(gu))
    report = ob.check_outputs(og.silu_mul64(gu), out.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


@pytest.mark.parametrize("m", [1, 2, 4, 5])
@pytest.mark.parametrize("k", [1024, 4096])
def test_fused_add_rmsnorm_linear_bit_identical(m, k):
    from klab_b200 import compressed_bf16 as cb
    from klab_b200 import decode_ops

    n = 257
    res, y = dev_bf16(og.normal_bf16_bits(m + k, (m, k), 1.0)), dev_bf16(og.normal_bf16_bits(3 * m + k, (m, k), 1.0))
    g = dev_bf16(ob.round_bf16_bits(0.5 + np.random.default_rng(k).random(k)))
    w = dev_bf16(og.normal_bf16_bits(n + k, (n, k), 0.02))
    x_ref, xn = decode_ops.add_rmsnorm(res, y, g)
    ref = cb.raw_linear(xn, w, threads=128, vector=8, output_dtype="bf16")
    x, out = decode_ops.add_rmsnorm_linear(res, y, g, w)
    assert same_bits(out, ref) and same_bits(x, x_ref)
    none, out2 = decode_ops.add_rmsnorm_linear(res, y, g, w, x_out=False)
    assert none is None and same_bits(out2, ref)


@pytest.mark.parametrize("m", [1, 3])
@pytest.mark.parametrize("inter", [1024, 3584])
def test_fused_silu_mul_linear_bit_identical(m, inter):
    from klab_b200 import compressed_bf16 as cb
    from klab_b200 import decode_ops

    n = 200
    gu = dev_bf16(og.normal_bf16_bits(m + inter, (m, 2 * inter), 2.0))
    w = dev_bf16(og.normal_bf16_bits(n + inter, (n, inter), 0.02))
    ref = cb.raw_linear(decode_ops.silu_mul(gu), w, threads=128, vector=8, output_dtype="bf16")
    assert same_bits(decode_ops.silu_mul_linear(gu, w), ref)


def test_fused_ops_replay_in_cuda_graph():
    from klab_b200 import decode_ops

    k, n = 4096, 512
    res, y = torch.randn(1, k, device="cuda").bfloat16(), torch.randn(1, k, device="cuda").bfloat16()
    g = torch.rand(k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    gu = torch.randn(1, 2 * k, device="cuda").bfloat16()
    x0, ref = decode_ops.add_rmsnorm_linear(res, y, g, w)
    ref2 = decode_ops.silu_mul_linear(gu, w)
    out, x_out, out2 = torch.empty_like(ref), torch.empty_like(x0), torch.empty_like(ref2)
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        decode_ops.add_rmsnorm_linear(res, y, g, w, out=out, x_out=x_out)
        decode_ops.silu_mul_linear(gu, w, out=out2)
    torch.cuda.current_stream().wait_stream(stream)
    with torch.cuda.graph(graph, stream=stream):
        decode_ops.add_rmsnorm_linear(res, y, g, w, out=out, x_out=x_out)
        decode_ops.silu_mul_linear(gu, w, out=out2)
    out.zero_()
    out2.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert same_bits(out, ref) and same_bits(x_out, x0) and same_bits(out2, ref2)


def test_validation():
    from klab_b200 import decode_ops

    a = torch.randn(2, 12, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        decode_ops.add_rmsnorm(a, a, torch.randn(12, device="cuda"))  # FP32 weight
    with pytest.raises(ValueError):
        decode_ops.add_rmsnorm(a[:, :11].contiguous(), a[:, :11].contiguous(), a[0, :11].contiguous())
    with pytest.raises(ValueError):
        decode_ops.add_rmsnorm_linear(a, a, a[0], torch.randn(4, 12, device="cuda").bfloat16())  # K % 8
    with pytest.raises(ValueError):
        decode_ops.silu_mul_linear(torch.randn(2, 20, device="cuda").bfloat16(),
                                   torch.randn(4, 10, device="cuda").bfloat16())


def test_fused_add_rmsnorm_linear_rejects_in_place_update(native):
    """x_out over res or y (an in-place residual update) would let later CTAs read the
    updated x; the Python layer raises ValueError and the C ABI returns KLAB_E_INVALID."""
    from klab_b200 import decode_ops

    m, k, n = 1, 1024, 64
    res, y = torch.randn(m, k, device="cuda").bfloat16(), torch.randn(m, k, device="cuda").bfloat16()
    g = torch.rand(k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    for x_out in (res, y):
        with pytest.raises(ValueError):
            decode_ops.add_rmsnorm_linear(res, y, g, w, x_out=x_out)
    with pytest.raises(ValueError):
        decode_ops.add_rmsnorm_linear(res, y, g, w, out=res[:, :n])
    gu = torch.randn(m, 2 * k, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        decode_ops.silu_mul_linear(gu, w, out=gu[:, :n])
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    rc = native.lib().klab_add_rmsnorm_linear(res.data_ptr(), y.data_ptr(), g.data_ptr(), 1e-6, w.data_ptr(),
                                              out.data_ptr(), res.data_ptr(), m, n, k, None, 0, stream)
    assert rc == native.E_INVALID
    # the legal call still matches the standalone op followed by the projection
    x, ref = decode_ops.add_rmsnorm_linear(res, y, g, w)
    assert same_bits(x, res + y)
