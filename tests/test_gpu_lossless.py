"""Lossless FP32 formats on the GPU: the B200 packers produce the reference
packers' bytes (pinned through the oracle and tests/golden/reference_lossless.npz),
the unpack kernels restore every bit, and the projections are bit-identical to
the FP32 projection of the unpacked weights (and within the reference's FP32
tolerance, atol 1e-5 + rtol 1e-4 of the FP64 result, on finite data)."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og
from oracle import lossless as ol

pytestmark = pytest.mark.gpu
CASES = ("mixed", "normal", "wide")


@pytest.fixture(scope="module")
def golden():
    from pathlib import Path

    return np.load(Path(__file__).resolve().parent / "golden" / "reference_lossless.npz")


def _weights(golden, name):
    if name in CASES:
        return golden[f"{name}__w"]
    rng = np.random.default_rng(7)
    w = rng.standard_normal((300, 2112), dtype=np.float32) * np.float32(0.02)   # 2 full chunks + 64 columns
    w[5, 1000:1064] *= np.float32(2.0 ** 40)                                     # a wide block mid-row
    return w


@pytest.mark.parametrize("name", CASES + ("ragged",))
def test_pack_bytes_and_unpack_bits(golden, name):
    from klab_b200 import lossless_weights as lw
    from klab_b200 import packed_fp32 as pf

    w = _weights(golden, name)
    wd = torch.from_numpy(w).cuda()
    v1 = lw.pack_weights(wd)
    m, e, meta = ol.lf32_pack(w)
    np.testing.assert_array_equal(v1.mantissa.cpu().numpy(), m)
    np.testing.assert_array_equal(v1.exponents.cpu().numpy(), e)
    np.testing.assert_array_equal(v1.metadata.cpu().numpy(), meta)
    np.testing.assert_array_equal(v1.unpack().cpu().numpy().view(np.uint32), w.view(np.uint32))
    p28 = pf.pack_weights(wd)
    payload, meta28 = ol.fp28_pack(w)
    np.testing.assert_array_equal(p28.payload.cpu().numpy(), payload)
    np.testing.assert_array_equal(p28.metadata.cpu().numpy(), meta28)
    np.testing.assert_array_equal(p28.unpack().cpu().numpy().view(np.uint32), w.view(np.uint32))
    if name in CASES:
        np.testing.assert_array_equal(m, golden[f"{name}__lf32_mantissa"])
        np.testing.assert_array_equal(payload, golden[f"{name}__fp28_payload"])
    assert v1.storage_bytes < w.nbytes or name == "wide"


@pytest.mark.parametrize("name", ("normal", "ragged", "wide"))
@pytest.mark.parametrize("m", [1, 3, 8])
def test_lossless_linear_equals_fp32_projection(golden, name, m):
    from klab_b200 import _native
    from klab_b200 import lossless_weights as lw
    from klab_b200 import packed_fp32 as pf

    w = _weights(golden, name)
    n, k = w.shape
    x = np.random.default_rng(m + k).standard_normal((m, k)).astype(np.float32)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    plain = torch.empty(m, n, device="cuda", dtype=torch.float32)
    _native.gemv(_native.W_F32, _native.DT_F32, xd, wd, None, None, plain, _native.DT_F32, m, n, k)
    y1 = lw.fused_linear(xd, lw.pack_weights(wd))
    y2 = pf.fused_linear(xd, pf.pack_weights(wd))
    y3 = torch.ops.kernel_lab.lossless_linear(xd, *lw.pack_weights(wd).__dict__.values())
    torch.cuda.synchronize()
    for y in (y1, y2, y3):
        assert torch.equal(y.view(torch.int32), plain.view(torch.int32))
    ref = og.projection64(x.astype(np.float64), w.astype(np.float64))
    report = ob.check_outputs(ref, y1.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


def test_non_finite_weights_decode_and_propagate(golden):
    """Infinities, NaN and -0 survive packing; the projection matches FP32 bit for bit."""
    from klab_b200 import _native
    from klab_b200 import packed_fp32 as pf

    w = golden["mixed__w"]
    n, k = w.shape
    wd = torch.from_numpy(w).cuda()
    xd = torch.ones(2, k, device="cuda")
    plain = torch.empty(2, n, device="cuda")
    _native.gemv(_native.W_F32, _native.DT_F32, xd, wd, None, None, plain, _native.DT_F32, 2, n, k)
    y = pf.fused_linear(xd, pf.pack_weights(wd))
    torch.cuda.synchronize()
    assert torch.equal(torch.isnan(y), torch.isnan(plain))
    finite = ~torch.isnan(plain)
    assert torch.equal(y[finite].view(torch.int32), plain[finite].view(torch.int32))


def test_validation_matches_reference_errors():
    from klab_b200 import lossless_weights as lw
    from klab_b200 import packed_fp32 as pf

    w = torch.randn(8, 128, device="cuda")
    with pytest.raises(ValueError):
        lw.pack_weights(torch.randn(8, 100, device="cuda"))           # K % 64
    with pytest.raises(ValueError):
        pf.pack_weights(w.cpu())                                       # not CUDA
    packed = lw.pack_weights(w)
    with pytest.raises(ValueError):
        lw.fused_linear(torch.randn(2, 128, device="cuda", dtype=torch.float16), packed)
    with pytest.raises(ValueError):
        lw.fused_linear(torch.randn(2, 64, device="cuda"), packed)
    with pytest.raises(ValueError):
        lw.fused_linear(torch.randn(2, 128, device="cuda"), packed, threads=96)
    p28 = pf.pack_weights(w)
    with pytest.raises(ValueError):
        pf.fused_linear(torch.randn(2, 128, device="cuda"), pf.PackedFP32Weights(p28.payload.float(), p28.metadata))
