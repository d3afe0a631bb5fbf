"""Parity at the five benchmark configurations, at their stated shapes and seeds,
through the same public entry points and launches the benchmark times.

Inputs come from torch's CPU generator (device-independent), seed 0 for the
weights; activations use the distribution each configuration states. Checks:
quantized codes, scales and lossless payloads bit-exact against the oracle;
projections inside the reference's check_outputs interval (projection_accuracy.py:
62-101: atol 1e-5 + rtol 1e-4 of FP64, BF16 outputs rounded into it) and within
one BF16 ulp of the FP64 result rounded once; lossless-coded outputs equal to
the raw BF16 projection of the same weights bit for bit; the 32-layer chain's
first two layers (Llama-3-8B projection shapes) against FP64 with the chain's
per-stage BF16 rounding, through the launch-per-stage chain and the persistent
one-launch chain. INT8 per-row and E2M1 run on every route (the default choice,
the warp-level tensor-core token tiles at every M, and the CUDA-core kernel), each
held to one ulp."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import codec as oc
from oracle import gemv as og
from oracle import quant as oq

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native():
    from klab_b200 import _native

    _native.lib()
    yield _native
    _native.set_option(_native.OPT_TENSOR, 1)
    assert _native.device_status(clear=True) == 0, "a kernel recorded a device-side error"


def normal(shape, std, gen):
    return torch.randn(shape, generator=gen, dtype=torch.float32) * std


def bits_of(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


def assert_one_ulp(ref64, y, what, ulps=1):
    report = ob.check_outputs(ref64, y.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= ulps, (what, report)
    return report


# ---------------------------------------------------------------- config 1

def test_c1_bf16_4096x4096_m1():
    """BF16 y = x.W^T, M=1, K=N=4096; x and W ~ N(0, 0.02^2), seed 0, rounded to BF16."""
    from klab_b200 import compressed_bf16 as cb

    gen = torch.Generator().manual_seed(0)
    w = normal((4096, 4096), 0.02, gen).bfloat16()
    x = normal((1, 4096), 0.02, gen).bfloat16()
    y = cb.raw_linear(x.cuda(), w.cuda(), threads=128, vector=8, output_dtype="bf16")
    ref = og.bf16_projection64(bits_of(x), bits_of(w))
    assert_one_ulp(ref, y, "c1")
    # FP32 output of the same launch: inside atol + rtol of FP64
    y32 = cb.raw_linear(x.cuda(), w.cuda(), threads=128, vector=8, output_dtype="fp32")
    assert ob.check_outputs(ref, y32.cpu().numpy(), output_dtype="fp32")["passed"]


# ---------------------------------------------------------------- config 2

@pytest.fixture(scope="module")
def c2_weights():
    from klab_b200 import int8_weights as i8

    gen = torch.Generator().manual_seed(0)
    w = normal((14336, 4096), 0.02, gen)
    q = i8.quantize_weights_per_row(w.cuda())
    codes, scales = oq.int8_quantize_row(w.numpy())
    np.testing.assert_array_equal(q.codes.cpu().numpy(), codes)
    np.testing.assert_array_equal(q.scales.cpu().numpy().view(np.uint32), scales.view(np.uint32))
    return q, oq.int8_dequantize(codes, scales)


@pytest.mark.parametrize("m", [1, 4, 16])
def test_c2_int8_per_row_14336x4096(native, c2_weights, m):
    """INT8 per-row weights (scale = max|row|/127, code = round(w/scale)), x ~ N(0, 1) BF16."""
    from klab_b200 import int8_weights as i8

    q, deq = c2_weights
    gen = torch.Generator().manual_seed(m)
    x = normal((m, 4096), 1.0, gen).bfloat16()
    ref = og.projection64(ob.bf16_values(bits_of(x)), deq)
    for route, name in ((1, "default route"), (3, "tensor-core token tile"), (0, "cuda cores")):
        native.set_option(native.OPT_TENSOR, route)
        try:
            y = i8.fused_linear(x.cuda(), q.codes, q.scales, output_dtype=torch.bfloat16)
        finally:
            native.set_option(native.OPT_TENSOR, 1)
        # The default route at M > 8 is tcgen05 (FP32 accumulation over the whole K in the
        # tensor core): inside the interval, near-zero outputs up to 2 BF16 ulps away.
        assert_one_ulp(ref, y, f"c2 m={m} {name}", ulps=2 if route == 1 and m > 8 else 1)


# ---------------------------------------------------------------- config 3

@pytest.mark.parametrize("m", [1, 8])
def test_c3_fp4_f16_scale_8192x8192(native, c3_weights, m):
    """E2M1 weights, FP16 scale per 32 K (max|group|/6), nearest-E2M1, low nibble = even k;
    x ~ N(0, 1) BF16."""
    q, deq = c3_weights
    gen = torch.Generator().manual_seed(10 + m)
    x = normal((m, 8192), 1.0, gen).bfloat16()
    ref = og.projection64(ob.bf16_values(bits_of(x)), deq)
    for route, name in ((1, "default route"), (3, "tensor-core token tile"), (0, "cuda cores")):
        native.set_option(native.OPT_TENSOR, route)
        try:
            y = q.linear(x.cuda(), output_dtype=torch.bfloat16)
        finally:
            native.set_option(native.OPT_TENSOR, 1)
        assert_one_ulp(ref, y, f"c3 m={m} {name}")


@pytest.fixture(scope="module")
def c3_weights():
    from klab_b200 import fp4

    gen = torch.Generator().manual_seed(0)
    w = normal((8192, 8192), 0.02, gen)
    q = fp4.quantize_weights_f16(w.cuda())
    packed, s16 = oq.fp4_quantize_f16(w.numpy())
    np.testing.assert_array_equal(q.packed.cpu().numpy(), packed)
    np.testing.assert_array_equal(q.scales.cpu().numpy().view(np.uint16), s16.view(np.uint16))
    deq = oq.fp4_dequantize_f16(packed, s16)
    np.testing.assert_array_equal(q.dequantize().cpu().numpy().view(np.uint32), deq.view(np.uint32))
    return q, deq


# ---------------------------------------------------------------- config 4

def test_c4_lossless_bf16_eight_layers():
    """Eight independent 4096 x 4096 BF16 layers (seeds 0..7) through the lossless codec:
    payload and metadata byte-exact against the oracle's packer, the GPU decode returns W
    bit for bit, and the coded projection equals the raw BF16 projection of the same W
    (config 1's path) bit for bit, within one ulp of FP64."""
    from klab_b200 import compressed_bf16 as cb

    x = normal((1, 4096), 1.0, torch.Generator().manual_seed(100)).bfloat16().cuda()
    for seed in range(8):
        w_bits = bits_of(normal((4096, 4096), 0.02, torch.Generator().manual_seed(seed)).bfloat16())
        mine, ref = cb.pack_bits(w_bits), oc.pack_bits(w_bits)
        np.testing.assert_array_equal(mine.metadata, ref.metadata)
        np.testing.assert_array_equal(mine.payload, ref.payload)
        packed = cb.upload(mine, "cuda")
        np.testing.assert_array_equal(bits_of(cb.unpack_weights(packed)), w_bits)
        coded = cb.fused_linear(x, packed, threads=128, vector=8, output_dtype="bf16")
        w = torch.from_numpy(w_bits.view(np.int16)).view(torch.bfloat16).cuda()
        raw = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
        assert same_bits(coded, raw), seed
        assert_one_ulp(og.bf16_projection64(bits_of(x), w_bits), coded, f"c4 layer {seed}")


# ---------------------------------------------------------------- config 5

def _up_of(chain):
    """The layer's up output after a step: plain BF16 in the launch chain, tagged
    words (tag << 16 | bf16) in the persistent chain's gather buffer."""
    if chain.persistent:
        return (chain.up_t & 0xFFFF).to(torch.int16).view(torch.bfloat16).view(1, -1).clone()
    return chain.up_full.clone()


def _check_layer(h_bits, entry, chain, down, what):
    """One chain layer in FP64 with the chain's rounding (every output rounded once to
    BF16): the stage-A outputs and up from the layer input h, down from the GPU's up."""
    for name, got in chain.a_out.items():
        assert_one_ulp(og.bf16_projection64(h_bits, bits_of(entry[name][0])), got, f"{what} {name}")
    up = _up_of(chain)
    assert_one_ulp(og.bf16_projection64(h_bits, bits_of(entry["up"][0])), up, f"{what} up")
    assert_one_ulp(og.bf16_projection64(bits_of(up), bits_of(entry["down"][0])), down, f"{what} down")


@pytest.mark.parametrize("persistent", [False, True])
def test_c5_chain_first_two_layers(native, persistent):
    """The 32-layer chain's layers 0 and 1 (same seeds as the benchmark's chain: the
    weights of layer i do not depend on the layer count) at Llama-3-8B shapes against
    FP64. Layer 0 is checked through a one-layer chain, layer 1 through a two-layer
    chain from the GPU's layer-0 output; the two chain modes agree bit for bit."""
    from klab_b200.chain import ChainShape, ProjectionChain

    x = normal((1, 4096), 1.0, torch.Generator().manual_seed(1234)).bfloat16().cuda()
    one = ProjectionChain(ChainShape(layers=1), seed=0, persistent=persistent)
    h1 = one.forward_eager(x).clone()
    _check_layer(bits_of(x), one.layers[0], one, h1, "layer 0")
    one.release()
    del one
    two = ProjectionChain(ChainShape(layers=2), seed=0, persistent=persistent)
    h2 = two.forward_eager(x).clone()
    _check_layer(bits_of(h1), two.layers[1], two, h2, "layer 1")
    other = ProjectionChain(ChainShape(layers=2), seed=0, persistent=not persistent)
    assert same_bits(other.forward_eager(x), h2)
    torch.cuda.synchronize()
    assert native.device_status() == 0
    two.release()
    other.release()
