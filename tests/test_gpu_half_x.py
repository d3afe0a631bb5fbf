"""FP16 staging of x for INT8 per-row and E2M1 weights.

BF16 activations are staged as FP16 after an exact per-token power-of-two
scaling when the token's exponent range allows it (the products then run as
fma.rn.f32.f16 on raw 16-bit pairs); otherwise the tile keeps BF16 staging and
the FP32 path. Both paths must give the same bits: a token computed alone (FP16
path) equals the same token inside a tile that a wide-range token forces onto
the FP32 path. Scaling x by a power of two scales the FP32 output exactly, and
wide-range, subnormal and non-finite tokens still meet the oracle's interval.
These are properties of the CUDA-core kernel: the module runs with the tensor-core
token tiles switched off (KLAB_OPT_TENSOR 0)."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og
from oracle import quant as oq

pytestmark = pytest.mark.gpu

FORMATS = ["int8_row", "fp4_f16", "fp4_e4m3"]


@pytest.fixture(scope="module", autouse=True)
def native():
    from klab_b200 import _native

    _native.lib()
    _native.set_option(_native.OPT_TENSOR, 0)
    yield _native
    _native.set_option(_native.OPT_TENSOR, 1)
    assert _native.device_status(clear=True) == 0, "a kernel recorded a device-side error"


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def make(fmt, n, k, seed):
    """(linear(x, out_dtype), dequantized FP32 weights) for one weight format."""
    from klab_b200 import fp4
    from klab_b200 import int8_weights as i8

    w = og.normal_f32(seed, (n, k), 0.02)
    if fmt == "int8_row":
        codes, scales = oq.int8_quantize_row(w)
        c, s = torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda()
        return (lambda x, o: i8.fused_linear(x, c, s, output_dtype=o)), oq.int8_dequantize(codes, scales)
    if fmt == "fp4_f16":
        packed, s16 = oq.fp4_quantize_f16(w)
        p, s = torch.from_numpy(packed).cuda(), torch.from_numpy(s16).cuda()
        return (lambda x, o: fp4.fused_linear(x, p, s, None, output_dtype=o)), oq.fp4_dequantize_f16(packed, s16)
    packed, scales, glob = oq.fp4_quantize_e4m3(w)
    p, s = torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda()
    g = torch.tensor(np.float32(glob), device="cuda")
    return (lambda x, o: fp4.fused_linear(x, p, s, g, output_dtype=o)), oq.fp4_dequantize_e4m3(packed, scales, glob)


def bf16_bits_of(values):
    return ob.round_bf16_bits(np.asarray(values, dtype=np.float64))


def wide_token(base, kind):
    """A copy of one token's bits that forces the FP32 path."""
    t = base.copy()
    if kind == "tiny":  # a nonzero value below 2^-88
        t[:2] = bf16_bits_of([1e-30, -3e-33])
    elif kind == "range":  # 34 binades between the smallest and largest value
        t[:2] = bf16_bits_of([2.0 ** -20, 2.0 ** 14])
    elif kind == "subnormal":
        t[0] = np.uint16(0x0003)
    elif kind == "huge":  # exponent field above 200
        t[0] = bf16_bits_of([2.0 ** 80])[0]
    return t


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("kind", ["tiny", "range", "subnormal", "huge"])
def test_fp16_path_equals_fp32_path(fmt, kind):
    n, k = 96, 4096
    linear, deq = make(fmt, n, k, 41)
    a = og.normal_bf16_bits(42, (1, k), 1.0)
    b = wide_token(a[0], kind)[None, :]
    alone = linear(dev_bf16(a), torch.float32)
    both = linear(dev_bf16(np.concatenate([a, b])), torch.float32)
    assert same_bits(both[0], alone[0])
    ref = og.projection64(ob.bf16_values(b), deq)
    report = ob.check_outputs(ref, both[1:].cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 8])
def test_mtile_with_one_wide_token(fmt, m):
    """Tokens of an 8-token tile that one wide token sends to the FP32 path keep
    the bits they have alone (FP16 path)."""
    n, k = 64, 8192
    linear, _ = make(fmt, n, k, 43)
    x = og.normal_bf16_bits(44, (8, k), 1.0)
    if m == 8:
        x[5] = wide_token(x[5], "range")
    tile = linear(dev_bf16(x), torch.float32)
    for t in range(8):
        if m == 8 and t == 5:
            continue
        assert same_bits(tile[t], linear(dev_bf16(x[t:t + 1]), torch.float32)[0]), t


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("shift", [-40, -7, 9, 60])
def test_power_of_two_scaling_is_exact(fmt, shift):
    n, k = 48, 2048
    linear, _ = make(fmt, n, k, 45)
    x = og.normal_bf16_bits(46, (2, k), 1.0)
    xs = bf16_bits_of(ob.bf16_values(x) * 2.0 ** shift)
    y = linear(dev_bf16(x), torch.float32).double()
    ys = linear(dev_bf16(xs), torch.float32).double()
    assert torch.equal(ys, y * 2.0 ** shift)


@pytest.mark.parametrize("fmt", FORMATS)
def test_bf16_output_and_zero_token(fmt):
    n, k = 80, 8192
    linear, deq = make(fmt, n, k, 47)
    x = og.normal_bf16_bits(48, (3, k), 1.0)
    x[1] = 0
    y = linear(dev_bf16(x), torch.bfloat16)
    ref = og.projection64(ob.bf16_values(x), deq)
    report = ob.check_outputs(ref, y.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report
    assert not y[1].float().abs().sum().item()


@pytest.mark.parametrize("fmt", FORMATS)
def test_nonfinite_token_propagates(fmt):
    n, k = 32, 1024
    linear, _ = make(fmt, n, k, 49)
    x = og.normal_bf16_bits(50, (2, k), 1.0)
    x[1, 3] = np.uint16(0x7f80)  # +inf
    y = linear(dev_bf16(x), torch.float32)
    assert torch.isfinite(y[0]).all()
    assert not torch.isfinite(y[1]).any()
    assert same_bits(y[0], linear(dev_bf16(x[:1]), torch.float32)[0])


@pytest.mark.parametrize("fmt", FORMATS)
def test_fp16_activations(fmt):
    n, k = 40, 4096
    linear, deq = make(fmt, n, k, 51)
    x32 = og.normal_f32(52, (4, k)).astype(np.float16)
    y = linear(torch.from_numpy(x32).cuda(), torch.float32)
    report = ob.check_outputs(og.projection64(x32.astype(np.float64), deq), y.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("xkind", ["normal", "range"])
def test_split_k_and_generic_fill_same_bits(native, fmt, xkind):
    """Split-K folds and the cooperative fill give the unsplit bulk-copy bits on
    both paths (the fold unscales after summing the chunk partials)."""
    n, k = 24, 16384
    linear, _ = make(fmt, n, k, 53)
    x = og.normal_bf16_bits(54, (2, k), 1.0)
    if xkind == "range":
        x[1] = wide_token(x[1], "range")
    results = []
    try:
        for split, generic in ((0, 0), (1, 0), (0, 1)):
            native.set_option(native.OPT_SPLIT, split)
            native.set_option(native.OPT_GENERIC, generic)
            results.append(linear(dev_bf16(x), torch.float32))
    finally:
        native.set_option(native.OPT_SPLIT, -1)
        native.set_option(native.OPT_GENERIC, 0)
    assert same_bits(results[1], results[0]) and same_bits(results[2], results[0])
