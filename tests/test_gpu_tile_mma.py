"""Warp-level tensor-core token tiles (tile_mma.cu) for INT8 per-row and E2M1 weights
with FP16 scales per 32 (the default route at M = 2..8 / 2..16). The module runs them at
every M <= 16 (KLAB_OPT_TENSOR 3), so that M = 1 exercises the same kernel.

Against the FP64 oracle: every output inside the reference's check_outputs interval
(atol 1e-5 + rtol 1e-4 of FP64, BF16 rounded into it) and within one BF16 ulp; FP32
outputs inside atol + rtol (FP16 operands, FP32 accumulation). Invariants (bit for bit): a token alone equals the same
token in any tile (M = 1..16), a row shard equals the full projection, and repeated
calls and CUDA-graph replays give the same bits (tickets reset themselves). Ragged N (partial 16-row groups), K that ends inside a phase, FP16 x,
zero, tiny, huge and wide-range tokens are covered. The CUDA-core kernel stays
reachable (KLAB_OPT_TENSOR 0) and meets the same oracle bound."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og
from oracle import quant as oq

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native():
    from klab_b200 import _native

    _native.lib()
    _native.set_option(_native.OPT_TENSOR, 3)
    yield _native
    _native.set_option(_native.OPT_TENSOR, 1)
    assert _native.device_status(clear=True) == 0, "a kernel recorded a device-side error"


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def make(fmt, n, k, seed):
    """(linear(x, out_dtype, out=None), dequantized FP32 weights as numpy)."""
    from klab_b200 import fp4
    from klab_b200 import int8_weights as i8

    w = og.normal_f32(seed, (n, k), 0.02)
    if fmt == "int8_row":
        codes, scales = oq.int8_quantize_row(w)
        c, s = torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda()
        return (lambda x, o, out=None: i8.fused_linear(x, c, s, output_dtype=o, out=out),
                oq.int8_dequantize(codes, scales))
    packed, s16 = oq.fp4_quantize_f16(w)
    p, s = torch.from_numpy(packed).cuda(), torch.from_numpy(s16).cuda()
    return (lambda x, o, out=None: fp4.fused_linear(x, p, s, None, output_dtype=o, out=out),
            oq.fp4_dequantize_f16(packed, s16))


FORMATS = ["int8_row", "fp4_f16"]
SHAPES = [(1, 96, 4096), (3, 100, 2048), (8, 64, 8192), (16, 48, 1024), (5, 33, 3072), (9, 200, 6144),
          (2, 16, 256), (12, 1000, 2304), (1, 4100, 2560)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matches_oracle_bf16_and_fp32(fmt, m, n, k):
    lin, deq = make(fmt, n, k, n + k)
    x_bits = og.normal_bf16_bits(m * 7 + k, (m, k), 1.0)
    ref = og.projection64(ob.bf16_values(x_bits), deq)
    x = dev_bf16(x_bits)
    y = lin(x, torch.bfloat16)
    report = ob.check_outputs(ref, y.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report
    y32 = lin(x, torch.float32)
    assert ob.check_outputs(ref, y32.cpu().numpy(), output_dtype="fp32")["passed"]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("k", [4096, 2048])
def test_token_alone_equals_token_in_tile(fmt, k):
    n = 80
    lin, _ = make(fmt, n, k, 5)
    x_all = dev_bf16(og.normal_bf16_bits(6, (16, k), 1.0))
    singles = torch.cat([lin(x_all[i:i + 1].contiguous(), torch.float32) for i in range(16)])
    for m in (2, 3, 5, 8, 9, 15, 16):
        y = lin(x_all[:m].contiguous(), torch.float32)
        assert same_bits(y, singles[:m]), m


@pytest.mark.parametrize("fmt", FORMATS)
def test_row_shards_bit_identical(fmt):
    from klab_b200 import fp4
    from klab_b200 import int8_weights as i8

    n, k = 512, 4096
    w = og.normal_f32(8, (n, k), 0.02)
    x = dev_bf16(og.normal_bf16_bits(9, (4, k), 1.0))
    if fmt == "int8_row":
        codes, scales = (torch.from_numpy(a).cuda() for a in oq.int8_quantize_row(w))
        run = lambda r0, r1: i8.fused_linear(x, codes[r0:r1].contiguous(), scales[r0:r1].contiguous(),  # noqa
                                             output_dtype=torch.bfloat16)
    else:
        packed, s16 = (torch.from_numpy(a).cuda() for a in oq.fp4_quantize_f16(w))
        run = lambda r0, r1: fp4.fused_linear(x, packed[r0:r1].contiguous(), s16[r0:r1].contiguous(), None,  # noqa
                                              output_dtype=torch.bfloat16)
    full = run(0, n)
    for g in (2, 4, 8):
        part = n // g
        for r in range(g):
            assert same_bits(run(r * part, (r + 1) * part), full[:, r * part:(r + 1) * part]), (g, r)


@pytest.mark.parametrize("fmt", FORMATS)
def test_without_workspace_the_cuda_cores_take_the_launch(native, fmt):
    """The token tiles keep phase partials in the workspace; a call without one runs on the
    CUDA cores, which meet the same oracle bound."""
    m, n, k = 4, 300, 8192
    w = og.normal_f32(21, (n, k), 0.02)
    x_bits = og.normal_bf16_bits(22, (m, k), 1.0)
    x = dev_bf16(x_bits)
    out = torch.empty(m, n, device="cuda")
    if fmt == "int8_row":
        codes, scales = oq.int8_quantize_row(w)
        deq = oq.int8_dequantize(codes, scales)
        native.gemv(native.W_I8_ROW, native.DT_BF16, x, torch.from_numpy(codes).cuda(),
                    torch.from_numpy(scales).cuda(), None, out, native.DT_F32, m, n, k, workspace=False)
    else:
        packed, s16 = oq.fp4_quantize_f16(w)
        deq = oq.fp4_dequantize_f16(packed, s16)
        native.gemv(native.W_FP4_G32H, native.DT_BF16, x, torch.from_numpy(packed).cuda(),
                    torch.from_numpy(s16).cuda(), None, out, native.DT_F32, m, n, k, workspace=False)
    ref = og.projection64(ob.bf16_values(x_bits), deq)
    assert ob.check_outputs(ref, out.cpu().numpy(), output_dtype="fp32")["passed"]


@pytest.mark.parametrize("fmt", FORMATS)
def test_repeated_calls_and_graph_replay(fmt):
    """Split row groups: the per-group tickets reset themselves, so every call and every
    graph replay returns the same bits."""
    m, n, k = 4, 300, 8192
    lin, _ = make(fmt, n, k, 11)
    x = dev_bf16(og.normal_bf16_bits(12, (m, k), 1.0))
    first = lin(x, torch.bfloat16).clone()
    for _ in range(3):
        assert same_bits(lin(x, torch.bfloat16), first)
    out = torch.empty_like(first)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        lin(x, torch.bfloat16, out=out)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):   # the stream whose workspace the warm-up created
        lin(x, torch.bfloat16, out=out)
    for _ in range(4):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert same_bits(out, first)


@pytest.mark.parametrize("fmt", FORMATS)
def test_fp16_activations(fmt):
    m, n, k = 6, 130, 4096
    lin, deq = make(fmt, n, k, 13)
    x = torch.from_numpy(og.normal_f32(14, (m, k))).to(torch.float16).cuda()
    ref = og.projection64(x.double().cpu().numpy(), deq)
    report = ob.check_outputs(ref, lin(x, torch.bfloat16).float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


@pytest.mark.parametrize("fmt", FORMATS)
def test_zero_tiny_huge_and_wide_tokens(fmt):
    """Token 0 all zero (exact zero out), token 1 scaled by 2^-100, token 2 by 2^+60,
    token 3 spanning 40 binades: all inside the oracle's interval."""
    m, n, k = 4, 64, 2048
    lin, deq = make(fmt, n, k, 15)
    x32 = og.normal_f32(16, (m, k))
    x32[0] = 0.0
    x32[1] *= np.float32(2.0 ** -100)
    x32[2] *= np.float32(2.0 ** 60)
    x32[3, ::7] *= np.float32(2.0 ** -40)
    x_bits = ob.f32_to_bf16_bits(x32)
    ref = og.projection64(ob.bf16_values(x_bits), deq)
    y = lin(dev_bf16(x_bits), torch.float32)
    assert torch.equal(y[0], torch.zeros_like(y[0]))
    report = ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


@pytest.mark.parametrize("fmt", FORMATS)
def test_cuda_core_route_still_meets_the_oracle(native, fmt):
    m, n, k = 8, 72, 4096
    lin, deq = make(fmt, n, k, 17)
    x_bits = og.normal_bf16_bits(18, (m, k), 1.0)
    ref = og.projection64(ob.bf16_values(x_bits), deq)
    native.set_option(native.OPT_TENSOR, 0)
    try:
        y = lin(dev_bf16(x_bits), torch.bfloat16)
    finally:
        native.set_option(native.OPT_TENSOR, 3)
    report = ob.check_outputs(ref, y.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


@pytest.mark.parametrize("fmt", FORMATS)
def test_unaligned_x_uses_16_bit_staging(fmt):
    """x starting 2 bytes past a 16-byte boundary (a contiguous view at storage offset 1):
    the tiles stage it with 16-bit loads and meet the same oracle bound."""
    m, n, k = 3, 90, 2048
    lin, deq = make(fmt, n, k, 19)
    x_bits = og.normal_bf16_bits(20, (m, k), 1.0)
    flat = torch.empty(m * k + 8, dtype=torch.bfloat16, device="cuda")
    x = flat[1:1 + m * k].view(m, k)
    x.copy_(dev_bf16(x_bits))
    assert x.data_ptr() % 16 == 2 and x.is_contiguous()
    ref = og.projection64(ob.bf16_values(x_bits), deq)
    report = ob.check_outputs(ref, lin(x, torch.bfloat16).float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report
