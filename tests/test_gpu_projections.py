"""GPU parity of every projection format against the CPU oracle, plus the
bit-identity invariants of the B200 kernels (coded == raw, any M-tile == M=1,
column shard == full, split-K == no split, bulk-copy fill == cooperative fill).
Tolerance: the reference's check_outputs interval (atol 1e-5 + rtol 1e-4 of the
FP64 reference, BF16 outputs rounded into it) and at most 1 BF16 ulp."""

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
    assert _native.device_status(clear=True) == 0, "a kernel recorded a device-side error"


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def host_bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def options(native, split=-1, generic=0):
    native.set_option(native.OPT_SPLIT, split)
    native.set_option(native.OPT_GENERIC, generic)


@pytest.fixture(autouse=True)
def reset_options(native):
    yield
    options(native)


SHAPES = [(1, 257, 4096), (1, 64, 2048), (3, 130, 1024), (1, 33, 4352), (2, 17, 6144)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("out", ["bf16", "fp32"])
def test_raw_bf16_matches_oracle(m, n, k, out):
    from klab_b200 import compressed_bf16 as cb

    x_bits = og.normal_bf16_bits(m * 7 + k, (m, k), 1.0)
    w_bits = og.normal_bf16_bits(n * 3 + k, (n, k), 0.02)
    y = cb.raw_linear(dev_bf16(x_bits), dev_bf16(w_bits), threads=128, vector=8, output_dtype=out)
    ref = og.bf16_projection64(x_bits, w_bits)
    report = ob.check_outputs(ref, y.float().cpu().numpy(), output_dtype=out)
    assert report["passed"], report
    if out == "bf16":
        assert report["max_ulp_error"] <= 1, report


@pytest.mark.parametrize("m,n,k", [(1, 96, 4096), (4, 40, 2048), (1, 31, 320), (8, 9, 8192)])
def test_coded_equals_raw_and_unpacks_exactly(m, n, k):
    from klab_b200 import compressed_bf16 as cb

    w_bits = og.normal_bf16_bits(k + n, (n, k), 0.02)
    w_bits[0, :64] = np.arange(64, dtype=np.uint16) << 7   # raw block
    w_bits[min(2, n - 1), 64:70] = [0x0000, 0x8000, 0x0001, 0x8001, 0x3F80, 0x0080]
    packed = cb.upload(cb.pack_bits(w_bits), "cuda")
    np.testing.assert_array_equal(host_bits(cb.unpack_weights(packed)), w_bits)
    x = dev_bf16(og.normal_bf16_bits(k, (m, k), 1.0))
    for out in ("bf16", "fp32"):
        coded = cb.fused_linear(x, packed, threads=128, vector=8, output_dtype=out)
        raw = cb.raw_linear(x, dev_bf16(w_bits), threads=128, vector=8, output_dtype=out)
        assert same_bits(coded, raw)
        report = ob.check_outputs(og.bf16_projection64(host_bits(x), w_bits), coded.float().cpu().numpy(),
                                  output_dtype=out)
        assert report["passed"], report


def test_cpu_codec_matches_oracle():
    from klab_b200 import compressed_bf16 as cb

    bits = np.arange(65536, dtype=np.uint16).reshape(1024, 64)
    mine, ref = cb.pack_bits(bits), oc.pack_bits(bits)
    np.testing.assert_array_equal(mine.metadata, ref.metadata)
    np.testing.assert_array_equal(mine.payload, ref.payload)
    np.testing.assert_array_equal(cb.unpack_bits(mine), bits)


def test_all_weight_patterns_coded_vs_raw_bits():
    """Every BF16 pattern as a weight (NaN, inf, subnormals included): coded and raw
    projections agree bit for bit (verify_compressed.py:179-182)."""
    from klab_b200 import compressed_bf16 as cb

    w_bits = np.arange(65536, dtype=np.uint16).reshape(1024, 64)
    x = dev_bf16(og.normal_bf16_bits(1, (3, 64), 1.0))
    packed = cb.upload(cb.pack_bits(w_bits), "cuda")
    for out in ("bf16", "fp32"):
        a = cb.fused_linear(x, packed, threads=128, vector=8, output_dtype=out)
        b = cb.raw_linear(x, dev_bf16(w_bits), threads=128, vector=8, output_dtype=out)
        assert same_bits(a, b)


def test_no_ftz_single_rne_known_answers():
    """verify_compressed.py:213-235: x = [1, 1, 0, ...]."""
    from klab_b200 import compressed_bf16 as cb

    w_bits = np.zeros((3, 64), dtype=np.uint16)
    w_bits[0, 0] = 0x0001
    w_bits[1], w_bits[1, 1] = 0x3F80, 0x3B80
    w_bits[2], w_bits[2, 1] = 0x3F81, 0x3B80
    w_bits[1, 2:] = 0
    w_bits[2, 2:] = 0
    x_bits = np.zeros((1, 64), dtype=np.uint16)
    x_bits[0, :2] = 0x3F80
    packed = cb.upload(cb.pack_bits(w_bits), "cuda")
    for fn in (lambda o: cb.fused_linear(dev_bf16(x_bits), packed, threads=32, vector=2, output_dtype=o),
               lambda o: cb.raw_linear(dev_bf16(x_bits), dev_bf16(w_bits), threads=32, vector=2, output_dtype=o)):
        f32 = fn("fp32").view(torch.int32).cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(f32, [[0x00010000, 0x3F808000, 0x3F818000]])
        b16 = host_bits(fn("bf16"))
        np.testing.assert_array_equal(b16, [[0x0001, 0x3F80, 0x3F82]])


@pytest.mark.parametrize("k", [4096, 1024])
@pytest.mark.parametrize("max_tile", [4, 8])
def test_mtile_tokens_bit_identical_to_single_token(native, k, max_tile):
    from klab_b200 import compressed_bf16 as cb

    n = 72
    w = dev_bf16(og.normal_bf16_bits(5, (n, k), 0.02))
    x_all = dev_bf16(og.normal_bf16_bits(6, (17, k), 1.0))
    singles = torch.cat([cb.raw_linear(x_all[i:i + 1], w, threads=128, vector=8, output_dtype="bf16")
                         for i in range(17)])
    native.set_option(native.OPT_MAX_TILE, max_tile)
    try:
        for m in (2, 3, 4, 5, 7, 8, 9, 15, 16, 17):
            y = cb.raw_linear(x_all[:m].contiguous(), w, threads=128, vector=8, output_dtype="bf16")
            assert same_bits(y, singles[:m]), m
    finally:
        native.set_option(native.OPT_MAX_TILE, 4)


def test_column_shards_bit_identical():
    from klab_b200 import compressed_bf16 as cb

    n, k = 1024, 4096
    w = dev_bf16(og.normal_bf16_bits(8, (n, k), 0.02))
    x = dev_bf16(og.normal_bf16_bits(9, (1, k), 1.0))
    full = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
    for g in (2, 4, 8):
        part = n // g
        for r in range(g):
            shard = cb.raw_linear(x, w[r * part:(r + 1) * part].contiguous(), threads=128, vector=8,
                                  output_dtype="bf16")
            assert same_bits(shard, full[:, r * part:(r + 1) * part]), (g, r)


@pytest.mark.parametrize("m,n,k", [(1, 40, 14336), (1, 7, 4096), (4, 20, 8192), (1, 300, 10240)])
def test_split_k_and_generic_fill_bit_identical(native, m, n, k):
    from klab_b200 import compressed_bf16 as cb

    w = dev_bf16(og.normal_bf16_bits(10, (n, k), 0.02))
    x = dev_bf16(og.normal_bf16_bits(11, (m, k), 1.0))
    results = {}
    for split, generic in ((0, 0), (1, 0), (0, 1), (1, 1)):
        options(native, split, generic)
        results[(split, generic)] = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="fp32")
        torch.cuda.synchronize()
    base = results[(0, 0)]
    for key, value in results.items():
        assert same_bits(value, base), key
    report = ob.check_outputs(og.bf16_projection64(host_bits(x), host_bits(w)), base.cpu().numpy(),
                              output_dtype="fp32")
    assert report["passed"], report


def test_split_k_replays_in_cuda_graph(native):
    """The self-resetting tickets keep the split kernel replayable."""
    from klab_b200 import compressed_bf16 as cb

    options(native, 1, 0)
    n, k = 24, 14336
    w = dev_bf16(og.normal_bf16_bits(12, (n, k), 0.02))
    x = dev_bf16(og.normal_bf16_bits(13, (1, k), 1.0))
    eager = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="fp32")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        cb.raw_linear(x, w, threads=128, vector=8, output_dtype="fp32")
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="fp32")
    for _ in range(5):
        graph.replay()
        torch.cuda.synchronize()
        assert same_bits(out, eager)


def test_ragged_and_misaligned_raw_use_generic_path():
    """K not a multiple of 8 (the reference's vector=2 contract) and misaligned views."""
    from klab_b200 import compressed_bf16 as cb

    for m, n, k in ((2, 5, 12), (1, 9, 1030), (3, 4, 2)):
        x_bits = og.normal_bf16_bits(k, (m, k), 1.0)
        w_bits = og.normal_bf16_bits(k + 1, (n, k), 0.02)
        for out in ("bf16", "fp32"):
            y = cb.raw_linear(dev_bf16(x_bits), dev_bf16(w_bits), threads=32, vector=2, output_dtype=out)
            report = ob.check_outputs(og.bf16_projection64(x_bits, w_bits), y.float().cpu().numpy(),
                                      output_dtype=out)
            assert report["passed"], (m, n, k, report)


def test_compressed_linear_op_and_graph_capture():
    from klab_b200 import compressed_bf16 as cb

    n, k = 131, 192
    w_bits = og.normal_bf16_bits(3, (n, k), 0.02)
    packed = cb.upload(cb.pack_bits(w_bits), "cuda")
    x = dev_bf16(og.normal_bf16_bits(4, (3, k), 1.0))
    eager = packed.linear(x, threads=128, vector=8, output_dtype="bf16")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = packed.linear(x, threads=128, vector=8, output_dtype="bf16")
    graph.replay()
    torch.cuda.synchronize()
    assert same_bits(captured, eager)


def test_guards_match_reference_errors():
    from klab_b200 import compressed_bf16 as cb

    w = dev_bf16(og.normal_bf16_bits(1, (8, 64), 0.02))
    x = dev_bf16(og.normal_bf16_bits(2, (1, 64), 1.0))
    with pytest.raises(ValueError):
        cb.raw_linear(x, w, threads=96, vector=8, output_dtype="bf16")
    with pytest.raises(ValueError):
        cb.raw_linear(x, w, threads=128, vector=8, output_dtype="fp16")
    with pytest.raises(ValueError):
        cb.raw_linear(x.float(), w, threads=128, vector=8, output_dtype="bf16")
    out = torch.empty((1, 8), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16", out=w[:1, :8])
    cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16", out=out)


# ---------------------------------------------------------------- INT8

@pytest.mark.parametrize("xdtype", [torch.float16, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,k", [(5, 64), (65, 256), (17, 512), (40, 4096), (3, 8192)])
def test_int8_reference_format(xdtype, n, k):
    from klab_b200 import int8_weights as i8

    w = og.normal_f32(n + k, (n, k), 1.0)
    q = i8.quantize_weights(torch.from_numpy(w).cuda())
    codes, scales = oq.int8_quantize_g64(w)
    np.testing.assert_array_equal(q.codes.cpu().numpy(), codes)
    np.testing.assert_array_equal(q.scales.cpu().numpy().view(np.uint32), scales.view(np.uint32))
    deq = oq.int8_dequantize(codes, scales)
    np.testing.assert_array_equal(q.dequantize().cpu().numpy().view(np.uint32), deq.view(np.uint32))
    x32 = (og.normal_f32(7, (3, k)) / np.float32(np.sqrt(k))).astype(np.float32)
    x = torch.from_numpy(x32).to(xdtype).cuda()
    y = i8.fused_linear(x, q.codes, q.scales)
    ref = og.projection64(x.double().cpu().numpy(), deq)
    report = ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


@pytest.mark.parametrize("m", [1, 4, 16])
def test_int8_per_row_bf16(m):
    from klab_b200 import int8_weights as i8

    n, k = 96, 4096
    w = og.normal_f32(21, (n, k), 0.02)
    q = i8.quantize_weights_per_row(torch.from_numpy(w).cuda())
    codes, scales = oq.int8_quantize_row(w)
    np.testing.assert_array_equal(q.codes.cpu().numpy(), codes)
    np.testing.assert_array_equal(q.scales.cpu().numpy().view(np.uint32), scales.view(np.uint32))
    x_bits = og.normal_bf16_bits(22, (m, k), 1.0)
    y = i8.fused_linear(dev_bf16(x_bits), q.codes, q.scales, output_dtype=torch.bfloat16)
    ref = og.projection64(ob.bf16_values(x_bits), oq.int8_dequantize(codes, scales))
    report = ob.check_outputs(ref, y.float().cpu().numpy(), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


def test_int8_zero_weights_exact_zero():
    from klab_b200 import int8_weights as i8

    q = i8.quantize_weights(torch.zeros(5, 64, device="cuda"))
    y = q.linear(torch.ones(1, 64, device="cuda"))
    assert torch.equal(y, torch.zeros(1, 5, device="cuda"))


# ---------------------------------------------------------------- FP4

def test_fp4_e2m1_table_known_answer():
    """bench_fp4.py:21-31: identity activations recover the E2M1 table."""
    from klab_b200 import fp4

    table = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], device="cuda")
    codes = torch.arange(16, dtype=torch.uint8, device="cuda").reshape(1, 16)
    packed = (codes[:, ::2] | (codes[:, 1::2] << 4)).contiguous()
    q = fp4.FP4Weights(packed, torch.tensor([[56]], dtype=torch.uint8, device="cuda"), torch.ones((), device="cuda"))
    np.testing.assert_array_equal(q.dequantize()[0].cpu().numpy(), table.cpu().numpy())
    x = torch.eye(16, device="cuda")
    for dtype in (torch.float16, torch.float32, torch.bfloat16):
        y = fp4.fused_linear(x.to(dtype), q.packed, q.scales, q.global_scale)
        assert torch.equal(y[:, 0], table), dtype


@pytest.mark.parametrize("xdtype", [torch.float16, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,k", [(5, 16), (65, 256), (17, 512), (24, 8192), (9, 1040)])
def test_fp4_reference_format(xdtype, n, k):
    from klab_b200 import fp4

    w = og.normal_f32(n * 5 + k, (n, k), 1.0)
    q = fp4.quantize_weights(torch.from_numpy(w).cuda())
    packed, scales, glob = oq.fp4_quantize_e4m3(w)
    np.testing.assert_array_equal(q.packed.cpu().numpy(), packed)
    np.testing.assert_array_equal(q.scales.cpu().numpy(), scales)
    deq = oq.fp4_dequantize_e4m3(packed, scales, glob)
    np.testing.assert_array_equal(q.dequantize().cpu().numpy().view(np.uint32), deq.view(np.uint32))
    x32 = (og.normal_f32(9, (3, k)) / np.float32(np.sqrt(k))).astype(np.float32)
    x = torch.from_numpy(x32).to(xdtype).cuda()
    y = fp4.fused_linear(x, q.packed, q.scales, q.global_scale)
    report = ob.check_outputs(og.projection64(x.double().cpu().numpy(), deq), y.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


@pytest.mark.parametrize("m", [1, 8])
def test_fp4_f16_scale_format_bf16(m):
    from klab_b200 import fp4

    n, k = 64, 8192
    w = og.normal_f32(31, (n, k), 0.02)
    q = fp4.quantize_weights_f16(torch.from_numpy(w).cuda())
    packed, s16 = oq.fp4_quantize_f16(w)
    np.testing.assert_array_equal(q.packed.cpu().numpy(), packed)
    np.testing.assert_array_equal(q.scales.cpu().numpy().view(np.uint16), s16.view(np.uint16))
    deq = oq.fp4_dequantize_f16(packed, s16)
    np.testing.assert_array_equal(q.dequantize().cpu().numpy().view(np.uint32), deq.view(np.uint32))
    x_bits = og.normal_bf16_bits(32, (m, k), 1.0)
    y = q.linear(dev_bf16(x_bits), output_dtype=torch.bfloat16)
    report = ob.check_outputs(og.projection64(ob.bf16_values(x_bits), deq), y.float().cpu().numpy(),
                              output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


def test_fp4_zero_and_subnormal():
    from klab_b200 import fp4

    zero = fp4.quantize_weights(torch.zeros(5, 16, device="cuda"))
    assert torch.equal(zero.linear(torch.ones(1, 16, device="cuda")), torch.zeros(1, 5, device="cuda"))
    tiny = fp4.quantize_weights(torch.full((5, 16), 1e-40, device="cuda"))
    assert torch.isfinite(tiny.dequantize()).all()


# ---------------------------------------------------------------- FP16 / FP32

@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_linear_fp32_out(dtype):
    from klab_b200 import half_projection as hp

    m, n, k = 3, 130, 4096
    x = torch.from_numpy(og.normal_f32(1, (m, k))).to(dtype).cuda()
    w = torch.from_numpy(og.normal_f32(2, (n, k), 0.02)).to(dtype).cuda()
    y = hp.linear(x, w)
    ref = og.projection64(x.double().cpu().numpy(), w.double().cpu().numpy())
    assert ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")["passed"]


@pytest.mark.parametrize("m,n,k", [(1, 300, 1024), (4, 33, 4096), (2, 7, 13)])
def test_fp32_matmul(m, n, k):
    from klab_b200 import kernel_lab

    x = torch.from_numpy(og.normal_f32(1, (m, k)) / np.float32(np.sqrt(k))).cuda()
    w = torch.from_numpy(og.normal_f32(2, (n, k))).cuda()
    y = kernel_lab.matmul(x, w)
    ref = og.projection64(x.double().cpu().numpy(), w.double().cpu().numpy())
    assert ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")["passed"]


# ---------------------------------------------------------------- prefetch / driver ABI

def test_prefetch_never_writes_and_driver_abi_path():
    from klab_b200 import l2prefetch

    t = torch.randn(1 << 20, device="cuda")
    before = t.clone()
    for kernel in ("l2_hint", "l2_hint_last", "l2_load", "l2_bulk"):
        l2prefetch.prefetch(t, blocks=4, kernel=kernel, stride=32)
        l2prefetch.prefetch(t, blocks=2, kernel=kernel, nbytes=4096)
    # bulk requests: clamped request sizes, an unaligned start and a length under 16 bytes
    b = t.view(torch.uint8)
    for stride, lo, n in ((1 << 20, 0, b.numel()), (17, 3, 100_001), (65536, 5, 9), (16, 0, 0)):
        l2prefetch.prefetch(b[lo:lo + n] if n else b[:1], blocks=3, kernel="l2_bulk", stride=stride, threads=32,
                            nbytes=n)
    import ctypes as ct
    mod = l2prefetch.module()
    sink = torch.zeros(1, dtype=torch.int32, device="cuda")
    for kernel in ("l2_hint", "l2_hint_last", "l2_load", "l2_bulk"):
        mod.launch(kernel, (8, 1), 256, t, ct.c_longlong(t.numel() * 4), ct.c_int(128), sink)
    torch.cuda.synchronize()
    assert torch.equal(t, before)
    assert int(sink.item()) == 0


# ---------------------------------------------------------------- multi-segment launches / chain

@pytest.mark.parametrize("m,split", [(1, 0), (1, 1), (3, 0)])
def test_multi_segment_equals_separate_launches(native, m, split):
    from klab_b200 import _native as nat
    from klab_b200 import compressed_bf16 as cb

    options(native, split, 0)
    k = 6144
    sizes = (96, 32, 8, 200)
    ws = [dev_bf16(og.normal_bf16_bits(40 + i, (n, k), 0.02)) for i, n in enumerate(sizes)]
    x = dev_bf16(og.normal_bf16_bits(50, (m, k), 1.0))
    full = torch.zeros((m, sum(sizes) + 5), dtype=torch.bfloat16, device="cuda")
    segments, col = [], 0
    for w, n in zip(ws, sizes):
        segments.append((w, None, full[:, col:], full.shape[1], n))
        col += n
    nat.gemv_multi(nat.W_BF16, nat.DT_BF16, x, segments, None, nat.DT_BF16, m, k)
    col = 0
    for w, n in zip(ws, sizes):
        alone = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
        assert same_bits(full[:, col:col + n].contiguous(), alone)
        col += n
    assert not full[:, col:].any()


def test_chain_fused_equals_unfused_and_graph():
    from klab_b200.chain import ChainShape, ProjectionChain

    shape = ChainShape(layers=3, hidden=512, kv=128, ffn=1536)
    x = dev_bf16(og.normal_bf16_bits(60, (1, 512), 1.0))
    fused = ProjectionChain(shape, seed=3, fuse=True)
    plain = ProjectionChain(shape, seed=3, fuse=False)
    a = fused.forward_eager(x).clone()
    b = plain.forward_eager(x).clone()
    assert same_bits(a, b)
    out = fused.capture(x)
    fused.replay()
    torch.cuda.synchronize()
    assert same_bits(out, a)
    # one layer against the oracle (up, then down, each rounded once to BF16)
    one = ProjectionChain(ChainShape(layers=1, hidden=512, kv=128, ffn=1536), seed=3)
    got = host_bits(one.forward_eager(x))
    entry = one.layers[0]
    up = ob.round_bf16_bits(og.bf16_projection64(host_bits(x), host_bits(entry["up"][0])))
    ref64 = og.bf16_projection64(up, host_bits(entry["down"][0]))
    report = ob.check_outputs(ref64, ob.bf16_values(got), output_dtype="bf16")
    assert report["passed"] and report["max_ulp_error"] <= 1, report


@pytest.mark.parametrize("stages_per_layer", [2, 4])
@pytest.mark.parametrize("dims", [(3, 512, 128, 1536), (2, 1024, 256, 3584), (2, 256, 64, 512)])
def test_persistent_chain_equals_launch_chain(native, dims, stages_per_layer):
    """The one-launch persistent chain (stage flags as a grid barrier, split rows
    folded in chunk order) gives the launch-per-stage chain's bits, eagerly and
    under graph replay, every step; every stage's local outputs match too."""
    from klab_b200.chain import ChainShape, ProjectionChain

    layers, hidden, kv, ffn = dims
    shape = ChainShape(layers=layers, hidden=hidden, kv=kv, ffn=ffn)
    x = dev_bf16(og.normal_bf16_bits(61 + hidden, (1, hidden), 1.0))
    ref_chain = ProjectionChain(shape, seed=4)
    ref = ref_chain.forward_eager(x).clone()
    ref_a = {k: v.clone() for k, v in ref_chain.a_out.items()}
    pc = ProjectionChain(shape, seed=4, persistent=True, stages_per_layer=stages_per_layer)
    assert pc.launches_per_step() == 1
    for _ in range(2):
        got = pc.forward_eager(x)
        torch.cuda.synchronize()
        assert same_bits(got, ref)
    for name, t in ref_a.items():
        assert same_bits(pc.a_out[name], t), name
    out = pc.capture(x)
    for _ in range(3):
        pc.replay()
    torch.cuda.synchronize()
    assert same_bits(out, ref)
    assert int(pc.epoch.item()) == 2 + 1 + 3  # eager steps, capture warm-up, replays
    assert native.device_status() == 0
    pc.release()


def test_persistent_chain_timeline(native):
    """trace_step returns ordered global-timer stamps for every stage and CTA
    (entered <= previous stage done <= x staged; per warp staged <= first item
    landed <= run computed <= done) and leaves the step's result unchanged."""
    from klab_b200.chain import ChainShape, ProjectionChain

    shape = ChainShape(layers=2, hidden=1024, kv=256, ffn=3584)
    x = dev_bf16(og.normal_bf16_bits(71, (1, 1024), 1.0))
    pc = ProjectionChain(shape, seed=4, persistent=True)
    ref = pc.forward_eager(x).clone()
    tr = pc.trace_step(x).numpy()
    assert same_bits(pc.forward_eager(x), ref)
    stages, grid, slots = tr.shape
    assert stages == len(pc.persistent_schedule()) * shape.layers and slots == 3 + 3 * 16
    assert (tr[:, :, :3] > 0).all()
    assert (tr[:, :, 0] <= tr[:, :, 1]).all() and (tr[:, :, 1] <= tr[:, :, 2]).all()
    first, run, done = tr[:, :, 3::3], tr[:, :, 4::3], tr[:, :, 5::3]
    staged = tr[:, :, 2:3]
    assert (run >= staged).all() and (done >= run).all()
    held = first > 0  # warps holding items of the stage
    assert held.any(axis=2).all()
    assert (first[held] >= np.broadcast_to(staged, first.shape)[held]).all() and (run[held] >= first[held]).all()
    assert native.device_status() == 0
    pc.release()
