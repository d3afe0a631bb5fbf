"""Prepared plans on the GPU: a plan's launch gives the bits of the same
klab_gemv call for every weight format, and the prepared wrappers
(PreparedBF16Projection, the prepared_bf16 / klab_native_v1 candidates,
prepare_projection) equal the unprepared projections bit for bit, eagerly and
under CUDA graph replay."""

import json

import numpy as np
import pytest
import torch

from oracle import gemv as og
from oracle import lossless as ol  # noqa: F401  (format pinned in test_gpu_lossless)

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def fp32_accumulation_contract():
    """The prepared objects require torch's reduced-precision matmul flags off."""
    m = torch.backends.cuda.matmul
    saved = (m.allow_tf32, m.allow_bf16_reduced_precision_reduction)
    m.allow_tf32, m.allow_bf16_reduced_precision_reduction = False, False
    yield
    m.allow_tf32, m.allow_bf16_reduced_precision_reduction = saved


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def _same(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (3, 1000, 2048), (1, 64, 14336)])
def test_bf16_plan_equals_gemv(m, n, k):
    from klab_b200 import _native
    from klab_b200.prepared import PreparedPlan

    x = _bf16(og.normal_bf16_bits(m + k, (m, k), 1.0))
    w = _bf16(og.normal_bf16_bits(n + k, (n, k), 0.02))
    for out_dtype in (torch.bfloat16, torch.float32):
        plan = PreparedPlan(_native.W_BF16, torch.bfloat16, out_dtype, m, n, k, "cuda")
        ref = torch.empty(m, n, dtype=out_dtype, device="cuda")
        _native.gemv(_native.W_BF16, _native.DT_BF16, x, w, None, None, ref,
                     _native.DT_BF16 if out_dtype == torch.bfloat16 else _native.DT_F32, m, n, k)
        got = plan.launch(x, w)
        torch.cuda.synchronize()
        assert _same(got, ref)
        info = plan.info
        assert info["shape_mnk"] == [m, n, k] and info["grid"][0] >= 1 and info["block"][0] in (256, 512)
        plan.close()


def test_quantized_and_lossless_plans_equal_gemv():
    from klab_b200 import _native, fp4, int8_weights, lossless_weights, packed_fp32
    from klab_b200.prepared import PreparedPlan

    m, n, k = 2, 512, 4096
    w32 = torch.randn(n, k, device="cuda") * 0.02
    xb = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    q = int8_weights.quantize_weights_per_row(w32)
    ref = int8_weights.fused_linear(xb, q.codes, q.scales, output_dtype=torch.bfloat16)
    got = PreparedPlan(_native.W_I8_ROW, torch.bfloat16, torch.bfloat16, m, n, k, "cuda").launch(xb, q.codes, q.scales)
    assert _same(got, ref)
    f = fp4.quantize_weights_f16(w32)
    ref = fp4.fused_linear(xb, f.packed, f.scales, None, output_dtype=torch.bfloat16)
    got = PreparedPlan(_native.W_FP4_G32H, torch.bfloat16, torch.bfloat16, m, n, k, "cuda").launch(xb, f.packed,
                                                                                                   f.scales)
    assert _same(got, ref)
    x32 = torch.randn(m, k, device="cuda")
    plain = PreparedPlan(_native.W_F32, torch.float32, torch.float32, m, n, k, "cuda").launch(x32, w32)
    lw = lossless_weights.pack_weights(w32)
    got = PreparedPlan(_native.W_LF32, torch.float32, torch.float32, m, n, k, "cuda").launch(
        x32, lw.mantissa, lw.metadata, lw.exponents)
    assert _same(got, plain)
    pf = packed_fp32.pack_weights(w32)
    got = PreparedPlan(_native.W_FP28, torch.float32, torch.float32, m, n, k, "cuda").launch(x32, pf.payload,
                                                                                            pf.metadata)
    assert _same(got, plain)
    torch.cuda.synchronize()


def test_plan_rejects_misaligned_and_wrong_inputs():
    from klab_b200 import _native
    from klab_b200.prepared import PreparedPlan

    plan = PreparedPlan(_native.W_BF16, torch.bfloat16, torch.bfloat16, 1, 256, 1024, "cuda")
    buf = torch.zeros(2048 + 8, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(256, 1024, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_native.KlabError):
        plan.launch(buf[1:1025].view(1, 1024), w)          # x not 16-byte aligned
    with pytest.raises(ValueError):
        plan.launch(torch.zeros(2, 1024, dtype=torch.bfloat16, device="cuda"), w)


def test_prepared_bf16_projection_and_graph():
    from klab_b200 import compressed_bf16 as cb
    from klab_b200.prepared_bf16 import PreparedBF16Projection

    n, k = 2048, 4096
    w = _bf16(og.normal_bf16_bits(9, (n, k), 0.02))
    x = _bf16(og.normal_bf16_bits(10, (1, k), 1.0))
    proj = PreparedBF16Projection(w, 1, output_dtype=torch.bfloat16)
    assert proj.plan["backend"] == "custom" and proj.shape_mnk == (1, n, k)
    ref = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
    assert _same(proj(x), ref)
    out = torch.empty(1, n, dtype=torch.bfloat16, device="cuda")
    assert _same(proj(x, out=out), ref)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        y = proj(x)
    g.replay()
    torch.cuda.synchronize()
    assert _same(y, ref)
    vendor = PreparedBF16Projection(w, 1, {"kind": "compressed-projection", "cases": []},
                                    output_dtype=torch.float32)
    assert vendor.plan["backend"] == "vendor" and vendor.strategy == "torch_mm_out_fp32"
    assert vendor(x).dtype == torch.float32


def test_candidates_equal_unprepared_wrappers():
    from klab_b200 import compressed_bf16 as cb
    from klab_b200.native_prepared import NativeCodedCandidate, NativeRawCandidate
    from klab_b200.prepared_kernels import CodedCandidate, RawCandidate

    m, n, k = 4, 768, 4096
    bits = og.normal_bf16_bits(12, (n, k), 0.02)
    w = _bf16(bits)
    packed = cb.upload(cb.pack_bits(bits), "cuda")
    x = _bf16(og.normal_bf16_bits(13, (m, k), 1.0))
    for output in ("bf16", "fp32"):
        ref = cb.raw_linear(x, w, threads=128, vector=8, output_dtype=output)
        for cand in (RawCandidate(w, m, threads=128, vector=8, output_dtype=output),
                     CodedCandidate(packed, m, threads=128, vector=8, output_dtype=output),
                     NativeRawCandidate(w, m, threads=128, vector=8, output_dtype=output),
                     NativeCodedCandidate(packed, m, threads=128, vector=8, output_dtype=output)):
            assert _same(cand(x), ref), type(cand).__name__
        assert json.loads(torch.ops.klab_native_v1.plan_info(cand.plan_id))["kind"] == "coded"
        cand.close()
        with pytest.raises(ValueError):
            torch.ops.klab_native_v1.plan_info(cand.plan_id)
    torch.cuda.synchronize()


def test_prepare_projection_routes():
    from klab_b200.dynamic_projection import prepare_projection

    n, k = 512, 1024
    w = torch.randn(n, k, device="cuda")
    x = torch.randn(1, k, device="cuda")
    plain = prepare_projection(w, 1)
    y = plain(x)
    report = {"kind": "streaming-projection", "status": "complete", "cases": [
        {"shape_mnk": [1, n, k], "seed": s, "selected": "lossless_t128", "candidate_gain_ci95_pct": [5.0, 8.0],
         "aa_time_saved_pct": 0.2, "bitwise_round_trip": True, "accepted_custom_win": True,
         "methods": {"torch_mm": {"median_us": 9.0}}} for s in (1, 2)]}
    lossless = prepare_projection(w, 1, report)
    assert lossless.strategy == "lossless_t128" and lossless.packed is not None
    assert _same(lossless(x), y)
    half = prepare_projection(w.to(torch.bfloat16), 1, output_dtype=torch.bfloat16)
    assert half(x.to(torch.bfloat16)).dtype == torch.bfloat16
    torch.cuda.synchronize()
