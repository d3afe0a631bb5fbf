"""Fused multi-output projections (kv_pair.prepare_pair_graph, drop-in for
examples/kv_pair_projection.py, and prepare_fused_projection): one launch over
several weights sharing x, each output bit-identical to that weight projected
alone, and inside the oracle's check_outputs interval."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def exact_matmul_flags():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = old


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def test_pair_graph_matches_separate_projections_and_oracle():
    from klab_b200 import compressed_bf16 as cb
    from klab_b200.kv_pair import prepare_pair_graph

    k = 4096
    wk_bits = og.normal_bf16_bits(1, (1024, k), 0.02)
    wv_bits = og.normal_bf16_bits(2, (1024, k), 0.02)
    x_bits = og.normal_bf16_bits(3, (1, k), 1.0)
    wk, wv, x = dev_bf16(wk_bits), dev_bf16(wv_bits), dev_bf16(x_bits)
    pair = prepare_pair_graph(wk, wv)
    out = torch.empty((1, 2048), device="cuda", dtype=torch.float32)
    kv, vv = pair(x, out)
    assert kv.data_ptr() == out.data_ptr() and tuple(vv.shape) == (1, 1024)
    assert torch.equal(kv, cb.raw_linear(x, wk, threads=128, vector=8, output_dtype="fp32"))
    assert torch.equal(vv, cb.raw_linear(x, wv, threads=128, vector=8, output_dtype="fp32"))
    ref = og.bf16_projection64(x_bits, np.concatenate([wk_bits, wv_bits]))
    assert ob.check_outputs(ref, out.cpu().numpy(), output_dtype="fp32")["passed"]
    # Graph capture of the prepared callable.
    graph = torch.cuda.CUDAGraph()
    out2 = torch.zeros_like(out)
    with torch.cuda.graph(graph):
        pair(x, out2)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out2, out)


@pytest.mark.parametrize("m", [1, 3])
def test_fused_qkv_bf16(m):
    from klab_b200 import compressed_bf16 as cb
    from klab_b200.kv_pair import prepare_fused_projection

    k = 2048
    ws = [dev_bf16(og.normal_bf16_bits(10 + i, (n, k), 0.02)) for i, n in enumerate((2048, 512, 512))]
    x = dev_bf16(og.normal_bf16_bits(20 + m, (m, k), 1.0))
    fused = prepare_fused_projection(ws, torch.bfloat16)
    out = torch.empty((m, 3072), device="cuda", dtype=torch.bfloat16)
    views = fused(x, out)
    for w, v in zip(ws, views):
        ref = cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
        assert torch.equal(v.view(torch.int16), ref.view(torch.int16))


def test_validation_matches_reference():
    from klab_b200.kv_pair import prepare_pair_graph

    wk = torch.randn(64, 128, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        prepare_pair_graph(wk, torch.randn(64, 64, device="cuda").bfloat16())
    with pytest.raises(ValueError):
        prepare_pair_graph(wk.float(), wk.float())
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = True
    with pytest.raises(ValueError):
        prepare_pair_graph(wk, wk.clone())
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    pair = prepare_pair_graph(wk, wk.clone())
    with pytest.raises(ValueError):
        pair(torch.randn(2, 128, device="cuda").bfloat16(), torch.empty(2, 128, device="cuda"))
    with pytest.raises(ValueError):
        pair(torch.randn(1, 128, device="cuda").bfloat16(), torch.empty(1, 128, device="cuda").bfloat16())
