"""Prefetch tuning on the GPU: every candidate plan leaves the chain's outputs
bit-identical, and the tuned wrappers (PrefetchSequential, PrefetchHooks) return
exactly what the plain modules return."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(n, dim, dtype=torch.bfloat16):
    torch.manual_seed(3)
    return [torch.nn.Linear(dim, dim, bias=False).to("cuda", dtype).eval() for _ in range(n)]


def test_tune_candidates_never_change_outputs():
    from klab_b200 import compressed_bf16 as cb
    from klab_b200 import prefetch_autotune as at

    dim = 2048
    weights = [torch.randn(dim, dim, device="cuda").to(torch.bfloat16) * 0.02 for _ in range(6)]
    ops = [lambda y, w=w: cb.raw_linear(y, w, threads=128, vector=8, output_dtype="bf16") for w in weights]
    reads = [[w] for w in weights]
    x0 = torch.randn(1, dim, device="cuda").to(torch.bfloat16)
    plan, report = at.tune(ops, reads, x0, at.stage_bytes(reads[0]), rounds=3)
    assert report["best"] in at.candidates(at.stage_bytes(reads[0]))
    assert plan is None or plan["kernel"] in ("l2_hint", "l2_bulk")
    plans, history = at.tune_positions(ops, reads, x0, period=2, rounds=3, log=None)
    assert len(plans) == 2 and len(history) == 2


def test_prefetch_sequential_and_hooks_keep_outputs():
    from klab_b200.prefetch_api import PrefetchHooks, PrefetchSequential

    layers = _layers(4, 2048)
    x = torch.randn(1, 2048, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        ref = x
        for layer in layers:
            ref = layer(ref)
        fast = PrefetchSequential(layers, x, rounds=3)
        assert len(fast.report) == 1 and fast.report[0]["layers"] == 4
        assert torch.equal(fast(x), ref)
        model = torch.nn.Sequential(*layers)
        hooks = PrefetchHooks(model, x, rounds=3)
        assert len(hooks.units) == 4
        assert torch.equal(model(x), ref)
        hooks.remove()
        assert not hooks.handles and torch.equal(model(x), ref)
    torch.cuda.synchronize()
