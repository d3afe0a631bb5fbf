"""Host logic of the prefetch tuner: candidate grid, static rule, paired statistics."""

import math

import pytest


def test_candidate_grid_is_distinct_and_clamped():
    from klab_b200 import prefetch_autotune as at

    small = at.candidates(2 << 20)         # whole tensor and the 1 MiB head; larger heads collapse
    assert all(p["nbytes"] <= 2 << 20 for p in small.values())
    assert len(small) == len({(p["blocks"], p["nbytes"]) for p in small.values()}) == len(at.BLOCKS) * 2
    big = at.candidates(64 << 20)
    assert len(big) == len(at.BLOCKS) * len(at.SIZES)
    assert {p["kernel"] for p in big.values()} == {"l2_hint"}


def test_static_policy_thresholds():
    from klab_b200 import prefetch_policy as pp

    assert pp.plan(pp.MAX_BYTES + 1, 1) is None
    assert pp.plan(1 << 20, pp.MAX_M + 1) is None
    p = pp.plan(32 << 20, 1)
    assert 1 <= p["blocks"] <= pp.MAX_BLOCKS and p["kernel"] == "l2_hint"
    assert pp.plan(1 << 20, 1)["blocks"] <= p["blocks"]


def test_paired_saving_statistics():
    from klab_b200.prefetch_harness import paired_saving

    base = [100.0 + (i % 5) for i in range(31)]
    same, ci = paired_saving(base, list(base))
    assert same == 0.0 and ci == (0.0, 0.0)
    faster = [b * 0.9 for b in base]
    saved, (lo, hi) = paired_saving(base, faster)
    assert math.isclose(saved, 10.0, rel_tol=1e-9) and lo <= saved <= hi
    slower = [b * 1.05 for b in base]
    assert paired_saving(base, slower)[0] == pytest.approx(-5.0)
