"""Host logic of the prefetch tuner: candidate grid, static rule, paired statistics."""

import math

import pytest


def test_candidate_grid_is_distinct_and_clamped():
    from klab_b200 import prefetch_autotune as at

    per_kind = {kind: len(spec["blocks"]) for kind, spec in at.KINDS.items()}
    small = at.candidates(2 << 20)         # whole tensor and the 1 MiB head; larger heads collapse
    assert all(p["nbytes"] <= 2 << 20 for p in small.values())
    keys = {(p["kernel"], p["blocks"], p["nbytes"]) for p in small.values()}
    assert len(small) == len(keys) == 2 * sum(per_kind.values())
    big = at.candidates(64 << 20)
    assert len(big) == len(at.HEADS) * sum(per_kind.values())
    assert {p["kernel"] for p in big.values()} == {"l2_hint", "l2_bulk"}
    assert all(p["stride"] % 16 == 0 and p["threads"] in (32, 256) for p in big.values())


def test_race_halves_the_field_until_one_is_left(monkeypatch):
    """Successive halving keeps the faster half each time with twice the rounds, and keeps
    the survivor only above the lower-bound threshold and when bit-identical."""
    from klab_b200 import prefetch_autotune as at

    speed = {"base": 100.0, "a": 99.5, "b": 90.0, "c": 95.0, "d": 101.0, "e": 97.0}
    calls = []

    def fake_run(variants, x0, calls_per, rounds, baseline):
        calls.append((sorted(variants), rounds))
        rows = {}
        for name in variants:
            t = speed[name]
            saved = 100.0 * (1.0 - t / speed[baseline])
            rows[name] = {"us_per_op": t, "saved_pct": saved, "ci95": (saved - 0.5, saved + 0.5),
                          "bit_identical": name != "e", "samples_us": [t]}
        return rows

    monkeypatch.setattr(at.H, "run_variants", fake_run)
    variants = {k: None for k in speed}
    kept, row, seen = at.race(variants, None, 1, 3, "base")
    assert kept == "b" and row["saved_pct"] == pytest.approx(10.0)
    assert [len(v) - 1 for v, _ in calls] == [5, 2, 1] and [r for _, r in calls] == [3, 6, 12]
    assert set(seen) == set(speed) - {"base"}
    speed.update(b=99.4, c=99.6, e=99.0)                # e wins but its output differs
    assert at.race(variants, None, 1, 3, "base")[0] is None
    speed.update(e=99.8)                                # winner b saves 0.6 %: below the +1 % bound
    assert at.race(variants, None, 1, 3, "base")[0] is None


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
