"""Host logic of bench.py that needs no GPU: the persistent chain's timeline summary
(`--trace`) on a synthetic trace with known stage costs, and the reference arm's
rank handling under a launcher's environment."""

import importlib.util
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _trace(layers, per_layer, ctas=4, warps=16, skew_ns=40):
    """Stamps with fixed costs: barrier 300 ns, staging 700 ns (+200 on the first stage of a
    layer), first item 400 ns later, runs of 2000 ns, done 100 ns after the run; stage s starts
    5000 ns after stage s-1; CTA c enters skew_ns * c late."""
    tr = np.zeros((layers * per_layer, ctas, 3 + 3 * warps), dtype=np.int64)
    for s in range(layers * per_layer):
        for c in range(ctas):
            e = 10_000 + s * 5000 + c * skew_ns
            staging = 700 + (200 if s % per_layer == 0 else 0)
            tr[s, c, 0], tr[s, c, 1], tr[s, c, 2] = e, e + 300, e + 300 + staging
            first = e + 300 + staging + 400
            tr[s, c, 3::3], tr[s, c, 4::3], tr[s, c, 5::3] = first, first + 2000, first + 2100
    return tr


def test_timeline_summary_recovers_known_costs():
    bench = _bench()
    out = bench.chain_timeline(_trace(layers=4, per_layer=2), 2, ["up", "down"])
    up, down = out["stages"]["up"], out["stages"]["down"]
    assert up["barrier_us"] == pytest.approx(0.3) and down["barrier_us"] == pytest.approx(0.3)
    assert up["staging_us"] == pytest.approx(0.9) and down["staging_us"] == pytest.approx(0.7)
    assert up["first_wait_us"] == pytest.approx(0.4) and up["run_us"] == pytest.approx(2.0)
    assert up["cta_span_us"] == pytest.approx(2.5) and up["enter_skew_us"] == pytest.approx(0.12)
    # layers 1..3: first CTA entering layer 1 (20,000 ns) to the last warp done in the last
    # stage (10,000 + 7 * 5,000 + 3 * 40 + 3,500 ns), over three layers
    assert out["per_layer_us"] == pytest.approx((45_000 + 120 + 3_500 - 20_000) / 3 / 1000, abs=0.01)
    lo, mid, hi = out["cta_busy_per_layer_us_p0_50_100"]
    assert lo == mid == hi == pytest.approx(5.0)


def test_timeline_needs_two_layers():
    assert _bench().chain_timeline(_trace(layers=1, per_layer=4), 4, ["up", "fill1", "down", "fill2"]) is None


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "", (r.stdout, r.stderr)
