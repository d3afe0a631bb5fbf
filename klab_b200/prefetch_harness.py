"""Paired timing of chain variants for the prefetch autotuner (the role of
research/l2-prefetch/src/harness.py:34-55 and harness2.py:11-23).

Every variant is captured once into a CUDA graph; each round replays all
variants in a shuffled order, timing each replay with CUDA events on the
replaying stream, so the rounds of two variants are paired by index. The saving
of a candidate against the baseline is the median of the per-round ratios
1 - cand/base, with a percentile-bootstrap 95 % interval over rounds; outputs are
compared bit for bit against the baseline's.
"""

from __future__ import annotations

import random
import time

import torch


def paired_saving(base, cand, draws=2000, seed=7):
    """(median saving %, (low, high) bootstrap 95 % interval) of paired samples."""
    ratios = [1.0 - c / b for b, c in zip(base, cand)]
    rng = random.Random(seed)

    def median(values):
        return sorted(values)[len(values) // 2]

    boots = sorted(median([rng.choice(ratios) for _ in ratios]) for _ in range(draws))
    return 100.0 * median(ratios), (100.0 * boots[int(0.025 * draws)], 100.0 * boots[int(0.975 * draws)])


def warm(variants, x0, seconds=2.0):
    """Run every variant repeatedly for `seconds` so clocks settle before timing."""
    end = time.monotonic() + seconds
    while time.monotonic() < end:
        for fn in variants.values():
            fn(x0)
        torch.cuda.synchronize()


def measure(variants, x0, rounds=15, seed=11):
    """name -> {"samples_us": [...], "median_us": m, "out": last output} by graph replay."""
    stream = torch.cuda.Stream()
    graphs, outs = {}, {}
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for name, fn in variants.items():
            fn(x0)  # eager run outside capture (module loads, workspaces)
        torch.cuda.synchronize()
        for name, fn in variants.items():
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                outs[name] = fn(x0)
            graphs[name] = g
    torch.cuda.synchronize()
    order = list(graphs)
    rng = random.Random(seed)
    samples = {name: [] for name in order}
    for _ in range(rounds):
        rng.shuffle(order)
        for name in order:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graphs[name].replay()
            b.record()
            b.synchronize()
            samples[name].append(a.elapsed_time(b) * 1000.0)
    result = {}
    for name in graphs:
        s = samples[name]
        result[name] = {"samples_us": s, "median_us": sorted(s)[len(s) // 2], "out": outs[name].clone()}
    del graphs
    return result


def run_variants(variants, x0, calls, rounds=15, baseline="torch", warm_seconds=0.5):
    """variants: name -> callable(x) -> y over the whole chain; calls = ops per chain."""
    with torch.no_grad():
        if warm_seconds:
            warm(variants, x0, warm_seconds)
        t = measure(variants, x0, rounds=rounds)
    ref = t[baseline]["out"]
    rows = {}
    for name, v in t.items():
        saved, ci = paired_saving(t[baseline]["samples_us"], v["samples_us"])
        rows[name] = {"us_per_op": v["median_us"] / calls, "saved_pct": saved, "ci95": ci,
                      "bit_identical": bool(torch.equal(v["out"], ref)), "samples_us": v["samples_us"]}
    return rows
