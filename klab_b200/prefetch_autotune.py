"""Capture-time choice of side-stream L2 prefetch plans.

Drop-in surface of research/l2-prefetch/src/autotune.py: `candidates(nbytes)`,
`stage_bytes(reads)`, `tune(ops, reads, x0, nbytes, ...)` and
`tune_positions(ops, reads, x0, period, ...)` keep their names, arguments and
return shapes, and a plan is still the keyword dict that
`l2prefetch.prefetch(tensor, **plan)` takes. The search is this module's own:

* The grid is sized for B200 (126 MB L2, 148 SMs) and has two kernel kinds:
  `l2_hint` (one prefetch.global.L2 per 128-byte line from 8, 32 or 148 CTAs)
  and `l2_bulk` (this library's bulk-copy prefetch: 64 KiB requests from 1, 4
  or 16 warps), each over the whole tensor or its first 16, 4 or 1 MiB.
* `race` runs successive halving: every candidate is timed against the
  baseline in paired, shuffled CUDA-graph rounds; the faster half (by median)
  advances and is timed again with twice the rounds, until one is left. The
  survivor is kept only when its paired saving has a bootstrap 95 % lower
  bound above `min_lower_ci` percent and its output is bit-identical to the
  baseline's, so a kept plan never changes results.
* `tune_positions` screens each position of a repeating pattern on its own
  (the other positions as currently chosen), then confirms the combined
  choice against no prefetch at all, dropping it if the combination loses.
"""

from __future__ import annotations

from . import prefetch_harness as H
from .l2prefetch import ChainRunner

HEADS = (None, 16 << 20, 4 << 20, 1 << 20)      # whole tensor, or its first 16 / 4 / 1 MiB
KINDS = {
    "l2_hint": {"blocks": (8, 32, 148), "threads": 256, "stride": 128},
    "l2_bulk": {"blocks": (1, 4, 16), "threads": 32, "stride": 64 << 10},
}


def candidates(nbytes):
    """name -> prefetch kwargs for every distinct (kind, blocks, head size) of the grid;
    heads at least as large as the tensor collapse into the whole tensor."""
    grid = {}
    for kind, spec in KINDS.items():
        for blocks in spec["blocks"]:
            for head in HEADS:
                size = nbytes if head is None or head >= nbytes else head
                name = f"{kind}_b{blocks}_{size >> 10}k"
                grid.setdefault(name, {"kernel": kind, "blocks": blocks, "threads": spec["threads"],
                                       "stride": spec["stride"], "nbytes": size})
    return grid


def stage_bytes(reads):
    """Bytes an op reads through the tensors listed for it."""
    return sum(t.numel() * t.element_size() for t in reads)


def race(variants, x0, calls, rounds, baseline, min_lower_ci=1.0):
    """Successive halving over `variants` (name -> callable(x) -> y; `baseline` is one of
    them). Returns (winner name or None, winner's row, {name: last row of every variant})."""
    field = [name for name in variants if name != baseline]
    if not field:
        return None, None, {}
    seen, n = {}, rounds
    while True:
        rows = H.run_variants({baseline: variants[baseline], **{k: variants[k] for k in field}}, x0, calls,
                              rounds=n, baseline=baseline)
        seen.update({k: v for k, v in rows.items() if k != baseline})
        if len(field) == 1:
            break
        field = sorted(field, key=lambda k: rows[k]["us_per_op"])[:max(1, len(field) // 2)]
        n *= 2
    name = field[0]
    row = seen[name]
    kept = row["ci95"][0] > min_lower_ci and row["bit_identical"]
    return (name if kept else None), row, seen


def tune(ops, reads, x0, nbytes, rounds=9, min_lower_ci=1.0):
    """One plan for every op of a chain of identical layers. Returns (plan or None, report)
    with report = {"best": name, "kept": bool, "candidates": {name: {saved_pct, ci95}}}."""
    grid = candidates(nbytes)
    variants = {"torch": ChainRunner(ops, reads)}
    variants.update({name: ChainRunner(ops, reads, [plan] * len(ops)) for name, plan in grid.items()})
    kept, row, rows = race(variants, x0, len(ops), rounds, "torch", min_lower_ci)
    best = kept or min(rows, key=lambda k: rows[k]["us_per_op"])
    report = {name: {"saved_pct": r["saved_pct"], "ci95": r["ci95"]} for name, r in rows.items()}
    return (grid[kept] if kept else None), {"best": best, "kept": kept is not None, "candidates": report}


def tune_positions(ops, reads, x0, period, rounds=7, passes=1, min_lower_ci=1.0, log=print):
    """Plans for a repeating pattern of `period` ops (op i uses plan i % period).

    Each pass screens every position: candidates for that position are raced with the
    other positions at their current plans (and, when the position has a plan, "off"
    among them). After the passes, the combined choice is raced against no prefetch; if
    it is not kept, every position is switched off. Returns (plans, history)."""

    def runner(assign):
        return ChainRunner(ops, reads, [assign[i % period] for i in range(len(ops))])

    plans, history = [None] * period, []
    for _ in range(passes):
        for pos in range(period):
            nbytes = stage_bytes(reads[pos])
            grid = candidates(nbytes)
            variants = {"current": runner(plans)}
            if plans[pos] is not None:
                variants["off"] = runner(plans[:pos] + [None] + plans[pos + 1:])
            for name, plan in grid.items():
                variants[name] = runner(plans[:pos] + [plan] + plans[pos + 1:])
            kept, row, rows = race(variants, x0, len(ops), rounds, "current", min_lower_ci)
            if kept is not None:
                plans[pos] = None if kept == "off" else grid[kept]
            best = kept or min(rows, key=lambda k: rows[k]["us_per_op"])
            history.append({"pos": pos, "bytes": nbytes, "best": best, "saved_vs_current": rows[best]["saved_pct"],
                            "ci95": rows[best]["ci95"], "kept": plans[pos] is not None})
            if log:
                log(f"  pos {pos} ({nbytes >> 10} KiB): {best} {rows[best]['saved_pct']:+.2f}% -> {plans[pos]}")
    if any(plans):
        kept, row, _ = race({"none": runner([None] * period), "chosen": runner(plans)}, x0, len(ops), rounds,
                            "none", min_lower_ci)
        history.append({"pos": "all", "bytes": sum(stage_bytes(reads[p]) for p in range(period)), "best": "chosen",
                        "saved_vs_current": row["saved_pct"], "ci95": row["ci95"], "kept": kept is not None})
        if kept is None:
            plans = [None] * period
    return plans, history
