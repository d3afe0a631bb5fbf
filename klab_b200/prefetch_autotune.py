"""Capture-time autotune of side-stream L2 prefetch plans (drop-in for
research/l2-prefetch/src/autotune.py:9-59).

A plan prefetches the head (or all) of the next op's weights with `blocks`
CTAs of the l2_hint kernel. A candidate is kept only when its measured saving
has a bootstrap 95 % lower bound above min_lower_ci % and the outputs stay bit
for bit the same. Candidate grid for B200 (126 MB L2, 148 SMs): the whole
tensor or its first 16 / 4 / 1 MiB, with 2, 8, 32 or 148 blocks (the
reference's grid, (all, 1 MiB, 512 KiB) x (1, 2, 4, 8) blocks, is sized for a
4 MiB L2 and 46 SMs).
"""

from __future__ import annotations

from . import prefetch_harness as H
from .l2prefetch import ChainRunner

SIZES = (None, 16 << 20, 4 << 20, 1 << 20)
BLOCKS = (2, 8, 32, 148)


def candidates(nbytes):
    """name -> plan for every distinct (blocks, size) pair."""
    out, seen = {}, set()
    for blocks in BLOCKS:
        for size in SIZES:
            size = nbytes if size is None or size >= nbytes else size
            if (blocks, size) in seen:
                continue
            seen.add((blocks, size))
            out[f"b{blocks}_{size >> 10}k"] = {"blocks": blocks, "kernel": "l2_hint", "stride": 128, "nbytes": size}
    return out


def stage_bytes(reads):
    return sum(t.numel() * t.element_size() for t in reads)


def tune(ops, reads, x0, nbytes, rounds=9, min_lower_ci=1.0):
    """One plan for every op of a chain of identical layers: (plan or None, report)."""
    cands = candidates(nbytes)
    variants = {"torch": ChainRunner(ops, reads)}
    for name, plan in cands.items():
        variants[name] = ChainRunner(ops, reads, [plan] * len(ops))
    rows = H.run_variants(variants, x0, len(ops), rounds=rounds)
    best = min(cands, key=lambda name: rows[name]["us_per_op"])
    keep = rows[best]["ci95"][0] > min_lower_ci and rows[best]["bit_identical"]
    report = {name: {"saved_pct": row["saved_pct"], "ci95": row["ci95"]} for name, row in rows.items()}
    return (cands[best] if keep else None), {"best": best, "kept": keep, "candidates": report}


def tune_positions(ops, reads, x0, period, rounds=7, passes=1, min_lower_ci=1.0, log=print):
    """Coordinate descent over the plan of each position of a repeating pattern of `period` ops."""
    plans = [None] * period

    def expand(ps):
        return [ps[i % period] for i in range(len(ops))]

    history = []
    for _ in range(passes):
        for pos in range(period):
            nbytes = stage_bytes(reads[pos])
            cands = candidates(nbytes)
            variants = {"current": ChainRunner(ops, reads, expand(plans))}
            if plans[pos] is not None:
                variants["off"] = ChainRunner(ops, reads, expand(plans[:pos] + [None] + plans[pos + 1:]))
            for name, plan in cands.items():
                variants[name] = ChainRunner(ops, reads, expand(plans[:pos] + [plan] + plans[pos + 1:]))
            rows = H.run_variants(variants, x0, len(ops), rounds=rounds, baseline="current")
            best = min((name for name in rows if name != "current"), key=lambda name: rows[name]["us_per_op"])
            if rows[best]["ci95"][0] > min_lower_ci and rows[best]["bit_identical"]:
                plans[pos] = None if best == "off" else cands[best]
            history.append({"pos": pos, "bytes": nbytes, "best": best, "saved_vs_current": rows[best]["saved_pct"],
                            "ci95": rows[best]["ci95"], "kept": plans[pos] is not None})
            if log:
                log(f"  pos {pos} ({nbytes >> 10} KiB): best {best} {rows[best]['saved_pct']:+.2f}% -> "
                    f"plan {plans[pos]}")
    return plans, history
