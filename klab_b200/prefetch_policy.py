"""Static side-stream prefetch rule (drop-in for research/l2-prefetch/src/policy.py:11-17,
which the capture-time autotuner supersedes).

Prefetch the next op's weights only when the current and the next op fit
together in about three quarters of L2 and M is small (a weight-streaming op);
size the grid so the prefetch finishes within the op's estimated duration.
B200 constants: L2 126 MB, HBM time at the measured 6.46 TB/s plus a 2 µs launch
floor, and a prefetch CTA issuing about 40 GB/s (one 256-thread l2_hint block
per SM covers HBM bandwidth at 148 blocks).
"""

from __future__ import annotations

import math

L2_BYTES = 126 << 20
MAX_BYTES = int(0.375 * L2_BYTES)   # current + next op within ~0.75 of L2
MAX_M = 32
HBM_BYTES_PER_US = 6.46e6
BLOCK_RATE = 40e3                    # bytes per µs one prefetch block issues
MARGIN = 1.25
MAX_BLOCKS = 148


def plan(nbytes, m):
    """Prefetch kwargs for an op that reads `nbytes` of weights with M rows, or None."""
    if nbytes > MAX_BYTES or m > MAX_M:
        return None
    t_est = 2.0 + nbytes / HBM_BYTES_PER_US
    blocks = min(MAX_BLOCKS, max(1, math.ceil(MARGIN * nbytes / (BLOCK_RATE * t_est))))
    return {"blocks": blocks, "kernel": "l2_hint", "stride": 128}
