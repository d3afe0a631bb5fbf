"""Timing of projections on the GPU: CUDA-graph replay over rings of distinct weights.

The protocol of the reference's benches (bench.py:50-106, bench_streaming.py:46-50)
scaled to B200: each timed call reads its own copy of the weights from a ring
totalling at least max(2 GiB, 16 x L2), so every call streams from HBM; the
calls of one ring are captured in one CUDA graph and replayed; the result is
the median over rounds of (replay time / calls), from CUDA events on the
replaying stream after warm-up replays.
"""

from __future__ import annotations

import math
import statistics

import torch

L2_BYTES = 126 * 1024 * 1024


def ring_count(nbytes):
    """Copies of an nbytes operand that together exceed max(2 GiB, 16 x L2)."""
    return max(8, math.ceil(max(2 << 30, 16 * L2_BYTES) / max(1, nbytes)))


def graph_of(fn, stream):
    """Run fn once eagerly on `stream` (module loads, workspaces), then capture it."""
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        fn()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    return graph


def time_graph(graph, calls, rounds, warmup=3):
    """Median µs per call over `rounds` replays of a graph holding `calls` calls."""
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(rounds):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) * 1000.0 / calls)
    return statistics.median(times)


def time_ring(fn, ring, rounds, stream=None):
    """Median µs of fn(i) for i over a ring of `ring` distinct operands."""
    stream = stream or torch.cuda.Stream()
    graph = graph_of(lambda: [fn(i) for i in range(ring)], stream)
    try:
        return time_graph(graph, ring, rounds)
    finally:
        del graph
