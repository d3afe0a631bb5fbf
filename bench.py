#!/usr/bin/env python
"""Benchmark of the B200 small-batch projection path (one JSON line on rank 0).

Headline workload (benchmark config 5): the 32-layer Llama-3-8B-shaped
projection chain at M=1 in one CUDA graph per token, column-sharded over the
GPUs with an all-gather of `up` and `down` outputs per layer. value = tokens/s
of the whole job (strong scaling: the per-token work is fixed as N grows).
Weights are 13.96 GB per token step, far larger than the 126 MB L2, so every
step reads HBM without an explicit flush.

Also reported (N=1): µs / achieved GB/s for configs 1-4 next to cuBLAS on the
same shapes (`projections`), the roofline of the dominant kernel, the
end-to-end rate through the public API with host buffers (`e2e`), the CPU
oracle timed on the host (`cpu_baseline`), and SM clocks sampled during the
timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "achieved HBM GB/s vs 8 TB/s & µs/projection at M=1..16; chain tok/s 1/2/4/8 GPU"
FALLBACK_HBM_GBS = 6650.0


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu_id)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.perf_counter(), [p.strip() for p in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1):
        rows = [s for (t, s) in self.samples if t0 - 0.06 <= t <= t1 + 0.06 and len(s) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][2]),
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


# ---------------------------------------------------------------- helpers

def gpu_uuid(torch, device):
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        return str(device)


def all_max(torch, value, world):
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------- per-config projections (N=1)

def bench_projections(torch, peak, quick=False):
    """Configs 1-4 through the public API over cold-L2 weight rings, beside two vendor
    routes on the same shapes with BF16 weights (dequantized for INT8/FP4): torch F.linear
    (cuBLAS) and a frozen cuBLASLt plan (the fastest heuristic candidate, lt_baseline).
    The reference's own INT8 per-64 and E4M3/16 + global FP4 formats are timed too."""
    import torch.nn.functional as F

    from klab_b200 import compressed_bf16 as cb
    from klab_b200 import fp4, int8_weights, measure
    from klab_b200 import lt_baseline as lt

    dev = torch.device("cuda")
    stream = torch.cuda.Stream()
    gen = torch.Generator(device=dev)
    results = []
    rounds = 5 if quick else 15

    def record(name, m, n, k, nbytes, fn_ours, ring, x=None, vw=None):
        """vw: BF16 weights (a ring) for the vendor routes on x."""
        g = measure.graph_of(lambda: [fn_ours(i) for i in range(ring)], stream)
        us = measure.time_graph(g, ring, rounds)
        del g
        row = {"config": name, "m": m, "n": n, "k": k, "bytes": nbytes, "us": round(us, 3),
               "gbs": round(nbytes / us / 1e3, 1), "frac_of_measured_peak": round(nbytes / us / 1e3 / peak, 4)}
        if vw is not None:
            vr = len(vw)
            gv = measure.graph_of(lambda: [F.linear(x, vw[i % vr]) for i in range(ring)], stream)
            vus = measure.time_graph(gv, ring, rounds)
            del gv
            row["cublas_us"] = round(vus, 3)
            row["speedup_vs_cublas"] = round(vus / us, 3)
            try:
                plan = lt.tune_plan(x, vw[0], torch.bfloat16, rounds=5)
                lout = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
                gl = measure.graph_of(lambda: [plan.run(x, vw[i % vr], lout) for i in range(ring)], stream)
                lus = measure.time_graph(gl, ring, rounds)
                del gl
                plan.close()
                row["cublaslt_frozen_us"] = round(lus, 3)
                row["speedup_vs_best_vendor"] = round(min(vus, lus) / us, 3)
            except (lt.LtUnavailable, RuntimeError, ValueError) as error:
                row["cublaslt_frozen_us"] = None
                row["cublaslt_note"] = str(error)[:120]
        results.append(row)
        torch.cuda.empty_cache()

    def bf16_normal(shape, std, seed):
        gen.manual_seed(seed)
        return torch.randn(shape, generator=gen, device=dev).mul_(std).to(torch.bfloat16)

    # C1: BF16 4096 x 4096, M = 1
    n = k = 4096
    gen.manual_seed(0)   # benchmark config 1: W then x from one seed-0 stream, N(0, 0.02^2)
    w = torch.randn((n, k), generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
    x = torch.randn((1, k), generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
    nbytes = n * k * 2 + k * 2 + n * 2
    ring = measure.ring_count(n * k * 2)
    ws = [w.clone() for _ in range(ring)]
    outs = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
    record("c1_bf16_m1", 1, n, k, nbytes,
           lambda i: cb.raw_linear(x, ws[i], threads=128, vector=8, output_dtype="bf16", out=outs), ring, x, ws)
    del ws, w

    # C2: INT8 per-row, K=4096, N=14336, M in {1, 4, 16}
    n, k = 14336, 4096
    gen.manual_seed(3)
    w32 = torch.randn((n, k), generator=gen, device=dev).mul_(0.02)
    q = int8_weights.quantize_weights_per_row(w32)
    deq = q.dequantize().to(torch.bfloat16)
    del w32
    ring = measure.ring_count(n * k)
    codes = [q.codes.clone() for _ in range(ring)]
    vring = max(4, math.ceil(ring / 2))
    deqs = [deq.clone() for _ in range(vring)]
    for m in ((1,) if quick else (1, 4, 16)):
        x = bf16_normal((m, k), 1.0, 4 + m)
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        nbytes = n * k + n * 4 + m * k * 2 + m * n * 2
        record(f"c2_int8_row_m{m}", m, n, k, nbytes,
               lambda i: int8_weights.fused_linear(x, codes[i], q.scales, out=out, output_dtype=torch.bfloat16),
               ring, x, deqs)
    del codes, deqs, deq, q
    # the reference's INT8 format: FP32 scale per 64 columns (int8_weights.py:23-35), M = 1
    gen.manual_seed(3)
    q = int8_weights.quantize_weights(torch.randn((n, k), generator=gen, device=dev).mul_(0.02))
    ring = measure.ring_count(n * k + n * k // 16)
    codes = [(q.codes.clone(), q.scales.clone()) for _ in range(ring)]
    x = bf16_normal((1, k), 1.0, 5)
    out = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
    record("c2_int8_g64_m1 (reference format)", 1, n, k, n * k + n * k // 16 + k * 2 + n * 2,
           lambda i: int8_weights.fused_linear(x, codes[i][0], codes[i][1], out=out, output_dtype=torch.bfloat16),
           ring)
    del codes, q

    # C3: FP4 E2M1 with FP16 scales per 32, K=N=8192, M in {1, 8}
    n = k = 8192
    gen.manual_seed(5)
    w32 = torch.randn((n, k), generator=gen, device=dev).mul_(0.02)
    q = fp4.quantize_weights_f16(w32)
    deq = q.dequantize().to(torch.bfloat16)
    del w32
    ring = measure.ring_count(n * k // 2 + n * k // 16)
    packs = [(q.packed.clone(), q.scales.clone()) for _ in range(ring)]
    vring = max(4, math.ceil(ring / 4))
    deqs = [deq.clone() for _ in range(vring)]
    for m in ((1,) if quick else (1, 8)):
        x = bf16_normal((m, k), 1.0, 6 + m)
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        nbytes = n * k // 2 + n * k // 16 + m * k * 2 + m * n * 2
        record(f"c3_fp4_f16s32_m{m}", m, n, k, nbytes,
               lambda i: fp4.fused_linear(x, packs[i][0], packs[i][1], None, out=out, output_dtype=torch.bfloat16),
               ring, x, deqs)
    del packs, deqs, deq, q
    # the reference's FP4 format: E4M3 scale per 16 columns and an FP32 global scale (fp4.py:33-60), M = 1
    gen.manual_seed(5)
    q = fp4.quantize_weights(torch.randn((n, k), generator=gen, device=dev).mul_(0.02))
    ring = measure.ring_count(n * k // 2 + n * k // 16)
    packs = [(q.packed.clone(), q.scales.clone()) for _ in range(ring)]
    x = bf16_normal((1, k), 1.0, 7)
    out = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
    record("c3_fp4_e4m3g16_m1 (reference format)", 1, n, k, n * k // 2 + n * k // 16 + 4 + k * 2 + n * 2,
           lambda i: fp4.fused_linear(x, packs[i][0], packs[i][1], q.global_scale, out=out,
                                      output_dtype=torch.bfloat16), ring)
    del packs, q

    # C4: lossless-coded BF16, 8 independent 4096 x 4096 layers
    n = k = 4096
    layers = []
    for seed in range(8):
        w = bf16_normal((n, k), 0.02, 100 + seed)
        bits = w.view(torch.int16).cpu().numpy().view("uint16")
        layers.append((cb.upload(cb.pack_bits(bits), dev), w))
    per = layers[0][0].storage_bytes
    ring = measure.ring_count(per)
    coded = [layers[i % 8][0] for i in range(8)]
    coded += [cb.PackedBF16(coded[i % 8].payload.clone(), coded[i % 8].metadata.clone(), n, k,
                            coded[i % 8].source_sha256, 1, coded[i % 8].module) for i in range(8, ring)]
    raws = [layers[i % 8][1] for i in range(8)] + [layers[i % 8][1].clone() for i in range(8, measure.ring_count(n * k * 2))]
    x = bf16_normal((1, k), 1.0, 9)
    out = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
    storage = sum(c.storage_bytes for c in coded) / len(coded)
    nbytes = int(storage) + k * 2 + n * 2
    record("c4_lossless_bf16_m1", 1, n, k, nbytes,
           lambda i: cb.fused_linear(x, coded[i], threads=128, vector=8, output_dtype="bf16", out=out), ring, x, raws)
    results[-1]["storage_fraction"] = round(storage / (n * k * 2), 4)
    results[-1]["effective_bf16_gbs"] = round((n * k * 2 + k * 2 + n * 2) / results[-1]["us"] / 1e3, 1)
    del coded, raws, layers
    torch.cuda.empty_cache()
    return results


def bench_decode_attention(torch, peak, quick=False):
    """Decode attention with the KV append (klab_b200.decode_attn, Llama-3-8B heads: 32 query, 8 kv,
    head 64, capacity 4096) over a ring of caches larger than L2, with torch's SDPA on the same
    caches. bytes = the K and V rows read (L + 1 per kv head) + q, the new rows and the output."""
    import torch.nn.functional as F

    from klab_b200 import measure
    from klab_b200.decode_attn import decode_attention

    dev = torch.device("cuda")
    stream = torch.cuda.Stream()
    heads, kv, cap = 32, 8, 4096
    per = 2 * kv * cap * 64 * 2
    ring = max(8, math.ceil(4 * measure.L2_BYTES / per))
    gen = torch.Generator(device=dev).manual_seed(21)
    caches = [(torch.randn((kv, cap, 64), generator=gen, device=dev).to(torch.bfloat16),
               torch.randn((kv, cap, 64), generator=gen, device=dev).to(torch.bfloat16)) for _ in range(ring)]
    q = torch.randn(heads * 64, generator=gen, device=dev).to(torch.bfloat16)
    kn = torch.randn(kv * 64, generator=gen, device=dev).to(torch.bfloat16)
    vn = torch.randn(kv * 64, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty(heads * 64, device=dev, dtype=torch.bfloat16)
    rows = []
    for length in ((4095,) if quick else (255, 1023, 4095)):
        def ours(i):
            decode_attention(q, kn, vn, caches[i][0], caches[i][1], length, out=out)

        def sdpa(i):
            F.scaled_dot_product_attention(q.view(1, heads, 1, 64), caches[i][0][:, :length + 1].unsqueeze(0),
                                           caches[i][1][:, :length + 1].unsqueeze(0), enable_gqa=True)

        nbytes = 2 * kv * (length + 1) * 64 * 2 + heads * 64 * 2 * 2 + 2 * kv * 64 * 2
        g = measure.graph_of(lambda: [ours(i) for i in range(ring)], stream)
        us = measure.time_graph(g, ring, 5 if quick else 15)
        del g
        gv = measure.graph_of(lambda: [sdpa(i) for i in range(ring)], stream)
        vus = measure.time_graph(gv, ring, 5 if quick else 15)
        del gv
        rows.append({"heads": heads, "kv_heads": kv, "length": length, "capacity": cap, "bytes": nbytes,
                     "us": round(us, 3), "gbs": round(nbytes / us / 1e3, 1),
                     "frac_of_measured_peak": round(nbytes / us / 1e3 / peak, 4), "sdpa_us": round(vus, 3),
                     "speedup_vs_sdpa": round(vus / us, 3)})
    del caches
    torch.cuda.empty_cache()
    return rows


def bench_prefetch(torch, quick=False):
    """Does a side-stream L2 prefetch lift a C5-shaped pair of projections on B200? The
    autotuner's per-position search (prefetch_autotune.tune_positions: every candidate of
    both kinds, successive halving, bootstrap lower bound > +1 %, bit-identical outputs)
    over 8 layers of (o 4096x4096, gate 14336x4096) BF16 projections at M=1 with distinct
    weights (1.2 GB, cold L2), timed by CUDA events on graph replays."""
    from klab_b200 import compressed_bf16 as cb
    from klab_b200 import prefetch_autotune as at

    gen = torch.Generator(device="cuda").manual_seed(31)
    shapes = [(4096, 4096), (14336, 4096)] * 8
    weights = [torch.randn(s, generator=gen, device="cuda").mul_(0.02).to(torch.bfloat16) for s in shapes]
    outs = [torch.empty((1, s[0]), device="cuda", dtype=torch.bfloat16) for s in shapes]
    x0 = torch.randn((1, 4096), generator=gen, device="cuda").to(torch.bfloat16)

    def op(i):
        # every op reads the same token x0 (the pair's weights, not its data flow, set the traffic)
        return lambda y, i=i: (cb.raw_linear(x0, weights[i], threads=128, vector=8, output_dtype="bf16",
                                             out=outs[i]), y)[1]

    ops = [op(i) for i in range(len(shapes))]
    reads = [[w] for w in weights]
    plans, history = at.tune_positions(ops, reads, x0, period=2, rounds=3 if quick else 7, log=None)
    rows = [{"position": ("o" if h["pos"] == 0 else "gate" if h["pos"] == 1 else "both"), "best": h["best"],
             "saved_pct": round(h["saved_vs_current"], 3), "ci95": [round(v, 3) for v in h["ci95"]],
             "kept": h["kept"]} for h in history]
    del weights, outs
    torch.cuda.empty_cache()
    return {"workload": "8 x (o 4096x4096, gate 14336x4096) bf16 M=1, distinct weights (1.2 GB)",
            "plans": [p if p is None else {k: p[k] for k in ("kernel", "blocks", "nbytes")} for p in plans],
            "search": rows}


# ---------------------------------------------------------------- dominant kernel roofline

# dram__bytes_read.sum + dram__bytes_write.sum of one gate launch (14336 x 4096 BF16,
# M=1), mean of the two launches captured for profiles/stream_gemv_gate_bf16_m1.md.
NCU_GATE_TRAFFIC_BYTES = 117_492_224 + 4_048_640


def bench_dominant_kernel(torch, chain, peak, rounds=10):
    """Average duration of the chain's gate projection (the largest BF16 GEMV),
    timed with CUDA events on its launch stream over the chain's 32 distinct gate
    weights (cold L2), inside a CUDA graph."""
    from klab_b200 import _native, measure

    shape = chain.shape
    gates = [layer["gate"] for layer in chain.layers]
    h = chain.hbuf[0]
    out = chain.a_out["gate"]
    n_shard = gates[0][1][1] - gates[0][1][0]
    stream = torch.cuda.Stream()

    def run():
        for w, rows, n in gates:
            _native.gemv(_native.W_BF16, _native.DT_BF16, h, w, None, None, out[:, rows[0]:], _native.DT_BF16,
                         h.shape[0], n_shard, shape.hidden, ldo=n)

    g = measure.graph_of(run, stream)
    torch.cuda.nvtx.range_push("dominant")   # ncu --nvtx-include "dominant/" selects these launches
    us = measure.time_graph(g, len(gates), rounds)
    torch.cuda.nvtx.range_pop()
    del g
    nbytes = n_shard * shape.hidden * 2 + shape.hidden * 2 + n_shard * 2
    achieved = nbytes / us / 1e3
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": NCU_GATE_TRAFFIC_BYTES if chain.world == 1 else None,
            "traffic_unit": "bytes per launch, from one ncu capture of this launch at N=1 "
                            "(profiles/stream_gemv_gate_bf16_m1.md); a cross-check, not measured in this run",
            "kernel": "stream_gemv_kernel<W_BF16,X_BF16,SMEM16,1>",
            "launch": f"gate {n_shard}x{shape.hidden} bf16, M=1", "bytes_per_launch": nbytes,
            "us_per_launch": round(us, 3)}


# ---------------------------------------------------------------- CPU baselines

LAYER_SHAPES = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096),
                (4096, 14336)]   # q, k, v, o, gate, up, down (one decoder layer of the chain)


def host_threads():
    """All host cores, whatever OMP_NUM_THREADS a launcher set (torchrun sets 1)."""
    return os.cpu_count() or 1


def cpu_reference_tok_s(seconds=10.0):
    """The reference's CPU path for this workload: torch.nn.functional.linear on CPU BF16
    tensors (the "bf16_reference / torch F.linear path" of benchmark config 1; torch 2.11 as
    the reference's requirements.lock pins it), with torch.set_num_threads(all host cores),
    over one 7-projection decoder layer of the chain (up feeds down), repeated for about
    `seconds` and scaled to 32 layers per token."""
    import torch

    before = torch.get_num_threads()
    torch.set_num_threads(host_threads())
    try:
        gen = torch.Generator().manual_seed(0)
        weights = [(torch.randn(shape, generator=gen) * 0.02).to(torch.bfloat16) for shape in LAYER_SHAPES]
        h = torch.randn((1, 4096), generator=gen).to(torch.bfloat16)
        F = torch.nn.functional

        def layer():
            for w in weights[:6]:
                y = F.linear(h, w)
            return F.linear(y, weights[6])          # y is up (the sixth projection): it feeds down

        layer()                                     # warm-up
        layers, t0 = 0, time.perf_counter()
        while True:
            layer()
            layers += 1
            if time.perf_counter() - t0 >= seconds:
                break
        elapsed = time.perf_counter() - t0
        threads = torch.get_num_threads()
    finally:
        torch.set_num_threads(before)
    per_token = elapsed / layers * 32
    return {"value": round(1.0 / per_token, 4), "unit": "tok/s", "cores": int(threads), "kind": "reference",
            "sample": f"{layers} passes over one 7-projection decoder layer (torch {torch.__version__} F.linear, "
                      f"CPU bf16, {threads} threads), {elapsed:.1f} s, scaled x32 layers per token"}


def cpu_oracle_tok_s(seconds=10.0):
    """The FP64 oracle port (oracle.gemv.projection64 + round_bf16_bits) timed the same way
    on all host cores; weights are widened to FP64 outside the timed region."""
    import numpy as np

    from oracle import bf16 as ob
    from oracle import gemv as og

    try:
        from threadpoolctl import threadpool_limits
        limits = threadpool_limits(host_threads())
    except Exception:
        limits = None
    import torch

    gen = torch.Generator().manual_seed(0)

    def values(shape, std):
        t = (torch.randn(shape, generator=gen) * std).to(torch.bfloat16)
        return ob.bf16_values(t.view(torch.int16).numpy().view(np.uint16))

    weights = [values(shape, 0.02) for shape in LAYER_SHAPES]
    x, up = values((1, 4096), 1.0), values((1, 14336), 1.0)
    layers = 0
    t0 = time.perf_counter()
    while True:
        for i, w in enumerate(weights):
            ob.round_bf16_bits(og.projection64(up if i == 6 else x, w))
        layers += 1
        if time.perf_counter() - t0 >= seconds:
            break
    elapsed = time.perf_counter() - t0
    if limits is not None:
        limits.restore_original_limits()
    return {"value": round(layers / (32.0 * elapsed), 4), "unit": "tok/s", "cores": host_threads(), "kind": "port",
            "sample": f"{layers} passes over one 7-projection decoder layer (FP64 oracle), {elapsed:.1f} s, "
                      f"scaled x32 layers per token"}


def chain_parity(torch):
    """The checker in the CPU leg: the benchmark chain's first two layers (same seeds as the
    timed chain) on this GPU against the FP64 oracle with the chain's per-stage BF16
    rounding (every projection output within the reference's check_outputs interval and one
    BF16 ulp of FP64; down checked from the GPU's own up output)."""
    import numpy as np

    from klab_b200.chain import ChainShape, ProjectionChain
    from oracle import bf16 as ob
    from oracle import gemv as og

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    gen = torch.Generator(device="cuda").manual_seed(1234)
    x = torch.randn((1, 4096), generator=gen, device="cuda").to(torch.bfloat16)
    worst, passed, checked = 0, True, 0
    h_bits = bits(x)
    for layers in (1, 2):
        chain = ProjectionChain(ChainShape(layers=layers), seed=0)
        h = chain.forward_eager(x)
        entry = chain.layers[layers - 1]
        got = dict(chain.a_out, up=chain.up_full, down=h)
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            src = bits(chain.up_full) if name == "down" else h_bits
            rep = ob.check_outputs(og.bf16_projection64(src, bits(entry[name][0])), got[name].float().cpu().numpy(),
                                   output_dtype="bf16")
            passed &= bool(rep["passed"]) and rep["max_ulp_error"] <= 1
            worst = max(worst, int(rep["max_ulp_error"]))
            checked += int(rep["elements_checked"])
        h_bits = bits(h)
        del chain, h, got
        torch.cuda.empty_cache()
    return {"layers_checked": 2, "elements_checked": checked, "passed": passed, "max_ulp_error": worst,
            "against": "FP64 oracle, check_outputs interval + <= 1 bf16 ulp"}


def chain_timeline(tr, per_layer, kinds):
    """Summary of one traced persistent step, tr [stages, CTAs, slots] of global-timer ns
    (slots: entered, previous stage done in the CTA, x staged, then per warp: first item
    landed, run computed, done). Layer 0 is left out (cold). Per stage kind, medians over
    stages and CTAs: barrier (entered -> every warp done with the previous stage), staging
    (-> x staged, including the wait for a gathered input), first_wait (staged -> a warp's
    first item landed), run (-> its last item computed), cta_span (staged -> the CTA's last
    warp done), enter_skew (first to last CTA entering the stage); per layer: time, and the
    spread of per-CTA busy time (staged -> last warp done, summed over the layer)."""
    import numpy as np

    stages, ctas, _ = tr.shape
    layers = stages // per_layer
    if layers < 2:
        return None
    out = {"per_layer_us": round(float((tr[-1, :, 5::3].max() - tr[per_layer, :, 0].min()) / 1e3 / (layers - 1)), 2)}
    busy = np.zeros(ctas)
    rows = {}
    for s in range(per_layer, stages):
        e, b, x_ = tr[s, :, 0], tr[s, :, 1], tr[s, :, 2]
        first, run, done = tr[s, :, 3::3], tr[s, :, 4::3], tr[s, :, 5::3]
        held = first > 0
        busy += (done.max(axis=1) - x_) / 1e3
        rows.setdefault(kinds[s % per_layer], []).append({
            "barrier_us": np.median(b - e) / 1e3, "staging_us": np.median(x_ - b) / 1e3,
            "first_wait_us": np.median((first - x_[:, None])[held]) / 1e3,
            "run_us": np.median((run - first)[held]) / 1e3,
            "cta_span_us": np.median(done.max(axis=1) - x_) / 1e3,
            "enter_skew_us": (e.max() - e.min()) / 1e3})
    out["stages"] = {k: {m: round(float(np.median([r[m] for r in v])), 2) for m in v[0]} for k, v in rows.items()}
    out["cta_busy_per_layer_us_p0_50_100"] = [round(float(q), 2) for q in np.percentile(busy / (layers - 1), [0, 50, 100])]
    return out


# ---------------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    """The reference's CPU implementation of the path (torch F.linear on CPU BF16, all host
    cores) on rank 0; other ranks exit without work."""
    if rank != 0:
        return 0
    seconds = max(3.0, min(30.0, 2.0 * (args.steps + args.warmup) / 10.0))
    base = cpu_reference_tok_s(seconds)
    line = {"metric": METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000.0 / base["value"], 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "c5_chain_llama3_8b_shapes_32_layers_m1", "layers": 32, "M": 1,
                       "hidden": 4096, "ffn": 14336, "kv": 1024,
                       "parallelism": f"column-shard x{world}" if world > 1 else "column-shard x1",
                       "bytes_per_token": 13_958_643_712},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- main

def main(argv=None):
    parser = argparse.ArgumentParser(description="B200 projection-path benchmark")
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=300)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--layers", type=int, default=32)
    parser.add_argument("--no-projections", action="store_true", help="skip the per-config projection lines")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--quick", action="store_true", help="fewer rounds and shapes (smoke runs)")
    parser.add_argument("--gather", choices=("nccl", "p2p"), default="p2p",
                        help="N>1: NCCL all-gathers, or gathers fused into the projections over NVLink")
    parser.add_argument("--trace", action="store_true",
                        help="persistent chain: after the timed steps, record one step's global-timer "
                             "stamps (ProjectionChain.trace_step) and add a per-stage summary (not timed)")
    parser.add_argument("--stages-per-layer", type=int, choices=(2, 4), default=2,
                        help="persistent chain: stages per layer (ProjectionChain.persistent_schedule)")
    parser.add_argument("--persistent", action=argparse.BooleanOptionalAction, default=None,
                        help="the whole token step as one persistent kernel launch "
                             "(default: with several GPUs; one launch per stage on one GPU)")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch

    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False

    from klab_b200 import _native
    from klab_b200.chain import ChainShape, ProjectionChain

    if args.persistent is None:
        args.persistent = world > 1
    peak, peak_kind = measured_peak()
    shape = ChainShape(layers=args.layers)
    chain = ProjectionChain(shape, rank=rank, world=world, group=group, seed=0, gather=args.gather,
                            persistent=args.persistent, stages_per_layer=args.stages_per_layer)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234)
    x = torch.randn((1, shape.hidden), generator=gen, device="cuda").to(torch.bfloat16)
    out = chain.capture(x)
    for _ in range(args.warmup):
        chain.replay()
    torch.cuda.synchronize()
    barrier(world)

    sampler = ClockSampler(gpu_uuid(torch, local)).start() if rank == 0 else None
    time.sleep(0.2 if sampler else 0.0)
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    torch.cuda.nvtx.range_push("chain")      # the timed token steps
    e0.record(stream)
    for _ in range(args.steps):
        chain.replay()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    t1 = time.perf_counter()
    barrier(world)
    torch.cuda.synchronize()
    local_s = e0.elapsed_time(e1) / 1000.0
    step_s = all_max(torch, local_s, world)
    clocks = None
    if sampler is not None:
        time.sleep(0.1)
        sampler.stop()
        clocks = sampler.summary(t0, t1)
    digest = hashlib.sha256(out.view(torch.int16).cpu().numpy().tobytes()).hexdigest()

    # End to end through the public API: pinned host token in, host result out, per step.
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    e2e_steps = max(20, args.steps // 3)
    barrier(world)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    for _ in range(e2e_steps):
        chain.static_x.copy_(x_host, non_blocking=True)
        chain.replay()
        y_host.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    t3 = time.perf_counter()
    e2e_s = all_max(torch, t3 - t2, world)

    timeline = None
    if args.trace and args.persistent:
        tr = chain.trace_step(x)            # every rank runs the traced step
        if rank == 0:
            timeline = chain_timeline(tr.numpy(), len(chain.persistent_schedule()),
                                      [kind for kind, _ in chain.persistent_schedule()])
        barrier(world)

    launches = chain.launches_per_step()
    roofline = bench_dominant_kernel(torch, chain, peak)
    roofline["peak_kind"] = peak_kind
    status = _native.device_status(clear=True)

    projections = attention = prefetch = None
    if world == 1 and not args.no_projections:
        del chain
        torch.cuda.empty_cache()
        chain = None
        projections = bench_projections(torch, peak, quick=args.quick)
        attention = bench_decode_attention(torch, peak, quick=args.quick)
        prefetch = bench_prefetch(torch, quick=args.quick)

    cpu = parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        seconds = 10.0 if not args.quick else 3.0
        cpu = cpu_reference_tok_s(seconds)
        cpu["oracle_fp64"] = cpu_oracle_tok_s(seconds)
        parity = chain_parity(torch)

    if rank == 0:
        value = args.steps / step_s
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_s * 1000.0 / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02^2) bf16 weights, N(0,1) bf16 token)",
            "config": {"workload": "c5_chain_llama3_8b_shapes_32_layers_m1", "layers": shape.layers, "M": 1,
                       "hidden": shape.hidden, "ffn": shape.ffn, "kv": shape.kv,
                       "parallelism": f"column-shard x{world}" + (
                           {"nccl": " + nccl all-gather", "p2p": " + all-gather fused into the projections "
                            "(NVLink peer stores)"}[args.gather] if world > 1 else ""),
                       "bytes_per_token": shape.bytes_per_token(),
                       "l2": "weights 13.96 GB per step >> 126 MB L2 (no flush needed)",
                       "graph": ("one CUDA graph per token step: input copy + one persistent chain kernel"
                                 if args.persistent else "one CUDA graph per token step, PDL launches")},
            "gpu_launches": args.steps * launches,
            "hbm_gbs_per_gpu": round(shape.bytes_per_token() / world * value / 1e9, 1),
            "roofline": roofline,
            "e2e": {"value": round(e2e_steps / e2e_s, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": int(x_host.numel() * x_host.element_size()),
                    "d2h_bytes_per_step": int(y_host.numel() * y_host.element_size())},
            "clocks": clocks, "output_sha256": digest, "device_status": status,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if parity is not None:
            line["parity"] = parity
        if projections is not None:
            line["projections"] = projections
        if attention is not None:
            line["decode_attention"] = attention
        if prefetch is not None:
            line["l2_prefetch"] = prefetch
        if timeline is not None:
            line["timeline"] = timeline
        print(json.dumps(line), flush=True)

    if chain is not None:
        chain.release()
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
