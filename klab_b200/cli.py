"""Command-line runner behind bin/klab (the role of the reference's experiments.py for
this path: `klab check` -> numerical checks, `klab run` -> a timed projection;
native/cli.cpp:37-44 execs experiments.py, experiments.py:253-334 dispatches).

    klab problems [--json]                 the path's problems
    klab show <problem> [--json]           what a problem covers
    klab doctor [--json]                   device, library and toolchain
    klab check [problem] [--all] [--json]  the parity suite for a problem (GPU tests
                                           against the FP64 oracle); exit 1 if any fails
    klab run [problem] [--shape M,N,K] [--rounds R] [--seed S] [--output FILE] [--json]
                                           time one projection (or the chain) the way
                                           the benchmark does, beside cuBLAS
    klab profile [problem] [--shape M,N,K] [--length L] [--calls C]
                                           a few calls of one case on one weight set,
                                           for a profiler (ncu -k ... -s/-c); not timed
    klab version | help [command]

Exit status: 0 success, 1 a failed check or a runtime error, 2 a usage error
(including an --output path that leaves the working directory or names a .md file).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import xml.etree.ElementTree as ET
from pathlib import Path

VERSION = "klab-b200 0.2.0"
ROOT = Path(__file__).resolve().parents[1]

PROBLEMS = [
    {"id": "bf16-projection", "config": "c1", "default_shape": (1, 4096, 4096),
     "precision": "BF16 weights and activations, FP32 accumulation, one RNE to BF16",
     "description": "Streaming BF16 projection (and its M-tiles) versus cuBLAS",
     "tests": ["tests/test_gpu_projections.py", "tests/test_gpu_baseline_configs.py::test_c1_bf16_4096x4096_m1",
               "tests/test_gpu_prepared.py", "tests/test_gpu_half_x.py"]},
    {"id": "int8-projection", "config": "c2", "default_shape": (1, 14336, 4096),
     "precision": "INT8 weights (per-row or per-64 FP32 scales), FP32 accumulation",
     "description": "INT8 weight-only projection: CUDA-core, warp-level tensor-core and tcgen05 token tiles",
     "tests": ["tests/test_gpu_baseline_configs.py::test_c2_int8_per_row_14336x4096",
               "tests/test_gpu_tensor_core.py", "tests/test_gpu_tile_mma.py"]},
    {"id": "fp4-projection", "config": "c3", "default_shape": (1, 8192, 8192),
     "precision": "E2M1 weights (FP16/32 or E4M3/16 + global scales), FP32 accumulation",
     "description": "FP4 weight projection with decode in registers; warp-level tensor-core token tiles at M >= 2",
     "tests": ["tests/test_gpu_baseline_configs.py::test_c3_fp4_f16_scale_8192x8192", "tests/test_gpu_tile_mma.py"]},
    {"id": "lossless-bf16-projection", "config": "c4", "default_shape": (1, 4096, 4096),
     "precision": "Exact BF16 (lossless exponent coding), FP32 accumulation",
     "description": "Lossless-coded BF16 projection, bit-identical to the raw projection",
     "tests": ["tests/test_gpu_baseline_configs.py::test_c4_lossless_bf16_eight_layers"]},
    {"id": "projection-chain", "config": "c5", "default_shape": (1, 4096, 4096),
     "precision": "BF16, every projection output rounded once to BF16",
     "description": "32-layer Llama-3-8B-shaped projection chain in one CUDA graph",
     "tests": ["tests/test_gpu_baseline_configs.py::test_c5_chain_first_two_layers", "tests/test_gpu_peer.py",
               "tests/test_gpu_multi.py"]},
    {"id": "fp32-projection", "config": None, "default_shape": (1, 4096, 4096),
     "precision": "FP32 equivalent (plain and lossless FP32 weights)",
     "description": "FP32 projections, lossless FP32 formats and residual RMSNorm",
     "tests": ["tests/test_gpu_lossless.py", "tests/test_gpu_rmsnorm.py"]},
    {"id": "decode-step", "config": None, "default_shape": None,
     "precision": "BF16 in, FP32 softmax and accumulation",
     "description": "Decode attention with the KV append, prologue fusions, fused multi-output projections",
     "tests": ["tests/test_gpu_decode_attn.py", "tests/test_gpu_decode_ops.py", "tests/test_gpu_kv_pair.py",
               "tests/test_gpu_prefetch_tuning.py"]},
]
_BY_ID = {p["id"]: p for p in PROBLEMS}
CPU_TESTS = ["tests/test_oracle_golden.py", "tests/test_prepared_cpu.py", "tests/test_cpu_native.py"]


class UsageError(Exception):
    """Bad arguments: exit status 2."""


def parser():
    p = argparse.ArgumentParser(prog="klab", description="B200 small-batch projection path")
    sub = p.add_subparsers(dest="command", required=True)
    for name in ("problems", "doctor"):
        sub.add_parser(name).add_argument("--json", action="store_true")
    show = sub.add_parser("show")
    show.add_argument("problem", choices=list(_BY_ID))
    show.add_argument("--json", action="store_true")
    check = sub.add_parser("check", aliases=["verify"])
    check.add_argument("problem", nargs="?", default="bf16-projection", choices=list(_BY_ID))
    check.add_argument("--all", action="store_true", help="every problem, plus the CPU oracle pins")
    check.add_argument("--json", action="store_true")
    run = sub.add_parser("run", aliases=["bench"])
    run.add_argument("problem", nargs="?", default="bf16-projection", choices=list(_BY_ID))
    run.add_argument("--shape", help="M,N,K (projection problems)")
    run.add_argument("--layers", type=int, default=32, help="projection-chain: decoder layers")
    run.add_argument("--rounds", type=int, default=15)
    run.add_argument("--seed", type=int, default=0)
    run.add_argument("--output", help="also write the JSON result to this file (under the working directory)")
    run.add_argument("--json", action="store_true")
    sub.add_parser("version")
    prof = sub.add_parser("profile")
    prof.add_argument("problem", nargs="?", default="bf16-projection", choices=list(_BY_ID))
    prof.add_argument("--shape", help="M,N,K (projection problems)")
    prof.add_argument("--length", type=int, default=4095, help="decode-step: cached tokens (capacity 4096)")
    prof.add_argument("--calls", type=int, default=4)
    prof.add_argument("--seed", type=int, default=1)
    helper = sub.add_parser("help")
    helper.add_argument("topic", nargs="?")
    return p


def _output_path(text):
    """An --output path inside the working directory that is not a Markdown file."""
    if text is None:
        return None
    path = Path(text)
    resolved = (Path.cwd() / path).resolve()
    if path.is_absolute() or ".." in path.parts or Path.cwd().resolve() not in resolved.parents:
        raise UsageError(f"--output must stay inside the working directory: {text}")
    if resolved.suffix.lower() == ".md":
        raise UsageError("--output must not be a Markdown file")
    return resolved


def _shape(text, default):
    if text is None:
        return default
    try:
        m, n, k = (int(v) for v in text.split(","))
    except ValueError:
        raise UsageError("--shape takes M,N,K") from None
    if min(m, n, k) <= 0:
        raise UsageError("--shape values must be positive")
    return m, n, k


def cmd_problems(args):
    rows = [{k: v for k, v in p.items() if k != "tests"} for p in PROBLEMS]
    if args.json:
        print(json.dumps(rows))
    else:
        for p in rows:
            print(f"{p['id']:26s} {p['description']}")
    return 0


def cmd_show(args):
    p = _BY_ID[args.problem]
    print(json.dumps(p, indent=None if args.json else 2))
    return 0


def cmd_doctor(args):
    import torch

    from . import _native

    info = {"version": VERSION, "library": str(_native.LIB_PATH), "torch": torch.__version__,
            "cuda_runtime": torch.version.cuda, "cuda_available": torch.cuda.is_available()}
    if torch.cuda.is_available():
        props = torch.cuda.get_device_properties(0)
        info.update(device=props.name, capability=list(torch.cuda.get_device_capability(0)),
                    sms=props.multi_processor_count, memory_gib=round(props.total_memory / 2 ** 30, 1))
        _native.lib()
    print(json.dumps(info, indent=None if args.json else 2))
    return 0


def _junit_counts(path):
    root = ET.parse(path).getroot()
    suites = [root] if root.tag == "testsuite" else list(root)
    totals = {"tests": 0, "failures": 0, "errors": 0, "skipped": 0}
    failed = []
    for suite in suites:
        for key in totals:
            totals[key] += int(suite.get(key, 0))
        for case in suite.iter("testcase"):
            if case.find("failure") is not None or case.find("error") is not None:
                failed.append(f"{case.get('classname')}::{case.get('name')}")
    return totals, failed


def cmd_check(args):
    problems = PROBLEMS if args.all else [_BY_ID[args.problem]]
    selections = sorted({t for p in problems for t in p["tests"]})
    if args.all:
        selections = CPU_TESTS + selections
    with tempfile.TemporaryDirectory() as tmp:
        report = Path(tmp) / "junit.xml"
        cmd = [sys.executable, "-m", "pytest", *selections, "-q", "-p", "no:cacheprovider", f"--junitxml={report}"]
        proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
        if not report.exists():
            raise RuntimeError(f"the test runner produced no report (exit {proc.returncode}):\n{proc.stdout[-2000:]}"
                               f"{proc.stderr[-2000:]}")
        totals, failed = _junit_counts(report)
    bad = totals["failures"] + totals["errors"]
    passed = totals["tests"] - bad - totals["skipped"]
    status = "failed" if bad or proc.returncode not in (0, 5) else ("passed" if passed else "skipped")
    result = {"problems": [p["id"] for p in problems], "status": status, "passed": passed, "failed": bad,
              "skipped": totals["skipped"], "selections": selections, "failures": failed}
    if args.json:
        print(json.dumps(result))
    else:
        print(f"{status}: {passed} passed, {bad} failed, {totals['skipped']} skipped "
              f"({', '.join(result['problems'])})")
        for name in failed:
            print(f"  FAILED {name}")
    return 1 if status == "failed" else 0


def _run_projection(problem, m, n, k, rounds, seed):
    """µs per call of this library's projection and of cuBLAS (F.linear on BF16 weights,
    dequantized for INT8/FP4) over cold-L2 rings of distinct weights."""
    import torch
    import torch.nn.functional as F

    from . import compressed_bf16 as cb
    from . import fp4, int8_weights, measure

    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
    w32 = torch.randn((n, k), generator=gen, device="cuda").mul_(0.02)
    out = torch.empty((m, n), device="cuda", dtype=torch.bfloat16)
    if problem in ("bf16-projection", "lossless-bf16-projection"):
        w = w32.to(torch.bfloat16)
        if problem == "bf16-projection":
            nbytes = n * k * 2
            ops = [w.clone() for _ in range(measure.ring_count(nbytes))]
            ours = lambda i: cb.raw_linear(x, ops[i], threads=128, vector=8, output_dtype="bf16", out=out)  # noqa
        else:
            if k % 64:
                raise UsageError("lossless-bf16-projection needs K % 64 == 0")
            packed = cb.upload(cb.pack_bits(w.view(torch.int16).cpu().numpy().view("uint16")), "cuda")
            nbytes = packed.storage_bytes
            ops = [packed] + [cb.PackedBF16(packed.payload.clone(), packed.metadata.clone(), n, k,
                                            packed.source_sha256, 1, packed.module)
                              for _ in range(measure.ring_count(nbytes) - 1)]
            ours = lambda i: cb.fused_linear(x, ops[i], threads=128, vector=8, output_dtype="bf16", out=out)  # noqa
        vendor_w = [w.clone() for _ in range(measure.ring_count(n * k * 2))]
    elif problem == "int8-projection":
        q = int8_weights.quantize_weights_per_row(w32)
        nbytes = n * k + n * 4
        ops = [q.codes.clone() for _ in range(measure.ring_count(n * k))]
        ours = lambda i: int8_weights.fused_linear(x, ops[i], q.scales, out=out, output_dtype=torch.bfloat16)  # noqa
        deq = q.dequantize().to(torch.bfloat16)
        vendor_w = [deq.clone() for _ in range(measure.ring_count(n * k * 2))]
    elif problem == "fp4-projection":
        if k % 32:
            raise UsageError("fp4-projection needs K % 32 == 0")
        q = fp4.quantize_weights_f16(w32)
        nbytes = n * k // 2 + n * k // 16
        ops = [(q.packed.clone(), q.scales.clone()) for _ in range(measure.ring_count(nbytes))]
        ours = lambda i: fp4.fused_linear(x, ops[i][0], ops[i][1], None, out=out,  # noqa
                                          output_dtype=torch.bfloat16)
        deq = q.dequantize().to(torch.bfloat16)
        vendor_w = [deq.clone() for _ in range(measure.ring_count(n * k * 2))]
    else:
        raise UsageError(f"klab run does not time {problem}")
    del w32
    nbytes += m * k * 2 + m * n * 2
    us = measure.time_ring(ours, len(ops), rounds)
    vus = measure.time_ring(lambda i: F.linear(x, vendor_w[i]), len(vendor_w), rounds)
    return {"problem": problem, "shape_mnk": [m, n, k], "us": round(us, 3), "bytes": nbytes,
            "gbs": round(nbytes / us / 1e3, 1), "cublas_us": round(vus, 3), "speedup_vs_cublas": round(vus / us, 3),
            "rounds": rounds, "ring": len(ops)}


def _run_chain(layers, rounds):
    import torch

    from . import measure
    from .chain import ChainShape, ProjectionChain

    shape = ChainShape(layers=layers)
    chain = ProjectionChain(shape, seed=0)
    x = torch.randn((1, shape.hidden), device="cuda").to(torch.bfloat16)
    chain.capture(x)
    us = measure.time_graph(chain.graph, 1, rounds)
    chain.release()
    return {"problem": "projection-chain", "layers": layers, "us_per_token": round(us, 2),
            "tokens_per_s": round(1e6 / us, 2), "gbs": round(shape.bytes_per_token() / us / 1e3, 1)}


def cmd_run(args):
    output = _output_path(args.output)
    problem = _BY_ID[args.problem]
    if args.rounds < 3:
        raise UsageError("--rounds must be at least 3")
    if args.problem not in ("projection-chain", "bf16-projection", "int8-projection", "fp4-projection",
                            "lossless-bf16-projection"):
        raise UsageError(f"klab run does not time {args.problem}; see klab check {args.problem}")
    shape = None if args.problem == "projection-chain" else _shape(args.shape, problem["default_shape"])
    if args.layers <= 0:
        raise UsageError("--layers must be positive")
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable; klab run times the GPU path")
    if shape is None:
        result = _run_chain(args.layers, args.rounds)
    else:
        result = _run_projection(args.problem, *shape, args.rounds, args.seed)
    result["device"] = torch.cuda.get_device_name()
    text = json.dumps(result)
    if output is not None:
        output.parent.mkdir(parents=True, exist_ok=True)
        output.write_text(text + "\n")
    print(text if args.json else json.dumps(result, indent=2))
    return 0


def _profile_case(problem, shape, length, seed):
    """A zero-argument callable running one call of the case: seeded synthetic weights and
    activations with the benchmark configs' distributions (W ~ N(0, 0.02^2), x ~ N(0, 1)), one
    weight set, so a profiler captures the kernel without rings of copies around it."""
    import torch

    from . import compressed_bf16 as cb
    from . import fp4, int8_weights

    gen = torch.Generator(device="cuda").manual_seed(seed)

    def normal(dims, std=1.0):
        return torch.randn(dims, generator=gen, device="cuda").mul_(std)

    if problem == "decode-step":
        from .decode_attn import decode_attention

        if not 0 <= length < 4096:
            raise UsageError("--length must be in [0, 4096)")
        kc, vc = normal((8, 4096, 64)).to(torch.bfloat16), normal((8, 4096, 64)).to(torch.bfloat16)
        q, kn, vn = (normal((n,)).to(torch.bfloat16) for n in (32 * 64, 8 * 64, 8 * 64))
        return lambda: decode_attention(q, kn, vn, kc, vc, length)
    m, n, k = shape
    x = normal((m, k)).to(torch.bfloat16)
    w32 = normal((n, k), 0.02)
    if problem == "bf16-projection":
        w = w32.to(torch.bfloat16)
        return lambda: cb.raw_linear(x, w, threads=128, vector=8, output_dtype="bf16")
    if problem == "lossless-bf16-projection":
        if k % 64:
            raise UsageError("lossless-bf16-projection needs K % 64 == 0")
        packed = cb.upload(cb.pack_bits(w32.to(torch.bfloat16).view(torch.int16).cpu().numpy().view("uint16")), "cuda")
        return lambda: cb.fused_linear(x, packed, threads=128, vector=8, output_dtype="bf16")
    if problem == "int8-projection":
        q = int8_weights.quantize_weights_per_row(w32)
        return lambda: int8_weights.fused_linear(x, q.codes, q.scales, output_dtype=torch.bfloat16)
    if problem == "fp4-projection":
        if k % 32:
            raise UsageError("fp4-projection needs K % 32 == 0")
        q = fp4.quantize_weights_f16(w32)
        return lambda: q.linear(x, output_dtype=torch.bfloat16)
    raise UsageError(f"klab profile does not run {problem}")


def cmd_profile(args):
    problem = _BY_ID[args.problem]
    if args.calls < 1:
        raise UsageError("--calls must be at least 1")
    if args.problem not in ("bf16-projection", "int8-projection", "fp4-projection", "lossless-bf16-projection",
                            "decode-step"):
        raise UsageError(f"klab profile does not run {args.problem}")
    shape = None if args.problem == "decode-step" else _shape(args.shape, problem["default_shape"])
    if shape is None and not 0 <= args.length < 4096:
        raise UsageError("--length must be in [0, 4096)")
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable; klab profile runs the GPU path")
    fn = _profile_case(args.problem, shape, args.length, args.seed)
    for _ in range(args.calls):
        fn()
    torch.cuda.synchronize()
    print("ok", args.problem, "x".join(map(str, shape)) if shape else f"length {args.length}", f"{args.calls} calls")
    return 0


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv in (["--help"], ["-h"]):
        print(__doc__)
        return 0
    if argv in (["--version"],):
        argv = ["version"]
    try:
        args = parser().parse_args(argv)
    except SystemExit as exit_:
        return int(exit_.code or 0)
    try:
        if args.command == "version":
            print(VERSION)
            return 0
        if args.command == "help":
            if args.topic is None:
                print(__doc__)
            else:
                sub = parser()._subparsers._group_actions[0].choices.get(args.topic)
                if sub is None:
                    raise UsageError(f"no command {args.topic!r}")
                sub.print_help()
            return 0
        handler = {"problems": cmd_problems, "show": cmd_show, "doctor": cmd_doctor, "check": cmd_check,
                   "verify": cmd_check, "run": cmd_run, "bench": cmd_run, "profile": cmd_profile}[args.command]
        return handler(args)
    except UsageError as error:
        print(f"klab: {error}", file=sys.stderr)
        return 2
    except Exception as error:  # noqa: BLE001 - the CLI reports, the library raises
        if os.environ.get("KLAB_DEBUG"):
            raise
        print(f"klab: {error}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())
