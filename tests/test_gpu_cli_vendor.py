"""On the GPU: every vendor route of kernel_lab::dynamic_vendor against the FP64
oracle (FP32 outputs within check_outputs), torch.library.opcheck of the two dynamic
operators, and bin/klab run / check end to end (JSON out, exit status)."""

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("config", ["torch_mm", "torch_mv", "torch_mm_out_fp32", "cublas_mm", "cublas_mv",
                                    "cublas_packed_mm", "cublas_packed_mv", "cublas_compute32",
                                    "cublas_packed_compute32"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_vendor_routes_match_oracle(config, dtype):
    from klab_b200 import dynamic_projection as dp

    if dtype != torch.float32 and config in ("cublas_mm", "cublas_mv", "cublas_packed_mm", "cublas_packed_mv"):
        pytest.skip("FP32-only route")
    m = 1 if config.endswith("_mv") else 3
    n, k = 72, 512
    x = torch.from_numpy(og.normal_f32(1, (m, k))).to(dtype).cuda()
    w = torch.from_numpy(og.normal_f32(2, (n, k), 0.05)).to(dtype).cuda()
    wt = w.T.contiguous() if "packed" in config else w
    torch.backends.cuda.matmul.allow_tf32 = False
    y = dp.dynamic_vendor(x, wt, config)
    assert y.dtype == torch.float32 and y.shape == (m, n)
    ref = og.projection64(x.double().cpu().numpy(), w.double().cpu().numpy())
    report = ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], (config, report)
    out = torch.empty(m, n, device="cuda")
    assert torch.equal(dp.vendor_call(x, wt, config, out), y)


def test_dynamic_operators_opcheck():
    from klab_b200 import dynamic_projection  # noqa: F401

    x = torch.randn(2, 256, device="cuda")
    w = torch.randn(48, 256, device="cuda") * 0.05
    torch.library.opcheck(torch.ops.kernel_lab.dynamic_vendor.default, (x, w, "cublas_mm"))
    torch.library.opcheck(torch.ops.kernel_lab.dynamic_tiny.default, (x, w, 64, 4))
    ref = og.projection64(x.double().cpu().numpy(), w.double().cpu().numpy())
    y = torch.ops.kernel_lab.dynamic_tiny(x, w, 64, 4)
    assert ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")["passed"]


def test_klab_run_and_check_end_to_end(tmp_path):
    from klab_b200.build import build_launcher

    klab = build_launcher()
    # The launcher runs in the project root (like the reference's), so --output is relative to it;
    # build/ is ignored by git.
    result = ROOT / "build" / "klab_run_test.json"
    r = subprocess.run([str(klab), "run", "bf16-projection", "--shape", "1,2048,4096", "--rounds", "3", "--json",
                        "--output", "build/klab_run_test.json"], cwd=tmp_path, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    row = json.loads(r.stdout)
    assert row["shape_mnk"] == [1, 2048, 4096] and row["us"] > 0 and row["cublas_us"] > 0
    assert json.loads(result.read_text())["us"] == row["us"]
    result.unlink()
    r = subprocess.run([str(klab), "check", "fp4-projection", "--json"], cwd=ROOT, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, (r.stdout, r.stderr)
    summary = json.loads(r.stdout)
    assert summary["status"] == "passed" and summary["passed"] >= 2 and summary["failed"] == 0


@pytest.mark.parametrize("m,n,k,out", [(1, 4096, 4096, torch.bfloat16), (4, 1024, 2048, torch.float32)])
def test_frozen_cublaslt_plan_round_trip(m, n, k, out):
    """tune -> freeze -> restore: the restored plan runs the same algorithm (same bits) and
    both meet the FP64 oracle; a record restored with another shape is refused."""
    import json

    from klab_b200 import lt_baseline as lt

    x = torch.from_numpy(og.normal_f32(1, (m, k))).to(torch.bfloat16).cuda()
    w = torch.from_numpy(og.normal_f32(2, (n, k), 0.02)).to(torch.bfloat16).cuda()
    plan = lt.tune_plan(x, w, out, rounds=3)
    y = torch.empty(m, n, device="cuda", dtype=out)
    plan.run(x, w, y)
    record = json.loads(json.dumps(plan.freeze()))
    again = lt.LtPlan.restore(record, x.device)
    y2 = torch.empty_like(y)
    again.run(x, w, y2)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.uint8), y2.view(torch.uint8))
    ref = og.projection64(x.double().cpu().numpy(), w.double().cpu().numpy())
    report = ob.check_outputs(ref, y.float().cpu().numpy(), output_dtype="bf16" if out == torch.bfloat16 else "fp32")
    assert report["passed"], report
    with pytest.raises(ValueError):
        lt.validate_frozen(record, lt.runtime_context(x.device, x.dtype, out, m + 1, n, k))


@pytest.mark.parametrize("args", [("int8-projection", "--shape", "4,1000,2048"), ("fp4-projection", "--shape", "8,512,4096"),
                                  ("lossless-bf16-projection", "--shape", "1,256,1024"), ("decode-step", "--length", "300")])
def test_klab_profile_runs_a_case(args):
    from klab_b200 import cli

    assert cli.main(["profile", *args, "--calls", "2"]) == 0
