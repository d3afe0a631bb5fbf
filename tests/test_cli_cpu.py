"""The bin/klab launcher and its runner without a GPU: version, problem listing and help,
argument errors (exit 2), the launcher handing the runner's exit status through, and
the new operators' schemas and fake kernels (as the reference's tests/test_cli.py and
dynamic_projection.py fake registrations)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
KLAB = ROOT / "bin" / "klab"


@pytest.fixture(scope="module", autouse=True)
def launcher():
    from klab_b200.build import build_launcher

    build_launcher()
    assert KLAB.exists()


def run(*args, cwd=ROOT, env=None):
    return subprocess.run([str(KLAB), *args], cwd=cwd, env=env, capture_output=True, text=True, timeout=120)


def test_version_problems_and_help_need_no_gpu():
    r = run("version")
    assert r.returncode == 0 and r.stdout.startswith("klab-b200")
    r = run("problems", "--json")
    assert r.returncode == 0, r.stderr
    ids = [p["id"] for p in json.loads(r.stdout)]
    assert ids[0] == "bf16-projection" and "projection-chain" in ids
    r = run("help", "run")
    assert r.returncode == 0 and "--shape" in r.stdout
    r = run("show", "fp4-projection", "--json")
    assert r.returncode == 0 and json.loads(r.stdout)["config"] == "c3"


@pytest.mark.parametrize("args", [("run", "--output", "../escape.json"), ("run", "--output", "/tmp/x.json"),
                                  ("run", "--output", "results/notes.md"), ("run", "--shape", "1,2"),
                                  ("nonsense",), ("run", "no-such-problem"), ("profile", "--shape", "1,2"),
                                  ("profile", "int8-projection", "--calls", "0"), ("profile", "projection-chain"),
                                  ("profile", "decode-step", "--length", "4096")])
def test_usage_errors_exit_2_before_any_gpu_work(args):
    r = run(*args)
    assert r.returncode == 2, (r.stdout, r.stderr)


def test_launcher_propagates_exit_status(tmp_path):
    """A project whose interpreter exits 23: the launcher execs it, so its status is ours."""
    (tmp_path / "klab_b200").mkdir()
    (tmp_path / "klab_b200" / "cli.py").touch()
    (tmp_path / "klab_b200" / "kernel_lab.py").touch()
    python = tmp_path / ".venv" / "bin" / "python"
    python.parent.mkdir(parents=True)
    python.write_text("#!/bin/sh\nexit 23\n")
    python.chmod(0o755)
    assert run("--project", str(tmp_path), "check").returncode == 23
    env = dict(os.environ, KERNEL_LAB_ROOT=str(tmp_path))
    assert run("problems", env=env).returncode == 23


def test_launcher_finds_its_project_from_any_directory(tmp_path):
    env = dict(os.environ)
    env.pop("KERNEL_LAB_ROOT", None)
    r = run("problems", "--json", cwd=tmp_path, env=env)
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout)[0]["id"] == "bf16-projection"


def test_launcher_rejects_a_directory_that_is_not_a_project(tmp_path):
    r = run("--project", str(tmp_path), "problems")
    assert r.returncode == 2 and "not a klab-b200 project" in r.stderr


def test_runner_module_matches_launcher():
    r = subprocess.run([sys.executable, "-m", "klab_b200.cli", "problems", "--json"], cwd=ROOT,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and json.loads(r.stdout) == json.loads(run("problems", "--json").stdout)


def test_dynamic_operators_schemas_and_fake_kernels():
    from torch._subclasses.fake_tensor import FakeTensorMode

    from klab_b200 import dynamic_projection  # noqa: F401 - registers the operators

    assert str(torch.ops.kernel_lab.dynamic_vendor.default._schema) == \
        "kernel_lab::dynamic_vendor(Tensor x, Tensor w, str config) -> Tensor"
    assert str(torch.ops.kernel_lab.dynamic_tiny.default._schema) == \
        "kernel_lab::dynamic_tiny(Tensor x, Tensor w, SymInt threads, SymInt vector) -> Tensor"
    with FakeTensorMode():
        x = torch.empty(3, 256, device="cuda", dtype=torch.bfloat16)
        w = torch.empty(40, 256, device="cuda", dtype=torch.bfloat16)
        y = torch.ops.kernel_lab.dynamic_vendor(x, w, "cublas_compute32")
        assert y.shape == (3, 40) and y.dtype == torch.float32
        y = torch.ops.kernel_lab.dynamic_vendor(x, w.T.contiguous(), "cublas_packed_compute32")
        assert y.shape == (3, 40)
        y = torch.ops.kernel_lab.dynamic_tiny(x.float(), w.float(), 64, 4)
        assert y.shape == (3, 40)


def test_vendor_call_rejects_bad_arguments_on_cpu_tensors():
    from klab_b200.vendor import vendor_call

    x, w = torch.zeros(1, 8), torch.zeros(4, 8)
    with pytest.raises(ValueError):
        vendor_call(x, w, "not_a_config")
    with pytest.raises(ValueError):
        vendor_call(x, w, "cublas_mm")   # CPU tensors
