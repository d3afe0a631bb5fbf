"""The column-sharded chain on 2 GPUs (NCCL all-gathers, or gathers fused into
the projections over NVLink peer memory, inside a CUDA graph) is bit-identical
to the same chain on one GPU. Needs at least 2 GPUs; the
ranks are separate processes started with torchrun."""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
HELPER = Path(__file__).resolve().parent / "_chain_ranks.py"


def _run(nproc, out, port, mode="nccl"):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(HELPER), str(out), mode]
    result = subprocess.run(["timeout", "-k", "30", "240", *cmd], env=env, capture_output=True, text=True)
    assert result.returncode == 0, result.stdout[-3000:] + result.stderr[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_chain_bit_identical_to_one_gpu(tmp_path):
    _run(1, tmp_path / "one.npy", 29611)
    _run(2, tmp_path / "two.npy", 29612)
    np.testing.assert_array_equal(np.load(tmp_path / "one.npy"), np.load(tmp_path / "two.npy"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_fused_p2p_chain_bit_identical_to_one_gpu(tmp_path):
    _run(1, tmp_path / "one.npy", 29613)
    _run(2, tmp_path / "two.npy", 29614, "p2p")
    np.testing.assert_array_equal(np.load(tmp_path / "one.npy"), np.load(tmp_path / "two.npy"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_persistent_chain_bit_identical_to_one_gpu(tmp_path):
    _run(1, tmp_path / "one.npy", 29615, "persistent")
    _run(1, tmp_path / "ref.npy", 29616)
    _run(2, tmp_path / "two.npy", 29617, "persistent")
    one, ref, two = (np.load(tmp_path / f) for f in ("one.npy", "ref.npy", "two.npy"))
    np.testing.assert_array_equal(one, ref)
    np.testing.assert_array_equal(two, ref)
