"""KernelLab.residual_rmsnorm / kernel_lab::residual_rmsnorm on the GPU against
the FP64 oracle (the reference's fused residual RMSNorm, kernels.cu:168-222),
plus the reference's argument validation (kernel_lab.py:281-294). Tolerance:
the reference's check_outputs interval for FP32 outputs (atol 1e-5 + rtol 1e-4
of the FP64 result)."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def native():
    from klab_b200 import _native

    _native.lib()
    yield _native
    assert _native.device_status(clear=True) == 0


@pytest.mark.parametrize("m,k", [(1, 4096), (3, 8192), (5, 1), (2, 17), (4, 1000), (7, 4104)])
@pytest.mark.parametrize("eps", [1e-6, 1e-3])
def test_matches_fp64_oracle(m, k, eps):
    from klab_b200.kernel_lab import KernelLab

    x = og.normal_f32(m * 3 + k, (m, k))
    r = og.normal_f32(m * 5 + k, (m, k), 0.5)
    w = og.normal_f32(k + 1, (k,), 1.0)
    lab = KernelLab()
    y = lab.residual_rmsnorm(torch.from_numpy(x).cuda(), torch.from_numpy(r).cuda(), torch.from_numpy(w).cuda(),
                             eps=eps, threads=128)
    report = ob.check_outputs(og.residual_rmsnorm64(x, r, w, eps), y.cpu().numpy(), output_dtype="fp32")
    assert report["passed"], report


def test_registered_op_and_out_buffer():
    from klab_b200 import kernel_lab  # noqa: F401  (registers the op)
    from klab_b200.kernel_lab import default_lab

    x = torch.randn(4, 4096, device="cuda")
    r = torch.randn(4, 4096, device="cuda")
    w = torch.randn(4096, device="cuda")
    y = torch.ops.kernel_lab.residual_rmsnorm(x, r, w, 1e-6)
    out = torch.empty_like(x)
    y2 = default_lab().residual_rmsnorm(x, r, w, eps=1e-6, out=out)
    assert y2.data_ptr() == out.data_ptr() and torch.equal(y, y2)
    ref = og.residual_rmsnorm64(x.cpu().numpy(), r.cpu().numpy(), w.cpu().numpy(), 1e-6)
    assert ob.check_outputs(ref, y.cpu().numpy(), output_dtype="fp32")["passed"]


def test_validation_matches_reference():
    from klab_b200.kernel_lab import KernelLab

    lab = KernelLab()
    x = torch.randn(2, 64, device="cuda")
    w = torch.randn(64, device="cuda")
    with pytest.raises(ValueError):
        lab.residual_rmsnorm(x, torch.randn(2, 32, device="cuda"), w)
    with pytest.raises(ValueError):
        lab.residual_rmsnorm(torch.randn(1, 8200, device="cuda"), torch.randn(1, 8200, device="cuda"),
                             torch.randn(8200, device="cuda"))
    with pytest.raises(ValueError):
        lab.residual_rmsnorm(x, x, w, eps=0.0)
    with pytest.raises(ValueError):
        lab.residual_rmsnorm(x, x, w, threads=64)
    with pytest.raises(ValueError):
        lab.residual_rmsnorm(x.half(), x.half(), w.half())
    with pytest.raises(ValueError):
        lab.residual_rmsnorm(x, x, w, out=x)
