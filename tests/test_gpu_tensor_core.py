"""Token tiles on the tcgen05 tensor cores: INT8 per-row weights (default for
M >= 2) and BF16 weights (option 2) against the FP64 oracle (the projection
contract: atol 1e-5 + rtol 1e-4, BF16 outputs rounded into that interval) and
against the CUDA-core kernel. Ragged rows, K not a multiple of the 64-column
stage, and several token tiles are covered."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu


@pytest.fixture
def native():
    from klab_b200 import _native

    _native.lib()
    yield _native
    _native.set_option(_native.OPT_TENSOR, 1)
    assert _native.device_status(clear=True) == 0


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("m,n,k", [(4, 14336 // 8, 4096), (16, 1000, 4112), (2, 128, 64), (17, 300, 2048),
                                   (33, 256, 1024)])
@pytest.mark.parametrize("out", ["bf16", "fp32"])
def test_int8_row_tensor_core_matches_oracle(native, m, n, k, out):
    from klab_b200 import int8_weights as iw

    w = torch.from_numpy(og.normal_f32(n + k, (n, k), 0.02)).cuda()
    q = iw.quantize_weights_per_row(w)
    x_bits = og.normal_bf16_bits(m * 31 + k, (m, k), 1.0)
    x = _bf16(x_bits)
    odt = torch.bfloat16 if out == "bf16" else torch.float32
    native.set_option(native.OPT_TENSOR, 2)          # tensor cores for every M >= 2
    y = iw.fused_linear(x, q.codes, q.scales, output_dtype=odt)
    native.set_option(native.OPT_TENSOR, 0)
    y_cc = iw.fused_linear(x, q.codes, q.scales, output_dtype=odt)
    torch.cuda.synchronize()
    codes = q.codes.cpu().numpy().astype(np.float64)
    scales = q.scales.cpu().numpy().astype(np.float64)
    ref = (ob.bf16_values(x_bits) @ codes.T) * scales[None, :]
    for got in (y, y_cc):
        report = ob.check_outputs(ref, got.float().cpu().numpy(), output_dtype=out)
        assert report["passed"], report


@pytest.mark.parametrize("m,n,k", [(8, 512, 4096), (16, 4096, 4096), (3, 130, 1024)])
def test_bf16_tensor_core_matches_oracle(native, m, n, k):
    x_bits = og.normal_bf16_bits(m + k, (m, k), 1.0)
    w_bits = og.normal_bf16_bits(n + k + 1, (n, k), 0.02)
    x, w = _bf16(x_bits), _bf16(w_bits)
    native.set_option(native.OPT_TENSOR, 2)
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    native.gemv(native.W_BF16, native.DT_BF16, x, w, None, None, y, native.DT_BF16, m, n, k)
    torch.cuda.synchronize()
    report = ob.check_outputs(og.bf16_projection64(x_bits, w_bits), y.float().cpu().numpy(), output_dtype="bf16")
    # Tensor-core FP32 accumulation stays inside the contract's interval; near-zero
    # outputs can be several BF16 ulps away (the CUDA-core path keeps <= 1 ulp).
    assert report["passed"], report


def test_tensor_core_option_values(native):
    native.set_option(native.OPT_TENSOR, 2)
    assert native.get_option(native.OPT_TENSOR) == 2
    with pytest.raises(native.KlabError):
        native.set_option(native.OPT_TENSOR, 4)
