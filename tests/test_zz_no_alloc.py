"""klab_raw_linear_noalloc: the projection for callers that cannot allocate
device memory (it takes its split-K scratch from a static array inside the
library). Called through the C ABI with ctypes; its output must equal the
allocating entry point's on shapes that split K, on two calls in a row. This
file is collected last so a failure here never hides another test."""

import ctypes as ct

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu


def _dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("m,n,k", [(1, 40, 14336), (3, 24, 10240), (1, 512, 8192)])
def test_noalloc_matches_allocating_entry_point(m, n, k):
    from klab_b200 import _native

    lib = _native.lib()
    assert lib.klab_gemv_workspace_bytes(_native.W_BF16, m, n, k) > 0  # these shapes can split K
    x_bits = og.normal_bf16_bits(100 + m, (m, k), 1.0)
    w_bits = og.normal_bf16_bits(200 + n, (n, k), 0.02)
    x, w = _dev(x_bits), _dev(w_bits)
    stream = torch.cuda.current_stream().cuda_stream

    # Reference output: the allocating C entry point with a caller-owned workspace.
    need = lib.klab_gemv_workspace_bytes(_native.W_BF16, m, n, k)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    expected = torch.empty((m, n), dtype=torch.float32, device="cuda")
    assert lib.klab_raw_linear(x.data_ptr(), w.data_ptr(), expected.data_ptr(), _native.DT_F32, m, n, k,
                               ws.data_ptr(), need, stream) == 0

    for _ in range(2):  # two calls in a row share (and must re-clear) the static scratch
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.klab_raw_linear_noalloc(x.data_ptr(), w.data_ptr(), out.data_ptr(), _native.DT_F32, m, n, k,
                                         stream)
        assert rc == 0, _native.error_string(rc)
        torch.cuda.synchronize()
        report = ob.check_outputs(og.bf16_projection64(x_bits, w_bits), out.cpu().numpy(), output_dtype="fp32")
        assert report["passed"], report
        np.testing.assert_allclose(out.cpu().numpy(), expected.cpu().numpy(), rtol=1e-4, atol=1e-5)
        assert torch.equal(out.view(torch.int32), expected.view(torch.int32))
    assert _native.device_status(clear=True) == 0


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    from klab_b200 import _native

    lib = _native.lib()
    m, n, k = 16, 14336, 65536  # split-K scratch far above 4 MiB
    assert lib.klab_gemv_workspace_bytes(_native.W_BF16, m, n, k) > 4 << 20
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    rc = lib.klab_raw_linear_noalloc(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), _native.DT_F32, m, n, k,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == _native.E_SCRATCH
    assert "4 MiB" in _native.error_string(rc)
