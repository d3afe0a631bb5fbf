"""The output gather fused into the projection kernel, on one GPU: a second
local buffer and flag array stand in for the peer's (the kernel stores through
the same pointers it would use for a peer mapping). The gathered copy must equal
the local output bit for bit, the local output must equal a launch without the
gather, flags must carry the step epoch, and a wait for a flag that nothing
raises must end with the flag-timeout status instead of hanging."""

import numpy as np
import pytest
import torch

from oracle import bf16 as ob
from oracle import gemv as og

pytestmark = pytest.mark.gpu

STATUS_FLAG_TIMEOUT = 2


@pytest.fixture(scope="module")
def native():
    from klab_b200 import _native

    _native.lib()
    _native.device_status(clear=True)
    return _native


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def _setup(m, n, k, seed):
    x_bits = og.normal_bf16_bits(seed, (m, k), 1.0)
    w_bits = og.normal_bf16_bits(seed + 1, (n, k), 0.02)
    return x_bits, w_bits, _bf16(x_bits), _bf16(w_bits)


@pytest.mark.parametrize("m,n,k,split", [(1, 512, 4096, 0), (1, 64, 14336, 1), (4, 384, 2048, -1)])
def test_fused_gather_matches_local_output_and_raises_flags(native, m, n, k, split):
    x_bits, w_bits, x, w = _setup(m, n, k, 100 + n)
    native.set_option(native.OPT_SPLIT, split)
    try:
        world, rank, slots = 2, 0, 3
        full = 2 * n                                  # full-width gather buffers, this rank owns [0, n)
        mine = torch.zeros((m, full), dtype=torch.bfloat16, device="cuda")
        peer = torch.zeros((m, full), dtype=torch.bfloat16, device="cuda")
        flags = [torch.zeros(slots * world, dtype=torch.int32, device="cuda") for _ in range(world)]
        ctrl = torch.zeros(64, dtype=torch.int32, device="cuda")
        epoch, done = ctrl[0:1], ctrl[32:33]
        stream = torch.cuda.current_stream()
        for step in (1, 2):
            native.step_begin(epoch, stream)
            g = native.make_gather(world, rank, epoch.data_ptr(), seg=0,
                                   peer_out=[mine.data_ptr(), peer.data_ptr()],
                                   peer_flags=[f.data_ptr() for f in flags], signal_slot=1, done=done.data_ptr())
            native.gemv_multi(native.W_BF16, native.DT_BF16, x, [(w, None, mine, full, n)], None,
                              native.DT_BF16, m, k, gather=g)
            torch.cuda.synchronize()
            assert int(epoch.item()) == step
            for f in flags:                                # rank 0's flag of slot 1, on both ranks
                expect = np.zeros(slots * world, dtype=np.int32)
                expect[1 * world + rank] = step
                np.testing.assert_array_equal(f.cpu().numpy(), expect)
            assert int(done.item()) == 0
        plain = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        native.gemv(native.W_BF16, native.DT_BF16, x, w, None, None, plain, native.DT_BF16, m, n, k)
        torch.cuda.synchronize()
        assert torch.equal(mine[:, :n].view(torch.int16), plain.view(torch.int16))
        assert torch.equal(peer[:, :n].view(torch.int16), plain.view(torch.int16))
        assert not torch.any(peer[:, n:].view(torch.int16))
        ref = og.bf16_projection64(x_bits, w_bits)
        assert ob.check_outputs(ref, plain.float().cpu().numpy(), output_dtype="bf16")["passed"]
        assert native.device_status() == 0
    finally:
        native.set_option(native.OPT_SPLIT, -1)


def test_wait_for_raised_flags_then_read_gathered_input(native):
    """A launch that waits for flags the host already raised proceeds at once
    and computes the same result as a launch without the wait."""
    m, n, k = 1, 256, 2048
    _, _, x, w = _setup(m, n, k, 7)
    world, slots = 2, 2
    flags = torch.zeros(slots * world, dtype=torch.int32, device="cuda")
    ctrl = torch.zeros(64, dtype=torch.int32, device="cuda")
    epoch = ctrl[0:1]
    native.step_begin(epoch, torch.cuda.current_stream())
    flags[1 * world:2 * world] = 1                     # both ranks raised slot 1 for epoch 1
    out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    g = native.make_gather(world, 0, epoch.data_ptr(), wait_flags=flags.data_ptr(), wait_slot=1)
    native.gemv_multi(native.W_BF16, native.DT_BF16, x, [(w, None, out, n, n)], None, native.DT_BF16, m, k,
                      gather=g)
    plain = torch.zeros_like(out)
    native.gemv(native.W_BF16, native.DT_BF16, x, w, None, None, plain, native.DT_BF16, m, n, k)
    native.wait_flags(flags.data_ptr(), 1, world, epoch, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), plain.view(torch.int16))
    assert native.device_status() == 0


def test_flag_wait_times_out_with_status_not_hang(native):
    """Nothing raises slot 0: the bounded device wait gives up, records the
    flag-timeout status and returns; the context stays usable."""
    world = 2
    flags = torch.zeros(2 * world, dtype=torch.int32, device="cuda")
    ctrl = torch.zeros(64, dtype=torch.int32, device="cuda")
    epoch = ctrl[0:1]
    stream = torch.cuda.current_stream()
    native.step_begin(epoch, stream)
    native.wait_flags(flags.data_ptr(), 0, world, epoch, stream)
    torch.cuda.synchronize()
    assert native.device_status(clear=True) == STATUS_FLAG_TIMEOUT
    assert float(torch.ones(4, device="cuda").sum().item()) == 4.0
    assert native.device_status() == 0


def test_gather_descriptor_validation(native):
    m, n, k = 1, 64, 1024
    _, _, x, w = _setup(m, n, k, 3)
    out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    ctrl = torch.zeros(64, dtype=torch.int32, device="cuda")
    bad = [
        native.make_gather(9, 0, ctrl.data_ptr()),                                   # too many peers
        native.make_gather(2, 2, ctrl.data_ptr()),                                   # rank out of range
        native.make_gather(2, 0, None),                                              # no epoch
        native.make_gather(2, 0, ctrl.data_ptr(), seg=0, peer_out=[out.data_ptr()]),  # missing peer pointer
        native.make_gather(2, 0, ctrl.data_ptr(), signal_slot=0,
                           peer_flags=[ctrl.data_ptr(), ctrl.data_ptr()]),           # no done counter
    ]
    for g in bad:
        with pytest.raises(native.KlabError):
            native.gemv_multi(native.W_BF16, native.DT_BF16, x, [(w, None, out, n, n)], None, native.DT_BF16, m,
                              k, gather=g)
    g = native.make_gather(2, 0, ctrl.data_ptr(), seg=0, peer_out=[out.data_ptr(), out.data_ptr()])
    with pytest.raises(native.KlabError):                                            # gather needs BF16 out
        native.gemv_multi(native.W_BF16, native.DT_BF16, x, [(w, None, out.float(), n, n)], None,
                          native.DT_F32, m, k, gather=g)
