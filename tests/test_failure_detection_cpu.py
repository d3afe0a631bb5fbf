"""Failure detection among chain ranks, on CPU: ranks are processes sharing a
torch.distributed TCPStore (the rendezvous store of a process group) and running
liveness.StepGuard between steps, through the real ProjectionChain (oracle projection,
gloo gathers) where a step runs. Cases: a rank that leaves between steps, a late rank
(inside and beyond the bound), a restarted rank with a stale epoch, a corrupted epoch
record, epoch wrap-around, and the device status check (a fake status word). Every
waiting rank raises within its bound; nothing waits without limit."""

import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from klab_b200 import liveness as lv


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _store(rank, world, port):
    return dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))


def _scenario(rank, world, port, name, result):
    store = _store(rank, world, port)
    guard = lv.StepGuard(store, rank, world, timeout=0.5, prefix=f"t/{name}")
    t0 = time.monotonic()
    outcome = "ok"
    try:
        guard.enter(1)                                  # both ranks take step 1
        if name == "leaves":
            if rank == 1:
                guard.leave()
                result[rank] = ("left", 0.0)
                return
            guard.enter(2)
        elif name == "late_within":
            if rank == 1:
                time.sleep(0.2)
            guard.enter(2)
        elif name == "late_beyond":
            if rank == 1:
                time.sleep(2.0)                         # misses rank 0's 0.5 s bound
            guard.enter(2)
        elif name == "stale":
            if rank == 1:
                guard.post(1)                           # restarted: posts an old epoch, then waits
                time.sleep(1.0)
                result[rank] = ("restarted", 0.0)
                return
            guard.enter(3)
        elif name == "corrupt":
            if rank == 1:
                store.set("t/corrupt/1", b"\xff\xfe")
                time.sleep(1.0)
                result[rank] = ("corrupted", 0.0)
                return
            guard.enter(2)
    except lv.PeerFailure as error:
        outcome = type(error).__name__
    result[rank] = (outcome, time.monotonic() - t0)
    if rank == 0:   # keep the store's host alive while the other rank finishes
        time.sleep(2.5 if name == "late_beyond" else 0.3)


@pytest.mark.parametrize("name,expect0,bound", [
    ("leaves", "PeerLost", 0.5),          # noticed at once, not after the bound
    ("late_within", "ok", 1.0),
    ("late_beyond", "PeerLate", 1.5),
    ("stale", "StaleEpoch", 0.5),
    ("corrupt", "CorruptEpoch", 0.5),
])
def test_waiting_rank_raises_within_its_bound(name, expect0, bound):
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    procs = [ctx.Process(target=_scenario, args=(r, 2, port, name, result)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    outcome, elapsed = result[0]
    assert outcome == expect0, result.copy()
    assert elapsed < bound + 0.5, elapsed


def test_epoch_comparison_wraps_like_the_device_flags():
    assert lv.epoch_reached(5, 5) and lv.epoch_reached(6, 5) and not lv.epoch_reached(4, 5)
    assert lv.epoch_reached(0, 0xFFFFFFFF) and lv.epoch_reached(1, 0xFFFFFFFF)   # wrapped past the target
    assert not lv.epoch_reached(0xFFFFFFFF, 0)
    assert lv.epoch_distance(2, 0xFFFFFFFE) == 4 and lv.epoch_distance(0xFFFFFFFE, 2) == -4


def test_guard_across_wrap_and_device_status():
    store = dist.HashStore()
    a, b = lv.StepGuard(store, 0, 2, timeout=0.2), lv.StepGuard(store, 1, 2, timeout=0.2)
    b.post(0xFFFFFFFF)
    with pytest.raises(lv.PeerLate):           # rank 1 is one epoch behind: waits, then gives up
        a.enter(0)
    b.post(0)
    a.enter(0)                                 # reached across the wrap
    lv.StepGuard.check_device(lambda: 0)
    with pytest.raises(lv.DeviceWaitExpired) as info:
        lv.StepGuard.check_device(lambda: 2)
    assert info.value.status == 2
    with pytest.raises(ValueError):
        lv.StepGuard(store, 2, 2)


def _chain_ranks(rank, world, port, result):
    """Two gloo ranks run the sharded chain (oracle projection) through step_guarded;
    rank 1 leaves after two steps and rank 0's third step raises PeerLost."""
    from klab_b200.chain import ChainShape, ProjectionChain
    from oracle import bf16 as ob
    from oracle import gemv as og

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    shape = ChainShape(layers=2, hidden=32, kv=16, ffn=48)

    def weights(layer, name, rows):
        n = {"down": shape.hidden, "k": shape.kv, "v": shape.kv, "gate": shape.ffn, "up": shape.ffn}.get(
            name, shape.hidden)
        k = shape.ffn if name == "down" else shape.hidden
        bits = og.normal_bf16_bits(layer * 8 + len(name), (n, k), 0.05)[rows[0]:rows[1]]
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)

    def project(x, w, n_rows, k, dst, ldo):
        xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
        y = ob.round_bf16_bits(og.bf16_projection64(xb, w.view(torch.int16).numpy().view(np.uint16)))
        dst[:, :n_rows].copy_(torch.from_numpy(y.view(np.int16)).view(torch.bfloat16))

    chain = ProjectionChain(shape, rank=rank, world=world, group=dist.group.WORLD, weights=weights, project=project)
    guard = lv.StepGuard(dist.distributed_c10d._get_default_store(), rank, world, timeout=1.0, prefix="chain")
    x = torch.zeros((1, shape.hidden), dtype=torch.bfloat16)
    steps, outcome = 0, "ok"
    try:
        for _ in range(3):
            if rank == 1 and steps == 2:
                guard.leave()
                break
            chain.step_guarded(guard, x)
            steps += 1
    except lv.PeerFailure as error:
        outcome = type(error).__name__
    result[rank] = (steps, outcome)
    time.sleep(0.5)


def test_chain_rank_leaving_between_steps_is_seen_before_the_next_launch():
    port = _free_port()
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    procs = [ctx.Process(target=_chain_ranks, args=(r, 2, port, result)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=90)
        assert pr.exitcode == 0
    assert result[0] == (2, "PeerLost") and result[1] == (2, "ok")
