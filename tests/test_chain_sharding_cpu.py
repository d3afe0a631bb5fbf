"""Host logic of the column-sharded chain on CPU: world_size-2 gloo ranks run the
real ProjectionChain (shards, full-width gather buffers, in-place all-gathers)
with the oracle as the projection; the result must be bit-identical to the
single-rank chain."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import bf16 as ob
from oracle import gemv as og

SHAPE = dict(layers=3, hidden=64, kv=32, ffn=96, tokens=1)


def _weights(layer, name, rows, shape):
    n = {"q": shape.hidden, "k": shape.kv, "v": shape.kv, "o": shape.hidden, "gate": shape.ffn,
         "up": shape.ffn, "down": shape.hidden}[name]
    k = shape.ffn if name == "down" else shape.hidden
    bits = og.normal_bf16_bits(layer * 16 + len(name), (n, k), 0.05)[rows[0]:rows[1]]
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _oracle_project(x, w, n_rows, k, dst, ldo):
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    y = ob.round_bf16_bits(og.bf16_projection64(xb, wb))
    dst[:, :n_rows].copy_(torch.from_numpy(y.view(np.int16)).view(torch.bfloat16))


def _run(rank, world, port, x_bits, result):
    from klab_b200.chain import ChainShape, ProjectionChain

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    shape = ChainShape(**SHAPE)
    chain = ProjectionChain(shape, rank=rank, world=world, group=dist.group.WORLD if world > 1 else None,
                            weights=lambda layer, name, rows: _weights(layer, name, rows, shape),
                            project=_oracle_project)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)
    out = chain.forward_eager(x)
    result[rank] = out.view(torch.int16).numpy().copy()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_chain_matches_single_rank():
    x_bits = og.normal_bf16_bits(7, (1, SHAPE["hidden"]), 1.0)
    single = {}
    _run(0, 1, _free_port(), x_bits, single)
    ctx = mp.get_context("spawn")  # the manager too: no fork of this multi-threaded process
    with ctx.Manager() as manager:
        shared = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_run, args=(r, 2, port, x_bits, shared)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        for r in range(2):
            np.testing.assert_array_equal(shared[r], single[0])
    # and the chain is a real computation, not an identity
    assert not np.array_equal(single[0], x_bits.view(np.int16))


def test_shard_ranges_cover_rows_exactly():
    from klab_b200.chain import _shard

    for n, g in ((4096, 8), (1024, 8), (14336, 4), (96, 2)):
        ranges = [_shard(n, r, g) for r in range(g)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    with pytest.raises(ValueError):
        _shard(100, 0, 3)


def test_p2p_schedule_waits_only_for_slots_signalled_earlier():
    """Every wait in a step is for a slot signalled by an earlier launch of the
    same step, each slot is signalled once, and each gathered buffer is written
    by peers only after every rank has finished reading it (the reader's next
    signal precedes the writer's wait)."""
    from klab_b200.chain import p2p_schedule

    for layers in (1, 2, 5, 32):
        sched = p2p_schedule(layers)
        signalled = []
        for kind, layer, wait_slot, signal_slot in sched:
            if wait_slot >= 0:
                assert wait_slot in signalled, (kind, layer, wait_slot)
            if signal_slot >= 0:
                assert signal_slot not in signalled
                signalled.append(signal_slot)
        assert sorted(signalled) == list(range(2 * layers))
        assert sched[-1] == ("end", layers, 2 * layers - 1, -1)
        # Stage A of layer i (i > 0) writes the peers' up buffer after waiting
        # for slot 2i-1, which every rank signals after its down of layer i-1,
        # the last reader of that buffer.
        for kind, layer, wait_slot, _ in sched:
            if kind == "stage_a" and layer:
                assert wait_slot == 2 * (layer - 1) + 1


def test_p2p_mode_argument_checks():
    from klab_b200.chain import ChainShape, ProjectionChain

    shape = ChainShape(layers=1, hidden=64, kv=32, ffn=128)
    with pytest.raises(ValueError):
        ProjectionChain(shape, gather="mpi", project=lambda *a: None)
    with pytest.raises(ValueError):
        ProjectionChain(shape, world=2, gather="p2p", project=lambda *a: None)


@pytest.mark.parametrize("stages_per_layer", [2, 4])
def test_persistent_schedule_covers_every_row_once(stages_per_layer):
    """Both persistent schedules list every row of q, k, v, o, gate, up and down exactly
    once per layer; the two-stage schedule leads with the gathered up rows and keeps every
    row that reads h_i in the first stage (host logic, oracle projection on CPU)."""
    from klab_b200.chain import ChainShape, ProjectionChain

    shape = ChainShape(**SHAPE)
    for world, rank in ((1, 0), (2, 1)):
        chain = ProjectionChain(shape, rank=rank, world=world,
                                weights=lambda layer, name, rows: _weights(layer, name, rows, shape),
                                project=_oracle_project, stages_per_layer=stages_per_layer)
        sched = chain.persistent_schedule()
        assert len(sched) == stages_per_layer
        covered = {}
        for _, parts in sched:
            for name, b, e in parts:
                n = chain.layers[0][name][1][1] - chain.layers[0][name][1][0]
                e = n if e is None else e
                covered.setdefault(name, []).append((b, e))
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            n = chain.layers[0][name][1][1] - chain.layers[0][name][1][0]
            spans = sorted(covered[name])
            assert spans[0][0] == 0 and spans[-1][1] == n, (name, spans)
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:])), (name, spans)
        kinds = [kind for kind, _ in sched]
        assert kinds.index("up") < kinds.index("down")
        if stages_per_layer == 2:
            assert sched[0][1][0][0] == "up" and [n for n, _, _ in sched[1][1]] == ["down"]


def test_stages_per_layer_is_checked():
    from klab_b200.chain import ChainShape, ProjectionChain

    with pytest.raises(ValueError):
        ProjectionChain(ChainShape(layers=1, hidden=64, kv=32, ffn=128), project=lambda *a: None, stages_per_layer=3)
