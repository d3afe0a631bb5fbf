"""Projection chain of benchmark config 5, column-sharded over ranks.

Per layer (Llama-3-8B projection shapes, M tokens, BF16 weights and outputs):
  stage A: q 4096->4096, k 4096->1024, v 4096->1024, o 4096->4096,
           gate 4096->14336, up 4096->14336, all reading the layer input h;
  gather:  up's output (14336) is all-gathered;
  stage B: down 14336->4096 reads the gathered vector;
  gather:  down's output (4096) is all-gathered and becomes the next h.
Rank r of g owns output rows [r*N/g, (r+1)*N/g) of every weight and writes its
rows straight into its slice of the full-width gather buffers (ldo = N), so the
all-gather is in place. The kernel's reduction order depends only on K, so the
sharded chain is bit-identical to the one-GPU chain. The whole token step is
captured in one CUDA graph; launches use programmatic dependent launch so a
projection's weight stream starts while the previous one drains.

The reference has no distributed code (its chain is single-GPU). Two gather
modes: "nccl" (all_gather_into_tensor through torch.distributed after each
gathered projection) and "p2p", where the gather is fused into the projection
kernel: its epilogue also stores every output value into each peer's copy of
the gather buffer over NVLink (CUDA IPC mappings), the grid's last CTA raises
this rank's flag on every rank, and the next projection waits (bounded, on the
device) for all flags of that slot before reading its input. Flags carry the
step's epoch, so they never need resetting; see p2p_schedule for the slots.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from ._module import get_module

HIDDEN, KV, FFN, LAYERS = 4096, 1024, 14336, 32
STAGE_A = (("q", HIDDEN), ("k", KV), ("v", KV), ("o", HIDDEN), ("gate", FFN), ("up", FFN))
_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass
class ChainShape:
    layers: int = LAYERS
    hidden: int = HIDDEN
    kv: int = KV
    ffn: int = FFN
    tokens: int = 1

    def projections(self):
        a = [("q", self.hidden), ("k", self.kv), ("v", self.kv), ("o", self.hidden), ("gate", self.ffn),
             ("up", self.ffn)]
        return a, ("down", self.hidden, self.ffn)

    def bytes_per_token(self):
        a, (_, dn, dk) = self.projections()
        per_layer = sum(n * self.hidden for _, n in a) * 2 + dn * dk * 2
        return per_layer * self.layers


def _shard(n, rank, world):
    if n % world:
        raise ValueError(f"{n} output rows do not split over {world} ranks")
    part = n // world
    return rank * part, (rank + 1) * part


def p2p_schedule(layers):
    """Flag slots of one step in "p2p" mode, as a list of launches
    (kind, layer, wait_slot, signal_slot): stage A of layer i signals slot 2i
    (its up output is gathered) and waits for slot 2i-1 (the previous down
    output, its input); down of layer i waits for 2i and signals 2i+1; the step
    ends with a wait on slot 2*layers-1. wait_slot -1: no wait (layer 0 reads
    the step input, which is local)."""
    out = []
    for i in range(layers):
        out.append(("stage_a", i, 2 * i - 1 if i else -1, 2 * i))
        out.append(("down", i, 2 * i, 2 * i + 1))
    out.append(("end", layers, 2 * layers - 1, -1))
    return out


class _DeviceBytes:
    """A raw device allocation seen by torch through __cuda_array_interface__
    (the memory is owned and freed by the chain)."""

    def __init__(self, address, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (address, False),
                                         "version": 3, "strides": None}


def make_weight(shape, layer, name, rows, device, std=0.02, seed=0):
    """Deterministic N(0, std^2) BF16 weight rows [r0, r1) of projection `name` in
    `layer`: the full matrix is generated from one seed and sliced, so every
    shard count sees the same values."""
    gen = torch.Generator(device=device)
    gen.manual_seed((seed * 1_000_003 + layer * 64 + _NAMES.index(name)) & 0x7FFFFFFF)
    n, k = shape
    full = torch.randn((n, k), generator=gen, device=device, dtype=torch.float32).mul_(std).to(torch.bfloat16)
    out = full[rows[0]:rows[1]].contiguous()
    del full
    return out


class ProjectionChain:
    """The sharded projection chain on one rank. `group` is a torch.distributed
    process group (NCCL) when world > 1."""

    def __init__(self, shape: ChainShape = ChainShape(), *, rank=0, world=1, device=None, group=None,
                 seed=0, std=0.02, weights=None, project=None, fuse=True, gather="nccl", persistent=False,
                 stages_per_layer=2):
        """weights(layer, name, rows) -> BF16 tensor supplies shard weights (default:
        seeded N(0, std^2)); project(x, w, n_rows, k, out, ldo) replaces the native
        projection (host-side tests drive the sharding and gathers on CPU with it).
        gather: "nccl" or "p2p" (fused peer stores; needs the native fused path).
        persistent: the whole step is one launch of the persistent chain kernel
        (one token; with world > 1 it needs gather="p2p"); stages_per_layer: 2 or 4
        stages of the persistent kernel per layer (persistent_schedule; 2, the
        default, measured faster on B200 at 2, 4 and 8 ranks)."""
        if gather not in ("nccl", "p2p"):
            raise ValueError(f"gather must be 'nccl' or 'p2p', not {gather!r}")
        if gather == "p2p" and (project is not None or not fuse):
            raise ValueError("gather='p2p' needs the native projection with fuse=True")
        if persistent and (project is not None or not fuse or shape.tokens != 1
                           or (world > 1 and gather != "p2p")):
            raise ValueError("persistent=True needs the native projection, fuse=True, one token and, "
                             "with several ranks, gather='p2p'")
        if stages_per_layer not in (2, 4):
            raise ValueError("stages_per_layer must be 2 or 4")
        self.persistent = persistent
        self.stages_per_layer = stages_per_layer
        self._plan = None
        if world > 8 and gather == "p2p":
            raise ValueError("gather='p2p' supports at most 8 ranks")
        self.gather = gather if world > 1 else "none"
        self._ipc = None
        self.shape = shape
        self.rank, self.world, self.group = rank, world, group
        if project is None:
            self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
            get_module(self.device)
        else:
            self.device = torch.device("cpu") if device is None else torch.device(device)
        self._project = project
        # One launch for the six stage-A projections (they share h and K); the
        # outputs equal separate launches bit for bit.
        self.fuse = fuse and project is None
        stage_a, (dname, dn, dk) = shape.projections()
        m = shape.tokens
        self.layers = []
        for layer in range(shape.layers):
            entry = {}
            for name, n in stage_a:
                rows = _shard(n, rank, world)
                w = weights(layer, name, rows) if weights else make_weight((n, shape.hidden), layer, name, rows,
                                                                           self.device, std, seed)
                entry[name] = (w, rows, n)
            rows = _shard(dn, rank, world)
            w = weights(layer, dname, rows) if weights else make_weight((dn, dk), layer, dname, rows, self.device,
                                                                        std, seed)
            entry[dname] = (w, rows, dn)
            self.layers.append(entry)
        bf = dict(dtype=torch.bfloat16, device=self.device)
        # Two full-width layer-input buffers used alternately: layer i reads
        # hbuf[i % 2] and its down projection (and gather) writes hbuf[(i+1) % 2].
        self.a_out = {name: torch.zeros((m, n), **bf) for name, n in stage_a if name not in ("up",)}
        if self.persistent:
            pass                                                   # buffers: _setup_persistent
        elif self.gather == "p2p":
            self._setup_p2p()
        else:
            self.hbuf = [torch.zeros((m, shape.hidden), **bf) for _ in range(2)]
            self.up_full = torch.zeros((m, shape.ffn), **bf)       # gather buffer for up
        self.graph = None
        self.stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        if self.persistent:
            self._setup_persistent()

    def persistent_schedule(self):
        """Stages of the persistent kernel for one layer i, in order. Every CTA takes
        an equal share of a stage's rows in at most two contiguous parts: of a
        gathered segment listed first, then of the other rows, so the gathered rows
        are produced first everywhere while the stage's other rows hide their
        gather. Only up and down feed later stages.

        stages_per_layer=2 (default): "up" = [up (gathered into up_t), q, k, v, o,
        gate] (x = h_i); "down" = [down] (gathered into h_t[(i+1) % 2]; x = up_t).
        stages_per_layer=4: up; fill1 (first half of the q, k, v, o, gate rows;
        x = h_i); down; fill2 (the other half; x = h_i again): a filler stage
        between each producer and consumer, at twice the stage boundaries.
        Measured on B200 (tok/s, 2 / 4 / 8 GPUs): 2 stages 773.7 / 1,207.8 /
        1,567.9; 4 stages 719.5 / 1,052.0 / 1,366.4.
        Returns, per layer, a list of (kind, [(name, local_row_begin, local_row_end)])."""
        names = [name for name, _ in self.shape.projections()[0] if name != "up"]
        fill = []
        for name in names:
            n = self.layers[0][name][1][1] - self.layers[0][name][1][0]
            fill.append((name, 0, n))
        if self.stages_per_layer == 2:
            return [("up", [("up", 0, None)] + fill), ("down", [("down", 0, None)])]
        total = sum(e - b for _, b, e in fill)
        half, fill1, fill2, acc = total // 2, [], [], 0
        for name, b, e in fill:
            if acc + (e - b) <= half:
                fill1.append((name, b, e))
            elif acc >= half:
                fill2.append((name, b, e))
            else:
                cut = b + (half - acc)
                fill1.append((name, b, cut))
                fill2.append((name, cut, e))
            acc += e - b
        return [("up", [("up", 0, None)]), ("fill1", fill1), ("down", [("down", 0, None)]), ("fill2", fill2)]

    def _setup_persistent(self):
        """Stage table of the persistent kernel (persistent_schedule). The up and
        down outputs live only as tagged words (tag << 16 | bf16) in the gather
        buffers up_t [ffn] and h_t[2] [hidden], which every rank writes into
        (IPC mappings when world > 1); layer i reads h_t[i % 2]."""
        shape, world, rank = self.shape, self.world, self.rank
        bf = dict(dtype=torch.bfloat16, device=self.device)
        self.hbuf = [torch.zeros((1, shape.hidden), **bf)]        # step input (plain BF16)
        self.out = torch.zeros((1, shape.hidden), **bf)           # step output (plain BF16)
        self.up_full = None
        words = {"ht0": shape.hidden * 4, "ht1": shape.hidden * 4, "upt": shape.ffn * 4}
        if world == 1:
            local = {name: torch.zeros(n // 4, dtype=torch.int32, device=self.device) for name, n in words.items()}
            bases = {name: [t.data_ptr()] for name, t in local.items()}
        else:
            raw, offsets = self._ipc_region(words)
            local = {name: raw[offsets[name]:offsets[name] + n].view(torch.int32) for name, n in words.items()}
            bases = {name: [a + offsets[name] for a in self._ipc["peers"]] for name in words}
        self.h_t = [local["ht0"], local["ht1"]]
        self.up_t = local["upt"]
        self.ctrl = torch.zeros(64, dtype=torch.int32, device=self.device)
        self.epoch = self.ctrl[0:1]
        stages, schedule = [], self.persistent_schedule()
        prev_down = -1
        for i, entry in enumerate(self.layers):
            h_ptr = self.hbuf[0].data_ptr() if i == 0 else self.h_t[i % 2].data_ptr()
            up_stage = None
            for kind, parts in schedule:
                st = _native.ChainStage()
                st.gather_seg = -1
                if kind == "up":
                    w, rows, _ = entry["up"]
                    st.x, st.k, st.x_stage, st.nseg, st.gather_seg = h_ptr, shape.hidden, prev_down, len(parts), 0
                    st.w[0], st.n[0] = w.data_ptr(), rows[1] - rows[0]
                    for q in range(world):
                        st.peer_out[q] = bases["upt"][q] + rows[0] * 4
                    for j, (name, b, e) in enumerate(parts[1:], start=1):   # rows that also read h_i
                        w, rows, _ = entry[name]
                        st.w[j] = w[b:].data_ptr()
                        st.out[j] = self.a_out[name][:, rows[0] + b:].data_ptr()
                        st.n[j] = e - b
                    up_stage = len(stages)
                elif kind == "down":
                    w, rows, _ = entry["down"]
                    st.x, st.k, st.x_stage, st.nseg, st.gather_seg = self.up_t.data_ptr(), shape.ffn, up_stage, 1, 0
                    st.w[0], st.n[0] = w.data_ptr(), rows[1] - rows[0]
                    dst = "ht1" if i % 2 == 0 else "ht0"
                    for q in range(world):
                        st.peer_out[q] = bases[dst][q] + rows[0] * 4
                    prev_down_next = len(stages)
                else:
                    st.x, st.k, st.x_stage, st.nseg = h_ptr, shape.hidden, prev_down, len(parts)
                    for j, (name, b, e) in enumerate(parts):
                        w, rows, _ = entry[name]
                        st.w[j] = w[b:].data_ptr()
                        st.out[j] = self.a_out[name][:, rows[0] + b:].data_ptr()
                        st.n[j] = e - b
                stages.append(st)
            prev_down = prev_down_next
        self._stage_kinds = [kind for _ in self.layers for kind, _ in schedule]
        sync = _native.ChainSync()
        sync.npeers, sync.rank = world, rank
        sync.epoch = self.epoch.data_ptr()
        sync.final_in = self.h_t[len(self.layers) % 2].data_ptr()
        sync.final_out = self.out.data_ptr()
        with torch.cuda.device(self.device):
            self._plan = _native.chain_create(stages, sync)

    def trace_step(self, x):
        """Run one eager step of the persistent kernel with its timeline on and
        return it as an int64 tensor [stages, CTAs, slots] of global-timer ns
        (slots: entered, previous stage done in this CTA, x staged, then per
        warp: first item of the stage landed, run computed, done)."""
        if not self.persistent:
            raise ValueError("trace_step needs persistent=True")
        grid, slots = _native.chain_info(self._plan)
        buf = torch.zeros((len(self._stage_kinds), grid, slots), dtype=torch.int64, device=self.device)
        _native.chain_trace(self._plan, buf)
        try:
            self.forward_eager(x)
            torch.cuda.synchronize(self.device)
        finally:
            _native.chain_trace(self._plan, None)
        return buf.cpu()

    def _ipc_region(self, sizes):
        """One zeroed IPC allocation per rank holding the named regions (bytes,
        each 256-byte aligned), mapped by every peer; handles are exchanged with
        all_gather_object. Returns (uint8 tensor over it, offsets)."""
        import torch.distributed as dist

        offsets, total = {}, 0
        for name, nbytes in sizes.items():
            offsets[name] = total
            total += (nbytes + 255) // 256 * 256
        with torch.cuda.device(self.device):
            base, handle = _native.ipc_malloc(total)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        peers = []
        with torch.cuda.device(self.device):
            for q in range(self.world):
                peers.append(base if q == self.rank else _native.ipc_open(handles[q]))
        self._ipc = {"base": base, "peers": peers, "offsets": offsets}
        self._raw = torch.as_tensor(_DeviceBytes(base, total), device=self.device)
        return self._raw, offsets

    def _setup_p2p(self):
        """Launch-per-stage gathers: regions [hbuf0][hbuf1][up_full][flags]."""
        shape, m, world = self.shape, self.shape.tokens, self.world
        self._slots = 2 * shape.layers
        raw, offsets = self._ipc_region({"h0": m * shape.hidden * 2, "h1": m * shape.hidden * 2,
                                         "up": m * shape.ffn * 2, "flags": self._slots * world * 4})
        view = lambda off, n: raw[off:off + n * 2].view(torch.bfloat16).view(m, n // m)  # noqa: E731
        self.hbuf = [view(offsets["h0"], m * shape.hidden), view(offsets["h1"], m * shape.hidden)]
        self.up_full = view(offsets["up"], m * shape.ffn)
        self.flags = raw[offsets["flags"]:offsets["flags"] + self._slots * world * 4].view(torch.int32)
        # epoch (word 0) and the CTA completion counter (word 32) on separate lines.
        self.ctrl = torch.zeros(64, dtype=torch.int32, device=self.device)
        self.epoch, self.done = self.ctrl[0:1], self.ctrl[32:33]
        self._gathers = self._make_gathers()

    def _make_gathers(self):
        """The Gather descriptors of every launch of a step (they never change)."""
        ipc, world, rank = self._ipc, self.world, self.rank
        off = ipc["offsets"]
        flags = [a + off["flags"] for a in ipc["peers"]]
        local_flags = ipc["base"] + off["flags"]
        epoch, done = self.epoch.data_ptr(), self.done.data_ptr()
        gathers = []
        for kind, i, wait_slot, signal_slot in p2p_schedule(self.shape.layers):
            if kind == "end":
                break
            entry = self.layers[i]
            if kind == "stage_a":
                r0 = entry["up"][1][0]
                dst, seg = off["up"], 5
            else:
                r0 = entry["down"][1][0]
                dst, seg = off["h1" if i % 2 == 0 else "h0"], 0
            gathers.append(_native.make_gather(
                world, rank, epoch, seg=seg, peer_out=[a + dst + r0 * 2 for a in ipc["peers"]],
                peer_flags=flags, signal_slot=signal_slot, wait_flags=local_flags if wait_slot >= 0 else None,
                wait_slot=wait_slot, done=done))
        return gathers

    def weight_bytes(self):
        return sum(w.numel() * 2 for layer in self.layers for (w, _, _) in layer.values())

    def launches_per_step(self):
        """Kernels of this library per step (p2p adds the epoch and end-wait kernels)."""
        if self.persistent:
            return 1
        return (2 if self.fuse else 7) * self.shape.layers + (2 if self.gather == "p2p" else 0)

    def _proj(self, x, w, rows, n, out, k):
        """Rows [r0, r1) of this projection into columns [r0, r1) of the full-width `out`."""
        m = x.shape[0]
        dst = out[:, rows[0]:]
        if self._project is not None:
            self._project(x, w, rows[1] - rows[0], k, dst, out.shape[1])
            return
        _native.gemv(_native.W_BF16, _native.DT_BF16, x, w, None, None, dst, _native.DT_BF16, m,
                     rows[1] - rows[0], k, ldo=out.shape[1])

    def _gather(self, full, n):
        if self.world == 1:
            return
        import torch.distributed as dist

        part = n // self.world
        m = full.shape[0]
        if m == 1:
            mine = full[0, self.rank * part:(self.rank + 1) * part]
            dist.all_gather_into_tensor(full.view(-1), mine, group=self.group)
        else:
            # Multi-token: gather rank-major chunks, then the layout is [world][m][part].
            chunk = full[:, self.rank * part:(self.rank + 1) * part].contiguous()
            tmp = torch.empty((self.world, m, part), dtype=full.dtype, device=full.device)
            dist.all_gather_into_tensor(tmp.view(-1), chunk.view(-1), group=self.group)
            full.copy_(tmp.permute(1, 0, 2).reshape(m, n))

    def _forward_p2p(self, x):
        shape, world = self.shape, self.world
        stream = torch.cuda.current_stream(self.device)
        _native.step_begin(self.epoch, stream)
        self.hbuf[0].copy_(x)
        for i, entry in enumerate(self.layers):
            h, nxt = self.hbuf[i % 2], self.hbuf[(i + 1) % 2]
            outs = dict(self.a_out, up=self.up_full)
            segments = []
            for name in ("q", "k", "v", "o", "gate", "up"):
                w, rows, n = entry[name]
                out = outs[name]
                segments.append((w, None, out[:, rows[0]:], out.shape[1], rows[1] - rows[0]))
            _native.gemv_multi(_native.W_BF16, _native.DT_BF16, h, segments, None, _native.DT_BF16, h.shape[0],
                               shape.hidden, gather=self._gathers[2 * i])
            w, rows, _ = entry["down"]
            _native.gemv_multi(_native.W_BF16, _native.DT_BF16, self.up_full,
                               [(w, None, nxt[:, rows[0]:], shape.hidden, rows[1] - rows[0])], None,
                               _native.DT_BF16, h.shape[0], shape.ffn, gather=self._gathers[2 * i + 1])
        _native.wait_flags(self._ipc["base"] + self._ipc["offsets"]["flags"], 2 * shape.layers - 1, world,
                           self.epoch, stream)
        return self.hbuf[len(self.layers) % 2]

    def forward_eager(self, x):
        """One token step: h <- x, run every layer, return the final h (full width)."""
        shape = self.shape
        if self.persistent:
            self.hbuf[0].copy_(x)
            _native.chain_launch(self._plan, torch.cuda.current_stream(self.device))
            return self.out
        if self.gather == "p2p":
            return self._forward_p2p(x)
        self.hbuf[0].copy_(x)
        for i, entry in enumerate(self.layers):
            h, nxt = self.hbuf[i % 2], self.hbuf[(i + 1) % 2]
            outs = dict(self.a_out, up=self.up_full)
            if self.fuse:
                segments = []
                for name in ("q", "k", "v", "o", "gate", "up"):
                    w, rows, n = entry[name]
                    out = outs[name]
                    segments.append((w, None, out[:, rows[0]:], out.shape[1], rows[1] - rows[0]))
                _native.gemv_multi(_native.W_BF16, _native.DT_BF16, h, segments, None, _native.DT_BF16,
                                   h.shape[0], shape.hidden)
            else:
                for name in ("q", "k", "v", "o", "gate", "up"):
                    w, rows, n = entry[name]
                    self._proj(h, w, rows, n, outs[name], shape.hidden)
            self._gather(self.up_full, shape.ffn)
            w, rows, _ = entry["down"]
            self._proj(self.up_full, w, rows, shape.hidden, nxt, shape.ffn)
            self._gather(nxt, shape.hidden)
        return self.hbuf[len(self.layers) % 2]

    def capture(self, x):
        """Capture one token step into a CUDA graph reading the static input x.
        Warm-up and capture use the chain's own stream, so split-K workspaces
        exist before capture."""
        self.static_x = x
        if self.gather == "p2p" and self._ipc is not None:
            import torch.distributed as dist

            # Start the ranks' first gathered step together: a flag wait is bounded.
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.forward_eager(self.static_x)
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.out = self.forward_eager(self.static_x)
        return self.out

    def replay(self):
        self.graph.replay()
        return self.out

    def step_guarded(self, guard, x=None):
        """One token step with host-side failure detection (liveness.StepGuard): every rank
        agrees, bounded, on the step's epoch before launching; after the step the device status
        word is checked. Replays the captured graph, or runs eagerly on x when nothing is
        captured. Raises a liveness.PeerFailure subclass or liveness.DeviceWaitExpired."""
        self._guard_epoch = getattr(self, "_guard_epoch", 0) + 1
        guard.enter(self._guard_epoch)
        out = self.replay() if self.graph is not None else self.forward_eager(x)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            guard.check_device()
        return out

    def release(self):
        """Drop the graph (release graphs holding NCCL calls before destroying the
        group) and, in p2p mode, unmap the peers' buffers and free this rank's
        (collective: every rank calls it)."""
        self.graph = None
        if self._plan is not None:
            torch.cuda.synchronize(self.device)
            _native.chain_destroy(self._plan)
            self._plan = None
        if self._ipc is None:
            return
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)          # no rank still writes into a peer
        with torch.cuda.device(self.device):
            for q, a in enumerate(self._ipc["peers"]):
                if q != self.rank:
                    _native.ipc_close(a)
        dist.barrier(group=self.group)          # every peer unmapped this rank's buffer
        self.hbuf = self.up_full = self.flags = self._raw = self.h_t = self.up_t = None
        with torch.cuda.device(self.device):
            _native.ipc_free(self._ipc["base"])
        self._ipc = None
