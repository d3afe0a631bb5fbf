"""Projection chain of BASELINE config 5, column-sharded over ranks.

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

The reference has no distributed code (its chain is single-GPU); the
all-gather is NCCL through torch.distributed.
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
                 seed=0, std=0.02, weights=None, project=None, fuse=True):
        """weights(layer, name, rows) -> BF16 tensor supplies shard weights (default:
        seeded N(0, std^2)); project(x, w, n_rows, k, out, ldo) replaces the native
        projection (host-side tests drive the sharding and gathers on CPU with it)."""
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
        self.hbuf = [torch.zeros((m, shape.hidden), **bf) for _ in range(2)]
        self.a_out = {name: torch.zeros((m, n), **bf) for name, n in stage_a if name not in ("up",)}
        self.up_full = torch.zeros((m, shape.ffn), **bf)       # gather buffer for up
        self.graph = None
        self.stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None

    def weight_bytes(self):
        return sum(w.numel() * 2 for layer in self.layers for (w, _, _) in layer.values())

    def launches_per_step(self):
        return (2 if self.fuse else 7) * self.shape.layers

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

    def forward_eager(self, x):
        """One token step: h <- x, run every layer, return the final h (full width)."""
        shape = self.shape
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

    def release(self):
        """Drop the graph (release graphs holding NCCL calls before destroying the group)."""
        self.graph = None
