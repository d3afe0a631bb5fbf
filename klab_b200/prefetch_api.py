"""Cross-op L2 prefetch for ordinary torch modules, chosen at capture time.

Public surface of research/l2-prefetch/src/api.py: `PrefetchSequential(modules,
example_input, ...)` (a module that runs a list of modules as a chain) and
`PrefetchHooks(model, example_input, ...)` (hooks on an unmodified model,
`remove()` restores it), with the same arguments, `report` rows and guarantee:
a prefetch plan is kept only when it measurably helps and leaves every output
bit-identical, otherwise that part runs as plain PyTorch.

How it is built here:

* A *unit* is what one prefetch serves: in a chain, each module; under hooks,
  each module called in the traced forward that owns parameters directly, plus
  the parameters of modules inside it that the forward never calls (they are
  read by their nearest called ancestor, e.g. a fused attention's out_proj).
  Tensors under `min_bytes` are ignored.
* Units with the same (module type, parameter shapes and dtypes) signature
  share one plan. `_GroupTuner` walks the groups in first-use order and, for
  each, races the autotuner's candidate grid (prefetch_autotune.race:
  successive halving, bootstrap lower bound) with the earlier groups' choices
  already applied, so tuning cost grows with distinct shapes, not depth.
* At run time a `_SideStream` issues the next unit's prefetch on a side stream
  that first waits for the current stream, and the current stream waits for
  the side stream once at the end of the forward (and of the backward).
  Everything is capturable in one CUDA graph.
"""

from __future__ import annotations

import torch

from . import prefetch_autotune as autotune
from .l2prefetch import ChainRunner, prefetch


def _large(params, min_bytes):
    return [p for p in params if p.numel() * p.element_size() >= min_bytes]


def _signature(module, reads):
    return (type(module).__name__, tuple((tuple(p.shape), p.dtype) for p in reads))


class _GroupTuner:
    """Chooses one plan per signature group of units. make_runner(assignment) returns a
    callable(x) that runs the whole workload with {unit index: plan} applied."""

    def __init__(self, signatures, unit_reads, make_runner, example_input, calls, rounds, min_lower_ci, log):
        self.groups = {}
        for i, sig in enumerate(signatures):
            self.groups.setdefault(sig, []).append(i)
        self.unit_reads, self.make_runner = unit_reads, make_runner
        self.x0, self.calls, self.rounds, self.min_lower_ci, self.log = (example_input, calls, rounds, min_lower_ci,
                                                                           log)

    def run(self, count_key):
        assignment, report = {}, []
        for sig, members in self.groups.items():
            nbytes = autotune.stage_bytes(self.unit_reads[members[0]])
            if nbytes == 0:
                continue
            grid = autotune.candidates(nbytes)
            variants = {"current": self.make_runner(dict(assignment))}
            for name, plan in grid.items():
                variants[name] = self.make_runner({**assignment, **{i: plan for i in members}})
            kept, row, _ = autotune.race(variants, self.x0, self.calls, self.rounds, "current", self.min_lower_ci)
            plan = grid[kept] if kept else None
            if plan is not None:
                assignment.update({i: plan for i in members})
            report.append({"signature": str(sig), count_key: len(members), "bytes": nbytes, "plan": plan,
                           "saved_pct": row["saved_pct"] if plan is not None else None})
            if self.log:
                self.log(f"{sig[0]} x{len(members)} ({nbytes >> 10} KiB): {plan}")
        return assignment, report


class PrefetchSequential(torch.nn.Module):
    """Runs `modules` in order like nn.Sequential, prefetching module i+1's parameters into L2
    on a side stream while module i runs, where a tuned plan pays (drop-in for
    research/l2-prefetch/src/api.py:27-66)."""

    def __init__(self, modules, example_input, min_bytes=64 << 10, rounds=7, log=None, min_lower_ci=1.0):
        super().__init__()
        self.layers = torch.nn.ModuleList(modules)
        ops = [m.__call__ for m in self.layers]
        reads = [_large(m.parameters(recurse=True), min_bytes) for m in self.layers]

        def make_runner(assignment):
            return ChainRunner(ops, reads, [assignment.get(i) for i in range(len(ops))])

        tuner = _GroupTuner([_signature(m, r) for m, r in zip(self.layers, reads)], reads, make_runner,
                            example_input, len(ops), rounds, min_lower_ci, log)
        with torch.no_grad():
            assignment, self.report = tuner.run("layers")
        self.runner = make_runner(assignment) if assignment else ChainRunner(ops, reads)

    def forward(self, x):
        return self.runner(x)


class _SideStream:
    """A side stream that prefetches after the issuing stream's work so far, and is joined
    back once per pass."""

    def __init__(self):
        self.stream = torch.cuda.Stream()
        self.pending = False

    def issue(self, after, tensors, plan):
        self.stream.wait_stream(after)
        with torch.cuda.stream(self.stream):
            for t in tensors:
                prefetch(t, **plan)
        self.pending = True

    def join(self, into):
        if self.pending:
            into.wait_stream(self.stream)
            self.pending = False


def trace_units(model, example_input, min_bytes):
    """[(module, [parameters it reads])] in first-call order of one no-grad forward."""
    members = {id(m) for m in model.modules()}
    order = []

    def record(module, args):
        if id(module) in members:
            order.append(module)

    handle = torch.nn.modules.module.register_module_forward_pre_hook(record)
    try:
        with torch.no_grad():
            model(example_input)
    finally:
        handle.remove()
    first = list({id(m): m for m in order}.values())
    called = {id(m) for m in first}
    owner = {}

    def assign(module, nearest):
        here = module if id(module) in called else nearest
        if here is not None and id(module) not in called:
            owner.setdefault(id(here), []).append(module)
        for child in module.children():
            assign(child, here)

    assign(model, None)
    units = []
    for m in first:
        params = list(m.parameters(recurse=False))
        for silent in owner.get(id(m), []):
            params += list(silent.parameters(recurse=False))
        reads = _large(params, min_bytes)
        if reads:
            units.append((m, reads))
    return units


class PrefetchHooks:
    """Prefetch for an unmodified model through hooks (drop-in for
    research/l2-prefetch/src/api.py:69-209). When unit i's forward starts, unit i+1's reads
    are prefetched; with backward=True, when unit i's backward starts, unit i-1's are.
    step(model, x) is what tuning times (default: the forward). remove() uninstalls."""

    def __init__(self, model, example_input, min_bytes=64 << 10, rounds=7, log=None, min_lower_ci=1.0,
                 backward=False, step=None):
        self.model, self.backward = model, backward
        self.step = step or (lambda m, x: m(x))
        self.units = trace_units(model, example_input, min_bytes)
        self.plans = {}
        self.handles = []
        self._side = _SideStream()
        self._active = False          # inside the root module's forward
        self._armed = False           # the root forward recorded autograd work to prefetch for
        self._fwd_stream = None
        self._install()

        def make_runner(assignment):
            def run(x):
                saved, self.plans = self.plans, assignment
                try:
                    return self.step(self.model, x)
                finally:
                    self.plans = saved
            return run

        tuner = _GroupTuner([_signature(m, r) for m, r in self.units], [r for _, r in self.units], make_runner,
                            example_input, 1, rounds, min_lower_ci, log)
        with torch.set_grad_enabled(backward):
            self.plans, self.report = tuner.run("units")

    def _prefetch(self, unit, after):
        plan = self.plans.get(unit)
        if plan is not None and 0 <= unit < len(self.units):
            self._side.issue(after, self.units[unit][1], plan)

    def _install(self):
        position = {id(m): i for i, (m, _) in enumerate(self.units)}

        def root_pre(module, args):
            self._active = True
            self._fwd_stream = torch.cuda.current_stream()

        def root_done(module, args, out):
            self._active = False
            self._armed = self.backward and torch.is_grad_enabled()
            self._side.join(torch.cuda.current_stream())

        def unit_pre(module, args):
            if self._active:   # a unit called outside the root's forward runs as plain torch
                self._prefetch(position[id(module)] + 1, torch.cuda.current_stream())

        def unit_back_pre(module, grad_output):
            # autograd runs a backward op on the stream of its forward op, which is not the
            # autograd thread's current stream under capture
            if self._armed:
                self._prefetch(position[id(module)] - 1, self._fwd_stream)

        def first_unit_back_done(module, grad_input, grad_output):   # unit 0's backward runs last
            self._armed = False
            self._side.join(self._fwd_stream)

        for m, _ in self.units:
            self.handles.append(m.register_forward_pre_hook(unit_pre))
            if self.backward:
                self.handles.append(m.register_full_backward_pre_hook(unit_back_pre))
        if self.backward and self.units:
            self.handles.append(self.units[0][0].register_full_backward_hook(first_unit_back_done))
        self.handles.append(self.model.register_forward_pre_hook(root_pre))
        self.handles.append(self.model.register_forward_hook(root_done))

    def remove(self):
        for h in self.handles:
            h.remove()
        self.handles.clear()
