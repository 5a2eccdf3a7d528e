"""Whole optimizer steps as CUDA graphs, replayed every step without capturing again.

``StepGraph(optimizer)`` captures one complete ``optimizer.step()`` -- every prepare,
Newton-Schulz, apply, centralisation and AdamW launch of it -- into a CUDA graph, and
``StepGraph.step()`` replays it. The multi-tensor launches inside the graph are the C ABI's
replayable ``*_rec`` variants: their kernels read the launch scalars and the per-tensor
entries (Philox keys, bias corrections, learning rates, decays) from records in device
memory. Each ``step()`` first runs the optimizer's own Python bookkeeping once more in a
refresh pass that issues no kernels -- step counters, seeds (deterministic, or drawn from
torch's generator in the eager order), the param groups' current hyperparameters -- and
writes the new scalars into a pinned host copy of the records; the graph's first node copies
that host copy to the device. Pointers and sizes stay those of the capture, so a replay
produces the eager step's bits, and a step whose structure differs from the capture (other
parameters with gradients, another tensor behind a ``.grad``, another launch sequence) is
refused rather than replayed.

Two graphs are captured (sharing one memory pool), each with its own record area, and
replayed alternately, so the host refreshes step k + 1 while step k runs. The sizing and
capture passes restore the optimizer's step counters and torch's RNG state, so building a
StepGraph does not advance the optimizer.

Requirements: one eager ``step()`` before construction (the optimizer state exists); the
parameters, their ``.grad`` tensors and the optimizer state keep their storage; one stream;
no ``Sharder``. The 8-bit optimizer is not captured (its step is one launch). The capture
uses CUDA's global capture mode, so no other thread of the process should issue CUDA work
(e.g. collectives in flight) while a StepGraph is being built.

The replay saves the host's launch work -- the per-launch C-ABI and CUDA launch costs, most
of all the ~16 launches and tensor-map encodings of every Newton-Schulz call -- which matters
when a step's GPU work is short; the Python bookkeeping of the refresh pass remains.
"""
import ctypes

import torch

from . import _lib
from . import kernels as K

# Entry fields a replay refreshes: everything except pointers and sizes.
_SCALAR_FIELDS = {
    "msr_muon_prepare_rec": ("ctr_base", "key"),
    "msr_muon_apply_rec": ("key", "scale"),
    "msr_adamw_sr_rec": ("key_m", "key_v", "key_p", "step_size", "bc2_sqrt"),
}

_CHANGED = ("the optimizer step no longer matches its captured graph (parameters with gradients, "
            "gradient tensors, shapes, baked-in constants or the launch sequence changed); build a new StepGraph")


def _align(n: int, a: int = 16) -> int:
    return (n + a - 1) // a * a


class _Launch:
    """One launch of a pass: its record (ctypes header + entries) and its place in the area."""
    __slots__ = ("fn", "offset", "header", "entries", "numels")

    def __init__(self, fn, offset, header, entries):
        self.fn, self.offset, self.header, self.entries = fn, offset, header, entries
        self.numels = [int(e.numel) for e in entries]


class _Recorder:
    """Installed with ``kernels.recorder`` during a pass: "measure" sizes the records,
    "record" writes them and issues the replayable launches (inside the capture), "refresh"
    rewrites the scalars of a capture's records and issues nothing."""

    def __init__(self, mode, host=None, dev=None, plan=None, constants=None):
        self.mode = mode
        self.launches = mode == "record"
        self.host, self.dev = host, dev
        self.plan = [] if plan is None else plan
        self.constants = [] if constants is None else constants
        self.size = 0
        self.cursor = 0
        self.seen = 0
        self.held = []  # scratch tensors the captured kernels use (kept alive with the graph)

    def hold(self, tensor):
        """Keep ``tensor`` alive as long as the captured graph: its address is baked in."""
        if not any(t is tensor for t in self.held):
            self.held.append(tensor)

    def constant(self, name, value):
        """A scalar the capture bakes into a kernel's parameters: a refresh must see the same."""
        if self.mode == "refresh":
            if self.seen >= len(self.constants) or self.constants[self.seen] != (name, value):
                raise RuntimeError(_CHANGED)
        else:
            self.constants.append((name, value))
        self.seen += 1

    def launch(self, fn, header, entries, device):
        if self.mode == "refresh":
            self._refresh(fn, header, entries)
            return
        offset = self.size
        self.size = _align(offset + ctypes.sizeof(header) + ctypes.sizeof(entries))
        launch = _Launch(fn, offset, header, entries)
        if self.mode == "record":
            if self.size > self.host.numel():
                raise RuntimeError(_CHANGED)
            self._write(launch)
            status = getattr(_lib.load(), fn)(entries, len(entries), ctypes.c_void_p(self.dev.data_ptr() + offset),
                                              K.stream_handle(device))
            _lib.check(status, fn)
        self.plan.append(launch)

    def _write(self, launch):
        base = self.host.data_ptr() + launch.offset
        hdr = ctypes.sizeof(launch.header)
        ctypes.memmove(base, ctypes.addressof(launch.header), hdr)
        ctypes.memmove(base + hdr, ctypes.addressof(launch.entries), ctypes.sizeof(launch.entries))

    def _refresh(self, fn, header, entries):
        if self.cursor >= len(self.plan):
            raise RuntimeError(_CHANGED)
        cap = self.plan[self.cursor]
        if cap.fn != fn or cap.numels != [int(e.numel) for e in entries]:
            raise RuntimeError(_CHANGED)
        for old, new in zip(cap.entries, entries):
            for f in _SCALAR_FIELDS[fn]:
                setattr(old, f, getattr(new, f))
        cap.header = header
        self._write(cap)
        self.cursor += 1

    def complete(self):
        return self.cursor == len(self.plan) and self.seen == len(self.constants)


def _snapshot(opt):
    """The host-side state a pass advances: non-tensor optimizer state (step counters), the
    batched groups' global step and torch's CPU generator (seeds of the MuonSR classes)."""
    state = {p: {k: v for k, v in st.items() if not torch.is_tensor(v)} for p, st in opt.state.items()}
    clock = getattr(opt, "_clock", None)
    return state, (clock.value if clock is not None else None), torch.get_rng_state()


def _restore(opt, snap):
    state, clock, rng = snap
    for p in list(opt.state.keys()):
        saved = state.get(p)
        if saved is None:
            del opt.state[p]
            continue
        st = opt.state[p]
        for k in [k for k, v in st.items() if not torch.is_tensor(v) and k not in saved]:
            del st[k]
        st.update(saved)
    if getattr(opt, "_clock", None) is not None:
        opt._clock.value = clock
    torch.set_rng_state(rng)


class _Slot:
    __slots__ = ("graph", "host", "dev", "plan", "constants", "done", "held")


class StepGraph:
    """Capture ``optimizer.step()`` once, replay it at every ``step()`` (see the module doc).

    Arguments:
        optimizer: a TritonMuonSR, TritonMuonSRWithAuxAdam, MuonSR, MuonSRWithAuxAdam or
            TritonAdamW that has run one eager step with the gradients the replays will use
        copies: graphs replayed alternately (2 lets the host refresh one while the other runs)
    """

    def __init__(self, optimizer, copies: int = 2):
        from .adamw import TritonAdamW
        from .muon import _MuonBase
        if not isinstance(optimizer, (_MuonBase, TritonAdamW)):
            raise TypeError("StepGraph captures the Muon classes and TritonAdamW of muon_sr_b200")
        if getattr(optimizer, "_shard", None) is not None:
            raise ValueError("StepGraph does not capture sharded steps")
        if copies < 1:
            raise ValueError("copies must be >= 1")
        self.optimizer = optimizer
        self._params = [p for g in optimizer.param_groups for p in g["params"]]
        with_grad = [p for p in self._params if p.grad is not None]
        if not with_grad:
            raise RuntimeError("no parameter has a gradient")
        if not all(p in optimizer.state and optimizer.state[p] for p in with_grad):
            raise RuntimeError("run one eager optimizer.step() before capturing it")
        self._device = with_grad[0].device
        self._grads = self._grad_ptrs()
        self._storage = None  # where the captured kernels write: taken after the first capture

        sizing = self._pass(_Recorder("measure"))
        size = max(16, sizing.size)
        self._slots = []
        pool = None
        for _ in range(copies):
            s = _Slot()
            s.host = torch.zeros(size, dtype=torch.uint8, pin_memory=True)
            s.dev = torch.zeros(size, dtype=torch.uint8, device=self._device)
            s.graph = torch.cuda.CUDAGraph()
            rec = _Recorder("record", s.host, s.dev)
            snap = _snapshot(optimizer)
            try:
                with K.recorder(rec), torch.cuda.graph(s.graph, pool=pool):
                    s.dev.copy_(s.host, non_blocking=True)
                    optimizer.step()
            finally:
                _restore(optimizer, snap)
            if [x.numels for x in rec.plan] != [x.numels for x in sizing.plan] or rec.constants != sizing.constants:
                raise RuntimeError(_CHANGED)
            storage = self._storage_ptrs()  # a pass may have built state (stacks after a load)
            if self._storage is not None and storage != self._storage:
                raise RuntimeError(_CHANGED)
            self._storage = storage
            pool = s.graph.pool()
            s.plan, s.constants, s.held = rec.plan, rec.constants, rec.held
            s.done = torch.cuda.Event()
            self._slots.append(s)
        self._next = 0
        self.records = len(sizing.plan)  # replayable multi-tensor launches per step

    def _grad_ptrs(self):
        return [p.grad.data_ptr() if p.grad is not None else None for p in self._params]

    def _storage_ptrs(self):
        """Where the parameters and their state tensors live: the captured kernels write there,
        so a replay after any of them moved (``load_state_dict`` rebuilds the momentum stacks,
        ``.to()`` moves parameters) would write to stale memory and is refused."""
        out = []
        for p in self._params:
            st = self.optimizer.state.get(p, {})
            out.append((p.data_ptr(), tuple((k, v.data_ptr()) for k, v in sorted(st.items()) if torch.is_tensor(v))))
        return out

    def _pass(self, rec):
        snap = _snapshot(self.optimizer)
        try:
            with K.recorder(rec):
                self.optimizer.step()
        finally:
            _restore(self.optimizer, snap)
        return rec

    def step(self):
        """One optimizer step: refresh the scalars on the host, replay the graph."""
        if self._grad_ptrs() != self._grads or self._storage_ptrs() != self._storage:
            raise RuntimeError(_CHANGED)
        s = self._slots[self._next]
        s.done.synchronize()  # the previous replay of this graph has read its records
        rec = _Recorder("refresh", s.host, s.dev, plan=s.plan, constants=s.constants)
        snap = _snapshot(self.optimizer)
        ok = False
        try:
            with K.recorder(rec):
                self.optimizer.step()
            # the pass itself may have moved state (momentum stacks rebuilt after a load)
            ok = rec.complete() and self._storage_ptrs() == self._storage
        finally:
            if not ok:
                _restore(self.optimizer, snap)  # a refused step leaves the optimizer as it was
        if not ok:
            raise RuntimeError(_CHANGED)
        s.graph.replay()
        s.done.record()
        self._next = (self._next + 1) % len(self._slots)
