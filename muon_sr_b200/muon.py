"""Muon with BF16 stochastic rounding on the B200 engine.

Public classes keep the reference's names, constructor signatures, param-group keys, state
keys and seed formulas (muon_sr/triton_muon_sr.py:180-373, muon_sr/muon_sr.py:234-418):

* ``TritonMuonSR``, ``TritonMuonSRWithAuxAdam`` -- deterministic seeds from (step, index).
* ``MuonSR``, ``MuonSRWithAuxAdam`` -- the reference's pure-PyTorch variants; here they run
  on the same CUDA kernels with seeds drawn from torch's default generator (the reference
  draws its rounding noise with ``torch.randint_like``), and keep those classes' state keys.

A Muon update is: a multi-tensor prepare kernel (momentum, Nesterov, SR momentum, RNE
update), the tcgen05 Newton-Schulz chain, and a multi-tensor apply kernel (decay, scaled
update, SR weights). With ``batch_ns`` the momentum of equal-shaped matrices lives in one
stack and Newton-Schulz runs on chunks of the stack. ``shard`` (optional) spreads the work
over the ranks of a process group (see ``sharding``).
"""
import contextlib

import torch
from torch.optim import Optimizer

from . import kernels as K
from . import staging
from .adamw import adamw_group_step
from .seeds import deterministic_seed

_nullctx = contextlib.nullcontext

# Max elements per batched Newton-Schulz call, as in the reference (triton_muon_sr.py:125).
# Each matrix is computed independently, so the bits do not depend on the chunking. Larger
# chunks fill the GEMM waves better, but measured on B200 inside a whole step 2^30 was
# slower (SM clock ~1260 vs ~1390 MHz under the 1 kW power cap, 483-497 vs 464-466 ms).
NS_CHUNK_NUMEL = 1 << 28

# Stacks whose matrices have a smaller dimension of at most this run on side streams,
# concurrently with each other and with the larger stacks: their Newton-Schulz GEMMs are too
# small to fill the GPU alone (tens of 256 x 256 tiles per launch, short K). Measured on B200:
# the GPT-2-small hybrid step (four stacks of smaller dimension 768) 4.17 -> 3.68 ms; the
# Llama-3-8B k/v stack (1024) gained nothing next to the large stacks. The streams are created
# once per device, outside any graph capture (the first step).
CONCURRENT_MAX_DIM = 768
SIDE_STREAMS = 4
_side = {}


def _side_streams(device):
    """(streams, start event) of a device; the event marks the start of a step."""
    entry = _side.get(device.index)
    if entry is None:
        entry = _side[device.index] = ([torch.cuda.Stream(device) for _ in range(SIDE_STREAMS)], torch.cuda.Event())
    return entry


# Option: in a stack of several Newton-Schulz chunks run on the step's stream (not sharded),
# the prepare of chunk c + 1 and the apply of chunk c run on a second stream while chunk c's
# Newton-Schulz runs. Same kernels and counters: the same bits. Off by default: measured on
# B200 in the Llama-3-8B step, 461.8 / 461.9 ms with it vs 461.8 / 463.3 ms without -- the
# step is bound by the 1 kW power cap, so overlapping moves energy around without saving it.
PIPELINE_CHUNKS = False
_ew = {}


def _ew_stream(device):
    s = _ew.get(device.index)
    if s is None:
        s = _ew[device.index] = torch.cuda.Stream(device)
    return s


# ---------------------------------------------------------------------------------------
# Step state
# ---------------------------------------------------------------------------------------
class _MomentumStacks:
    """Momentum of a batched Muon group: one bf16 ``[count, *shape]`` tensor per distinct
    parameter shape (shapes in order of first appearance) with each parameter's
    ``state["momentum_buffer"]`` a view of its row, so ``state_dict()`` still holds one buffer
    per parameter (muon_sr/muon_sr.py:112-146). A buffer already present in the state (a
    loaded checkpoint) is copied into its row."""

    def __init__(self, params, state):
        self.by_shape = {}
        for p in params:
            self.by_shape.setdefault(p.shape, []).append(p)
        self.tensor = {}
        self.row = {}
        for shape, members in self.by_shape.items():
            t = torch.zeros((len(members),) + tuple(shape), dtype=torch.bfloat16, device=members[0].device)
            for r, p in enumerate(members):
                self.row[id(p)] = r
                loaded = state[p].get("momentum_buffer")
                if loaded is not None:
                    t[r].copy_(loaded)
                state[p]["momentum_buffer"] = t[r]
            self.tensor[shape] = t


class _GlobalStep:
    """The batched groups' shared step counter (muon_sr/triton_muon_sr.py:13-15, 320-326): on
    first use after construction or ``load_state_dict`` it resumes from the largest "step"
    recorded in the state of those groups' parameters; it advances once per batched group
    per ``step()`` call and is recorded in the state of every parameter of that group."""

    def __init__(self):
        self.value = None

    def advance(self, state, groups, params):
        if self.value is None:
            self.value = max((state[p].get("step", 0) for g in groups for p in g["params"]), default=0)
        self.value += 1
        for p in params:
            state[p]["step"] = self.value
        return self.value


class _Seeder:
    """Seeds of one step: deterministic (Triton classes) or from torch's RNG (MuonSR)."""

    def __init__(self, random_seeds: bool):
        self.random = random_seeds

    def __call__(self, step, idx, salt):
        if self.random:
            return int(torch.randint(0, 1 << 32, (1,), dtype=torch.int64).item())
        return deterministic_seed(step, idx, salt)

    def skip(self, step, idx, salt):
        """Consume the seed of a tensor another rank updates, so that every rank draws the
        same sequence from torch's generator as a single-GPU run."""
        self(step, idx, salt)


def _grad_of(p):
    g = p.grad
    if g.dtype != torch.bfloat16:
        raise ValueError("gradients must be bfloat16")
    return g if g.is_contiguous() else g.contiguous()


def _validate(p, name):
    assert p.dtype == torch.bfloat16, "only bfloat16 is supported."
    if p.grad is not None and p.grad.is_sparse:
        raise RuntimeError(f"{name} does not support sparse gradients")


# ---------------------------------------------------------------------------------------
# Muon updates
# ---------------------------------------------------------------------------------------
def muon_single_step(p, buf, beta, nesterov, ns_steps, lr, weight_decay, step, param_idx, seeder):
    """Per-parameter Muon step (``_triton_muon_step``, triton_muon_sr.py:116-120)."""
    if p.ndim < 2:
        raise AssertionError("Newton-Schulz needs ndim >= 2 parameters")
    staging.need([p])
    update = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
    K.muon_prepare([(_grad_of(p), buf, update, 0, seeder(step, param_idx, 0))], beta, nesterov)
    out = K.newton_schulz(update, ns_steps)
    K.muon_apply([(p, out, K.ns_scale(p.shape), seeder(step, param_idx, 1))], lr, weight_decay)
    staging.done([p])


def _segments(n, count):
    """Split range(n) into ``count`` consecutive index ranges of near-equal length."""
    count = max(1, min(n, count))
    bounds = [n * s // count for s in range(count + 1)]
    return [range(bounds[s], bounds[s + 1]) for s in range(count)]


class _Work:
    """Where a batched step may do its work: ``owner(stack_idx, row) -> bool`` (None = all),
    ``share(params)`` after each stack / segment and ``segments(shape, n)`` (None = whole
    stacks), all from a ``sharding.Sharder``; ``side``: a stream on which the weight updates
    (apply) run after their chunk's Newton-Schulz, overlapping the next chunk (None: in line)."""

    def __init__(self, owner=None, share=None, segments=None, side=None):
        self.owner, self.share, self.segments, self.side = owner, share, segments, side

    def mine(self, stack_idx, row):
        return self.owner is None or self.owner(stack_idx, row)


def muon_batch_step(stacks, beta, nesterov, ns_steps, lr, weight_decay, step, seeder, work=None, after_first=None):
    """Batched step over the shape stacks (``_triton_muon_batch_step``,
    triton_muon_sr.py:128-177).

    For stack number s of ``stacks.by_shape`` (first-appearance order): prepare with seed
    S(step, s, 0) and counters running over the whole stack; Newton-Schulz on chunks of at most
    NS_CHUNK_NUMEL elements; apply of row r with S(step, s * 10000 + r, 1). Prepare, Newton-
    Schulz and apply are issued chunk by chunk (the prepare's counters are those of the whole
    stack, so the bits are the reference's), which keeps the scratch at one chunk and lets a
    ``staging.HostStaging`` step upload the next chunk's gradients meanwhile. A stack
    where only some parameters have gradients falls back to per-parameter steps with
    param_idx = s * 10000 + r. With ``work`` only this rank's rows are computed (seeds and
    counters stay global, so results do not depend on the number of ranks) and the weights
    are shared as they are finished. Without ``work``, stacks of small matrices (smaller
    dimension <= CONCURRENT_MAX_DIM) run on side streams that start with the step and join the
    current stream at its end; every stack touches only its own tensors, so the bits do not
    depend on the overlap. ``after_first`` (if given) is called once, after the first stack
    issued on the current stream (or at the end when there is none)."""
    work = work or _Work()
    order = list(enumerate(stacks.by_shape.items()))
    if work.share is not None and not seeder.random:
        # Largest stacks first, so that the stack whose weights are still in flight when the
        # step ends is the smallest. Seeds keep each stack's own index, so the bits do not
        # depend on this order (seeds drawn from torch's generator do: those keep the order).
        order.sort(key=lambda e: -len(e[1][1]) * K.numel_of(e[1][0]))
    concurrent = {s for s, (shape, _) in order
                  if work.share is None and len(shape) >= 2 and min(shape[-2:]) <= CONCURRENT_MAX_DIM
                  and stacks.tensor[shape].is_cuda}
    used = []
    if concurrent:
        device = next(stacks.tensor[shape].device for s, (shape, _) in order if s in concurrent)
        main = torch.cuda.current_stream(device)
        sides, start = _side_streams(device)
        start.record(main)
    for s, (shape, members) in order:
        if s in concurrent:
            side = sides[len(used) % len(sides)]
            side.wait_event(start)
            with torch.cuda.stream(side):
                _stack_step(s, shape, members, stacks.tensor[shape], beta, nesterov, ns_steps, lr, weight_decay,
                            step, seeder, work, pipeline=False)
            used.append(side)
        else:
            _stack_step(s, shape, members, stacks.tensor[shape], beta, nesterov, ns_steps, lr, weight_decay, step,
                        seeder, work)
            if after_first is not None:
                after_first()
                after_first = None
        if work.share is not None:
            work.share(members)
    if after_first is not None:
        after_first()
    for side in dict.fromkeys(used):
        main.wait_stream(side)


def _stack_step(s, shape, members, momentum, beta, nesterov, ns_steps, lr, weight_decay, step, seeder, work,
                pipeline=True):
    """One shape stack of ``muon_batch_step``. With ``work.segments`` the stack's rows are cut
    into consecutive segments; each rank runs its own rows segment by segment and
    ``work.share`` is called after every segment (on every rank, also when it owned none of
    it), so the weights start travelling while the rest of the stack computes. Chunks never
    span segments; the bits are those of the unsegmented step. ``pipeline`` allows the
    pipelined chunk loop (``PIPELINE_CHUNKS``); stacks that already run on a side stream
    pass False."""
    if all(p.grad is None for p in members):
        return
    if any(p.grad is None for p in members):
        for r, p in enumerate(members):
            if p.grad is None:
                continue
            if work.mine(s, r):
                muon_single_step(p, momentum[r], beta, nesterov, ns_steps, lr, weight_decay, step, s * 10000 + r,
                                 seeder)
            else:
                seeder.skip(step, s * 10000 + r, 0)
                seeder.skip(step, s * 10000 + r, 1)
        return
    if len(shape) < 2:
        raise AssertionError("Newton-Schulz needs ndim >= 2 parameters")
    rows = [r for r in range(len(members)) if work.mine(s, r)]
    parts = _segments(len(members), work.segments(shape, len(members)) if (work.segments and work.share) else 1)
    numel = K.numel_of(shape)
    # seeds in the single-GPU draw order: the stack's prepare seed, then one apply seed per
    # row in row order (all of them on every rank)
    prep_seed = seeder(step, s, 0)
    apply_seed = [seeder(step, s * 10000 + r, 1) for r in range(len(members))]
    chunk = max(1, NS_CHUNK_NUMEL // max(1, numel))
    scale = K.ns_scale(shape)
    if pipeline and PIPELINE_CHUNKS and work.share is None and momentum.is_cuda and len(rows) > chunk:
        _pipelined_chunks(members, rows, chunk, momentum, numel, prep_seed, apply_seed, scale, shape, beta, nesterov,
                          ns_steps, lr, weight_decay)
        return
    upd = torch.empty((min(chunk, len(rows)),) + tuple(shape), dtype=torch.bfloat16, device=momentum.device) \
        if rows else None
    lo = 0  # first position in `rows` of the current segment
    for part in parts:
        hi = lo
        while hi < len(rows) and rows[hi] in part:
            hi += 1
        for c in range(lo, hi, chunk):
            # prepare of the chunk's rows with the stack's seed and counters: the same bits as
            # one prepare over the whole stack
            mine = [members[rows[c + j]] for j in range(min(chunk, hi - c))]
            staging.need(mine)
            x = upd[:len(mine)]
            K.muon_prepare([(_grad_of(p), momentum[rows[c + j]], x[j], rows[c + j] * numel, prep_seed)
                            for j, p in enumerate(mine)], beta, nesterov)
            out = K.newton_schulz(x, ns_steps)
            items = [(p, out[j], scale, apply_seed[rows[c + j]]) for j, p in enumerate(mine)]
            if work.side is not None:
                # the weight update on the side stream: it waits for this chunk's Newton-Schulz
                # only, so its (multicast) stores overlap the next chunk's GEMMs
                ns_done = torch.cuda.Event()
                ns_done.record()
                with torch.cuda.stream(work.side):
                    work.side.wait_event(ns_done)
                    out.record_stream(work.side)
                    K.muon_apply(items, lr, weight_decay)
                    staging.done(mine)
            else:
                K.muon_apply(items, lr, weight_decay)
                staging.done(mine)
            del out
        lo = hi
        if len(parts) > 1:
            work.share([members[r] for r in part])
    del upd


def _pipelined_chunks(members, rows, chunk, momentum, numel, prep_seed, apply_seed, scale, shape, beta, nesterov,
                      ns_steps, lr, weight_decay):
    """The chunk loop of ``_stack_step`` with the elementwise work on a second stream: prepare
    of chunk i + 1 and apply of chunk i overlap the Newton-Schulz of chunk i. Two update
    buffers alternate; the prepare writing one waits until the Newton-Schulz two chunks back
    has read it. The current stream waits for the second one at the end."""
    device = momentum.device
    main = torch.cuda.current_stream(device)
    ew = _ew_stream(device)
    groups = [rows[c:c + chunk] for c in range(0, len(rows), chunk)]
    bufs = [torch.empty((chunk,) + tuple(shape), dtype=torch.bfloat16, device=device) for _ in range(2)]
    start = torch.cuda.Event()
    start.record(main)
    ew.wait_event(start)
    ns_done = []

    def prepare(i):
        with torch.cuda.stream(ew):
            if i >= 2:
                ew.wait_event(ns_done[i - 2])
            mine = [members[r] for r in groups[i]]
            staging.need(mine)
            x = bufs[i % 2][:len(mine)]
            K.muon_prepare([(_grad_of(p), momentum[r], x[j], r * numel, prep_seed)
                            for j, (p, r) in enumerate(zip(mine, groups[i]))], beta, nesterov)
            ready = torch.cuda.Event()
            ready.record(ew)
        return x, ready

    nxt = prepare(0)
    for i, grp in enumerate(groups):
        x, ready = nxt
        main.wait_event(ready)
        out = K.newton_schulz(x, ns_steps)
        done = torch.cuda.Event()
        done.record(main)
        ns_done.append(done)
        if i + 1 < len(groups):
            nxt = prepare(i + 1)
        with torch.cuda.stream(ew):
            ew.wait_event(done)
            out.record_stream(ew)
            mine = [members[r] for r in grp]
            K.muon_apply([(p, out[j], scale, apply_seed[r]) for j, (p, r) in enumerate(zip(mine, grp))], lr,
                         weight_decay)
            staging.done(mine)
        del out
    main.wait_stream(ew)
    del bufs


# ---------------------------------------------------------------------------------------
# Optimizers
# ---------------------------------------------------------------------------------------
class _MuonBase(Optimizer):
    """Shared machinery of the Muon classes: batched-group stacks, the global step, seeds
    and the optional sharder."""

    _random_seeds = False   # True: seeds from torch's generator (MuonSR classes)
    _record_step = True     # False: no "step" in the Muon state (MuonSR classes)

    def _setup(self, shard):
        self._shard = shard
        self._reset_batched()

    def _reset_batched(self):
        self._stacks = {}
        self._clock = _GlobalStep()

    def load_state_dict(self, state_dict):
        # stacks and the global step are rebuilt from the loaded state on the next step
        # (muon_sr/muon_sr.py:149-158)
        super().load_state_dict(state_dict)
        self._reset_batched()

    def _run_muon_group(self, gi, group, batched, batched_groups, seeder, after_first=None):
        name = type(self).__name__
        beta, nesterov, ns_steps = group["momentum"], group["nesterov"], group["ns_steps"]
        lr, wd = group["lr"], group["weight_decay"]
        sh = self._shard
        if batched:
            if id(group) not in self._stacks:
                self._stacks[id(group)] = _MomentumStacks(group["params"], self.state)
            stacks = self._stacks[id(group)]
            for p in group["params"]:
                _validate(p, name)
            step = self._clock.advance(self.state, batched_groups, group["params"]) if self._record_step else 0
            work = _Work(sh.muon_owner(gi, stacks.by_shape), sh.share, sh.segments, sh.update_stream) if sh else None
            muon_batch_step(stacks, beta, nesterov, ns_steps, lr, wd, step, seeder, work, after_first)
            return
        for i, p in enumerate(group["params"]):
            _validate(p, name)
            if p.grad is None:
                continue
            st = self.state[p]
            if not st:
                if self._record_step:
                    st["step"] = 0
                st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.bfloat16)
            if self._record_step:
                st["step"] += 1
            step = st.get("step", 0)
            if sh and not sh.owns(gi, i):
                seeder.skip(step, i, 0)
                seeder.skip(step, i, 1)
                continue
            muon_single_step(p, st["momentum_buffer"], beta, nesterov, ns_steps, lr, wd, step, i, seeder)
            if after_first is not None:
                after_first()
                after_first = None
        if after_first is not None:
            after_first()
        if sh:
            sh.share(group["params"])


class TritonMuonSR(_MuonBase):
    r"""Muon for bf16 matrices with stochastic rounding (drop-in for muon_sr.TritonMuonSR,
    muon_sr/triton_muon_sr.py:180-255).

    Arguments:
        params: ndim >= 2 parameters to optimize
        lr (float): learning rate (default: 0.02)
        weight_decay (float): weight decay (default: 0)
        momentum (float): momentum coefficient (default: 0.95)
        nesterov (bool): Nesterov momentum (default: True)
        ns_steps (int): Newton-Schulz iterations (default: 5)
        batch_ns (bool): stacked momentum buffers, Newton-Schulz batched by shape (default: False)
        shard: optional ``sharding.Sharder`` spreading the matrices over ranks
    """

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95, nesterov=True, ns_steps=5, batch_ns=False,
                 shard=None):
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                                      ns_steps=ns_steps, batch_ns=batch_ns))
        self._setup(shard)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._shard:
            self._shard.bind(self)
        seeder = _Seeder(self._random_seeds)
        batched_groups = [g for g in self.param_groups if g["batch_ns"]]
        for gi, group in enumerate(self.param_groups):
            self._run_muon_group(gi, group, group["batch_ns"], batched_groups, seeder)
        if self._shard:
            self._shard.sync_params(self)
        return loss


class MuonSR(TritonMuonSR):
    r"""``muon_sr.MuonSR`` (muon_sr/muon_sr.py:234-302) on the CUDA engine: same arguments and
    state keys (``momentum_buffer`` only); SR noise seeded from torch's default generator."""

    _random_seeds = True
    _record_step = False


_MUON_DEFAULTS = dict(lr=0.02, momentum=0.95, nesterov=True, ns_steps=5, weight_decay=0)
_ADAM_DEFAULTS = dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0)


class TritonMuonSRWithAuxAdam(_MuonBase):
    r"""Hybrid Muon + AdamW with stochastic rounding (drop-in for
    muon_sr.TritonMuonSRWithAuxAdam, muon_sr/triton_muon_sr.py:258-373).

    Arguments:
        param_groups: list of param group dicts, each with a ``use_muon`` flag
        batch_ns (bool): stacked momentum buffers, Newton-Schulz batched by shape (default: False)
        shard: optional ``sharding.Sharder`` spreading the work over ranks
    """

    def __init__(self, param_groups, batch_ns=False, shard=None):
        for group in param_groups:
            assert "use_muon" in group
            for key, value in (_MUON_DEFAULTS if group["use_muon"] else _ADAM_DEFAULTS).items():
                group.setdefault(key, value)
        self.batch_ns = batch_ns
        super().__init__(param_groups, {})
        self._setup(shard)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        sh = self._shard
        if sh:
            sh.bind(self)
        seeder = _Seeder(self._random_seeds)
        groups = self.param_groups
        offsets = [sum(len(g["params"]) for g in groups[:gi]) for gi in range(len(groups))]
        muon_groups = [g for g in groups if g["use_muon"]]
        order = range(len(groups))
        if sh and not self._random_seeds:
            # AdamW groups (embedding, head) first so their transfers overlap the Muon work;
            # every group's math is independent of the processing order (seeds drawn from
            # torch's generator are not: those classes keep the order).
            order = sorted(order, key=lambda gi: bool(groups[gi]["use_muon"]))

        def adam(gi):
            group = groups[gi]
            side = sh.update_stream if sh else None
            with torch.cuda.stream(side) if side is not None else _nullctx():
                # (multicast weights: the AdamW updates run under the Muon groups' GEMMs)
                adamw_group_step(self.state, group, offsets[gi], lambda step, idx: seeder(step, idx, 0),
                                 owns=(lambda i, gi=gi: sh.owns(gi, i)) if sh else None)
            if sh:
                sh.share(group["params"])

        # Fed from host memory (HostStaging), the AdamW groups run right after the first Muon
        # stack: the download of their weights then overlaps the remaining Newton-Schulz work
        # instead of trailing the step, and their uploads queue behind that stack's. Bits do
        # not depend on the order; seeds drawn from torch's generator do, so those classes
        # keep it.
        deferred = [gi for gi in order if not groups[gi]["use_muon"]] \
            if staging.active() and not sh and not self._random_seeds and muon_groups else []
        skip = set(deferred)

        def run_deferred():
            while deferred:
                adam(deferred.pop(0))

        for gi in order:
            group = groups[gi]
            if group["use_muon"]:
                if group["params"]:
                    self._run_muon_group(gi, group, self.batch_ns, muon_groups, seeder,
                                         after_first=run_deferred if deferred else None)
                continue
            if gi not in skip:
                adam(gi)
        run_deferred()
        if sh:
            sh.sync_params(self)
        return loss


class MuonSRWithAuxAdam(TritonMuonSRWithAuxAdam):
    r"""``muon_sr.MuonSRWithAuxAdam`` (muon_sr/muon_sr.py:305-418) on the CUDA engine: same
    arguments and state keys; SR noise seeded from torch's default generator."""

    _random_seeds = True
    _record_step = False
