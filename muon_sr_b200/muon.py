"""Muon with BF16 stochastic rounding on the B200 engine.

Public classes keep the reference's names, constructor signatures, param-group keys, state
keys and seed formulas (muon_sr/triton_muon_sr.py:180-373, muon_sr/muon_sr.py:234-418):

* ``TritonMuonSR``, ``TritonMuonSRWithAuxAdam`` -- deterministic seeds from (step, index).
* ``MuonSR``, ``MuonSRWithAuxAdam`` -- the reference's pure-PyTorch variants; here they run
  on the same CUDA kernels with seeds drawn from torch's default generator (the reference
  draws its rounding noise with ``torch.randint_like``), and keep those classes' state keys.

Every step is: a multi-tensor prepare kernel (momentum, Nesterov, SR momentum, RNE update),
the tcgen05 Newton-Schulz chain over each shape stack,
and a multi-tensor apply kernel (decay, scaled update, SR weights). ``shard`` (optional)
spreads the matrices over the ranks of a process group (see ``sharding``).
"""
from collections import defaultdict

import torch
from torch.optim import Optimizer

from . import kernels as K
from .seeds import deterministic_seed

# Max elements per batched Newton-Schulz call, as in the reference (triton_muon_sr.py:125).
# Each matrix is computed independently, so results do not depend on the chunking.
NS_CHUNK_NUMEL = 1 << 28


def _restore_global_step(state, groups):
    """muon_sr/triton_muon_sr.py:13-15."""
    return max((state[p].get("step", 0) for g in groups for p in g["params"]), default=0)


def _init_stacked_bufs(params, device, state):
    """One bf16 [N, *shape] momentum stack per distinct shape; ``state[p]["momentum_buffer"]``
    is a view into it (muon_sr/muon_sr.py:112-146)."""
    shape_groups = defaultdict(list)
    for p in params:
        shape_groups[p.shape].append(p)
    stacked_bufs, buf_indices = {}, {}
    for shape, grp in shape_groups.items():
        stacked = torch.zeros(len(grp), *shape, dtype=torch.bfloat16, device=device)
        for i, p in enumerate(grp):
            buf_indices[id(p)] = i
            p_state = state[p]
            if "momentum_buffer" in p_state:
                stacked[i].copy_(p_state["momentum_buffer"])
            p_state["momentum_buffer"] = stacked[i]
        stacked_bufs[shape] = stacked
    return dict(shape_groups), stacked_bufs, buf_indices


class _StackedBufsMixin:
    """Stacked buffers and the global step live outside ``self.state``; rebuild them from
    the loaded state on the next step (muon_sr/muon_sr.py:149-158)."""

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        self._batch_state = {}
        self.__dict__.pop("_global_step", None)


def _grad_of(p):
    g = p.grad
    if g.dtype != torch.bfloat16:
        raise ValueError("gradients must be bfloat16")
    return g if g.is_contiguous() else g.contiguous()


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


def muon_single_step(p, grad, buf, beta, nesterov, ns_steps, lr, weight_decay, step, param_idx, seeder):
    """Per-parameter Muon step (``_triton_muon_step``, triton_muon_sr.py:116-120)."""
    if p.ndim < 2:
        raise AssertionError("Newton-Schulz needs ndim >= 2 parameters")
    update = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
    K.muon_prepare([(grad, buf, update, 0, seeder(step, param_idx, 0))], beta, nesterov)
    out = K.newton_schulz(update, ns_steps)
    K.muon_apply([(p, out, K.ns_scale(p.shape), seeder(step, param_idx, 1))], lr, weight_decay)


def muon_batch_step(shape_groups, stacked_bufs, buf_indices, beta, nesterov, ns_steps, lr, weight_decay, step,
                    seeder, owner=None, share=None, segments=None):
    """Batched step over shape stacks (``_triton_muon_batch_step``, triton_muon_sr.py:128-177).

    Prepare runs once per stack with seed S(step, shape_idx, 0) and counters running over the
    whole stack; Newton-Schulz runs on chunks of the stack; apply uses
    S(step, shape_idx * 10000 + i, 1). A stack where only some parameters have gradients
    falls back to per-parameter steps with param_idx = shape_idx * 10000 + i.
    ``owner(shape_idx, i) -> bool`` restricts the work to this rank's matrices; seeds and
    counters stay global, so results do not depend on the number of ranks. ``share(params)``
    is called after each stack (and, with ``segments``, after each segment of a stack) so its
    weights can travel while the rest computes.
    """
    stacks = list(enumerate(shape_groups.items()))
    if share is not None and not seeder.random:
        # Largest stacks first, so that the stack whose weights are still in flight when the
        # step ends is the smallest. Seeds keep each stack's own index, so the bits do not
        # depend on this order (seeds drawn from torch's generator do: those keep the order).
        stacks.sort(key=lambda e: -len(e[1][1]) * K.numel_of(e[1][0]))
    for shape_idx, (shape, grp) in stacks:
        _stack_step(shape_idx, shape, grp, stacked_bufs, buf_indices, beta, nesterov, ns_steps, lr, weight_decay,
                    step, seeder, owner, share, segments)
        if share is not None:
            share(grp)


def _segments(n, count):
    """Split range(n) into ``count`` consecutive index ranges of near-equal length."""
    count = max(1, min(n, count))
    bounds = [n * s // count for s in range(count + 1)]
    return [range(bounds[s], bounds[s + 1]) for s in range(count)]


def _stack_step(shape_idx, shape, grp, stacked_bufs, buf_indices, beta, nesterov, ns_steps, lr, weight_decay, step,
                seeder, owner, share=None, segments=None):
    """One shape stack of ``muon_batch_step``. With ``segments(shape, n) -> count`` the
    stack's global index range is cut into that many consecutive segments; each rank runs
    its own matrices segment by segment and ``share`` is called after every segment (on
    every rank, also when it owned none of it), so the weights start travelling while the
    rest of the stack computes. Chunks never span segments; the bits are those of the
    unsegmented step."""
    active = [p for p in grp if p.grad is not None]
    if not active:
        return
    stacked_buf = stacked_bufs[shape]
    if len(active) < len(grp):
        for p in active:
            i = buf_indices[id(p)]
            if owner is None or owner(shape_idx, i):
                muon_single_step(p, _grad_of(p), stacked_buf[i], beta, nesterov, ns_steps, lr, weight_decay,
                                 step, shape_idx * 10000 + i, seeder)
            else:
                seeder.skip(step, shape_idx * 10000 + i, 0)
                seeder.skip(step, shape_idx * 10000 + i, 1)
        return
    mine = [i for i in range(len(grp)) if owner is None or owner(shape_idx, i)]
    segs = _segments(len(grp), segments(shape, len(grp)) if (segments and share) else 1)
    if len(shape) < 2:
        raise AssertionError("Newton-Schulz needs ndim >= 2 parameters")
    numel = K.numel_of(shape)
    work = None
    # seeds in the single-GPU draw order: the stack's prepare seed, then one apply seed per
    # matrix in index order (all of them on every rank)
    prep_seed = seeder(step, shape_idx, 0)
    apply_seeds = [seeder(step, shape_idx * 10000 + i, 1) for i in range(len(grp))]
    if mine:
        work = torch.empty(len(mine), *shape, dtype=torch.bfloat16, device=stacked_buf.device)
        K.muon_prepare([(_grad_of(grp[i]), stacked_buf[i], work[j], i * numel, prep_seed)
                        for j, i in enumerate(mine)], beta, nesterov)
    k = max(1, NS_CHUNK_NUMEL // max(1, numel))
    scale = K.ns_scale(shape)
    pos = 0  # position in `mine` (and `work`) where the current segment starts
    for seg in segs:
        end = pos
        while end < len(mine) and mine[end] in seg:
            end += 1
        for s in range(pos, end, k):
            out = K.newton_schulz(work[s:min(s + k, end)], ns_steps)
            K.muon_apply([(grp[mine[s + j]], out[j], scale, apply_seeds[mine[s + j]]) for j in range(out.shape[0])],
                         lr, weight_decay)
            del out
        pos = end
        if len(segs) > 1:
            share([grp[i] for i in seg])
    del work


def _check_params(params, name):
    for p in params:
        assert p.dtype == torch.bfloat16, "only bfloat16 is supported."
        if p.grad is not None and p.grad.is_sparse:
            raise RuntimeError(f"{name} does not support sparse gradients")


class TritonMuonSR(_StackedBufsMixin, Optimizer):
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

    _random_seeds = False
    _record_step = True

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95, nesterov=True, ns_steps=5, batch_ns=False,
                 shard=None):
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                        batch_ns=batch_ns)
        super().__init__(params, defaults)
        self._batch_state = {}
        self._shard = shard

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        seeder = _Seeder(self._random_seeds)
        name = type(self).__name__
        if self._shard:
            self._shard.bind(self)
        for gi, group in enumerate(self.param_groups):
            lr, wd = group["lr"], group["weight_decay"]
            beta, nesterov, ns_steps = group["momentum"], group["nesterov"], group["ns_steps"]
            if group["batch_ns"]:
                gid = id(group)
                if gid not in self._batch_state:
                    self._batch_state[gid] = _init_stacked_bufs(group["params"], group["params"][0].device, self.state)
                shape_groups, stacked_bufs, buf_indices = self._batch_state[gid]
                _check_params(group["params"], name)
                step = 0
                if self._record_step:
                    if not hasattr(self, "_global_step"):
                        self._global_step = _restore_global_step(
                            self.state, [g for g in self.param_groups if g["batch_ns"]])
                    self._global_step += 1
                    step = self._global_step
                    for p in group["params"]:
                        self.state[p]["step"] = self._global_step
                owner = self._shard.muon_owner(gi, shape_groups) if self._shard else None
                muon_batch_step(shape_groups, stacked_bufs, buf_indices, beta, nesterov, ns_steps, lr, wd, step,
                                seeder, owner, self._shard.share if self._shard else None,
                                self._shard.segments if self._shard else None)
            else:
                for param_idx, p in enumerate(group["params"]):
                    assert p.dtype == torch.bfloat16, "only bfloat16 is supported."
                    if p.grad is None:
                        continue
                    if p.grad.is_sparse:
                        raise RuntimeError(f"{name} does not support sparse gradients")
                    state = self.state[p]
                    if len(state) == 0:
                        if self._record_step:
                            state["step"] = 0
                        state["momentum_buffer"] = torch.zeros_like(p, dtype=torch.bfloat16)
                    if self._record_step:
                        state["step"] += 1
                    if self._shard and not self._shard.owns(gi, param_idx):
                        seeder.skip(state.get("step", 0), param_idx, 0)
                        seeder.skip(state.get("step", 0), param_idx, 1)
                        continue
                    muon_single_step(p, _grad_of(p), state["momentum_buffer"], beta, nesterov, ns_steps, lr, wd,
                                     state.get("step", 0), param_idx, seeder)
                if self._shard:
                    self._shard.share(group["params"])
        if self._shard:
            self._shard.sync_params(self)
        return loss


class MuonSR(TritonMuonSR):
    r"""``muon_sr.MuonSR`` (muon_sr/muon_sr.py:234-302) on the CUDA engine: same arguments and
    state keys (``momentum_buffer`` only); SR noise seeded from torch's default generator."""

    _random_seeds = True
    _record_step = False


class TritonMuonSRWithAuxAdam(_StackedBufsMixin, Optimizer):
    r"""Hybrid Muon + AdamW with stochastic rounding (drop-in for
    muon_sr.TritonMuonSRWithAuxAdam, muon_sr/triton_muon_sr.py:258-373).

    Arguments:
        param_groups: list of param group dicts, each with a ``use_muon`` flag
        batch_ns (bool): stacked momentum buffers, Newton-Schulz batched by shape (default: False)
        shard: optional ``sharding.Sharder`` spreading the work over ranks
    """

    _random_seeds = False
    _record_muon_step = True

    def __init__(self, param_groups, batch_ns=False, shard=None):
        for group in param_groups:
            assert "use_muon" in group
            if group["use_muon"]:
                group.setdefault("lr", 0.02)
                group.setdefault("momentum", 0.95)
                group.setdefault("nesterov", True)
                group.setdefault("ns_steps", 5)
                group.setdefault("weight_decay", 0)
            else:
                group.setdefault("lr", 3e-4)
                group.setdefault("betas", (0.9, 0.95))
                group.setdefault("eps", 1e-10)
                group.setdefault("weight_decay", 0)
        self.batch_ns = batch_ns
        self._batch_state = {}
        self._shard = shard
        super().__init__(param_groups, {})

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        seeder = _Seeder(self._random_seeds)
        name = type(self).__name__
        if self._shard:
            self._shard.bind(self)
        offsets, total = [], 0
        for group in self.param_groups:
            offsets.append(total)
            total += len(group["params"])
        order = list(range(len(self.param_groups)))
        if self._shard and not self._random_seeds:
            # AdamW groups (embedding, head) first so their broadcasts overlap the Muon work;
            # every group's math is independent of the processing order (seeds drawn from
            # torch's generator are not: those classes keep the order).
            order.sort(key=lambda gi: bool(self.param_groups[gi]["use_muon"]))
        for gi in order:
            group = self.param_groups[gi]
            group_offset = offsets[gi]
            if group["use_muon"]:
                lr, wd = group["lr"], group["weight_decay"]
                beta, nesterov, ns_steps = group["momentum"], group["nesterov"], group["ns_steps"]
                if not group["params"]:
                    continue
                if self.batch_ns:
                    gid = id(group)
                    if gid not in self._batch_state:
                        self._batch_state[gid] = _init_stacked_bufs(group["params"], group["params"][0].device,
                                                                     self.state)
                    shape_groups, stacked_bufs, buf_indices = self._batch_state[gid]
                    _check_params(group["params"], name)
                    step = 0
                    if self._record_muon_step:
                        if not hasattr(self, "_global_step"):
                            self._global_step = _restore_global_step(
                                self.state, [g for g in self.param_groups if g["use_muon"]])
                        self._global_step += 1
                        step = self._global_step
                        for p in group["params"]:
                            self.state[p]["step"] = self._global_step
                    owner = self._shard.muon_owner(gi, shape_groups) if self._shard else None
                    muon_batch_step(shape_groups, stacked_bufs, buf_indices, beta, nesterov, ns_steps, lr, wd,
                                    step, seeder, owner, self._shard.share if self._shard else None,
                                    self._shard.segments if self._shard else None)
                else:
                    for param_idx, p in enumerate(group["params"]):
                        assert p.dtype == torch.bfloat16, "only bfloat16 is supported."
                        if p.grad is None:
                            continue
                        if p.grad.is_sparse:
                            raise RuntimeError(f"{name} does not support sparse gradients")
                        state = self.state[p]
                        if len(state) == 0:
                            if self._record_muon_step:
                                state["step"] = 0
                            state["momentum_buffer"] = torch.zeros_like(p, dtype=torch.bfloat16)
                        if self._record_muon_step:
                            state["step"] += 1
                        if self._shard and not self._shard.owns(gi, param_idx):
                            seeder.skip(state.get("step", 0), param_idx, 0)
                            seeder.skip(state.get("step", 0), param_idx, 1)
                            continue
                        muon_single_step(p, _grad_of(p), state["momentum_buffer"], beta, nesterov, ns_steps, lr, wd,
                                         state.get("step", 0), param_idx, seeder)
                    if self._shard:
                        self._shard.share(group["params"])
            else:
                lr = group["lr"]
                beta1, beta2 = group["betas"]
                eps, wd = group["eps"], group["weight_decay"]
                items = []
                for i, p in enumerate(group["params"]):
                    assert p.dtype == torch.bfloat16, "only bfloat16 is supported."
                    if p.grad is None:
                        continue
                    if p.grad.is_sparse:
                        raise RuntimeError(f"{name} does not support sparse gradients")
                    state = self.state[p]
                    if len(state) == 0:
                        state["step"] = 0
                        state["ema"] = torch.zeros_like(p, dtype=torch.bfloat16)
                        state["ema_squared"] = torch.zeros_like(p, dtype=torch.bfloat16)
                    state["step"] += 1
                    seed = seeder(state["step"], group_offset + i, 0)
                    if self._shard and not self._shard.owns(gi, i):
                        continue
                    items.append((p, _grad_of(p), state["ema"], state["ema_squared"], state["step"], seed))
                K.adamw_sr(items, lr, beta1, beta2, eps, wd)
                if self._shard:
                    self._shard.share(group["params"])
        if self._shard:
            self._shard.sync_params(self)
        return loss


class MuonSRWithAuxAdam(TritonMuonSRWithAuxAdam):
    r"""``muon_sr.MuonSRWithAuxAdam`` (muon_sr/muon_sr.py:305-418) on the CUDA engine: same
    arguments and state keys; SR noise seeded from torch's default generator."""

    _random_seeds = True
    _record_muon_step = False
