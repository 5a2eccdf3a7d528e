"""AdamW with stochastic rounding and SR gradient accumulation on the B200 engine.

Drop-ins for ``muon_sr.TritonAdamW``, ``muon_sr.TritonSRAccumulator``
(muon_sr/triton_adamw.py:117-280) and ``muon_sr.SRAccumulator`` (muon_sr/muon_sr.py:28-80).
"""
import random

import torch
from torch.optim import Optimizer

from . import kernels as K
from . import staging
from .seeds import deterministic_seed


def adamw_group_step(state, group, offset, seed_of, owns=None, centralization=0.0):
    """The AdamW-SR update of one param group (``_adamw_kernel`` launches,
    triton_adamw.py:9-114, and the hybrid's AdamW groups, triton_muon_sr.py:356-371).

    Per parameter with a gradient: state ``step``/``ema``/``ema_squared`` (created at zero),
    the step advanced, the seed ``seed_of(step, offset + i)`` with ``offset`` the number of
    parameters in earlier groups; then the whole group in one multi-tensor launch. ``owns(i)``
    restricts the kernel work to this rank's parameters (state and seeds still advance, so
    every rank stays in step). ``centralization`` != 0 first centres each gradient with the
    fused kernel (triton_adamw.py:179-187). While a ``staging.HostStaging`` step runs, the
    launch is cut into batches of whole parameters so that uploads overlap updates."""
    beta1, beta2 = group["betas"]
    todo = []
    for i, p in enumerate(group["params"]):
        assert p.dtype == torch.bfloat16, "only bfloat16 is supported."
        if p.grad is None:
            continue
        if p.grad.is_sparse:
            raise RuntimeError("TritonAdamW does not support sparse gradients")
        st = state[p]
        if not st:
            st.update(step=0, ema=torch.zeros_like(p, dtype=torch.bfloat16),
                      ema_squared=torch.zeros_like(p, dtype=torch.bfloat16))
        st["step"] += 1
        seed = seed_of(st["step"], offset + i)
        if owns is not None and not owns(i):
            continue
        if p.grad.dtype != torch.bfloat16:
            raise ValueError("gradients must be bfloat16")
        todo.append((p, st, seed))
    for part in staging.batches(todo, lambda e: e[0].numel()):
        staging.need([p for p, _, _ in part])
        batch = []
        for p, st, seed in part:
            grad = K.centralize(p.grad, centralization) if centralization else p.grad.contiguous()
            batch.append((p, grad, st["ema"], st["ema_squared"], st["step"], seed))
        K.adamw_sr(batch, group["lr"], beta1, beta2, group["eps"], group["weight_decay"])
        staging.done([p for p, _, _ in part])


class TritonAdamW(Optimizer):
    r"""AdamW with stochastic rounding as one fused multi-tensor kernel per param group.

    Arguments:
        params: parameters to optimize
        lr (float): learning rate (default: 1e-3)
        betas (Tuple[float, float]): EMA coefficients (default: (0.9, 0.999))
        eps (float): denominator epsilon (default: 1e-8)
        weight_decay (float): decoupled weight decay (default: 0)
        centralization (float): gradient centralization strength (default: 0)
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0, centralization=0):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, centralization=centralization)
        super().__init__(params, defaults)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        offset = 0
        for group in self.param_groups:
            adamw_group_step(self.state, group, offset, deterministic_seed,
                             centralization=group["centralization"])
            offset += len(group["params"])
        return loss


class TritonSRAccumulator:
    """Gradient accumulation into bf16 ``p.acc_grad`` buffers with stochastic rounding.

    Usage is identical to the reference (muon_sr/triton_adamw.py:232-280)::

        TritonSRAccumulator.assign_hooks(model)
        for step in range(total_steps):
            for _ in range(grad_accum):
                loss = model(x); loss.backward()
            TritonSRAccumulator.reassign_grad_buffer(model)
            optimizer.step(); optimizer.zero_grad()

    Each hook call is one kernel launch with a seed from Python's ``random`` module. The
    first micro-batch writes the buffer without reading it (no zero fill).
    """

    @staticmethod
    def _accum_hook(p):
        seed = random.getrandbits(32)
        grad = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
        if hasattr(p, "acc_grad"):
            K.grad_accum_(p.acc_grad, grad, seed)
        else:
            p.acc_grad = torch.empty_like(p.data, dtype=torch.bfloat16, memory_format=torch.contiguous_format)
            K.grad_accum_(p.acc_grad, grad, seed, first=True)
        del p.grad

    @staticmethod
    def reassign_grad_buffer(model):
        for _, p in model.named_parameters():
            if p.requires_grad and hasattr(p, "acc_grad"):
                p.grad = p.acc_grad
                del p.acc_grad

    @staticmethod
    def assign_hooks(model):
        hooks = []
        for _, p in model.named_parameters():
            if p.requires_grad:
                hooks.append(p.register_post_accumulate_grad_hook(TritonSRAccumulator._accum_hook))
        return hooks


class SRAccumulator:
    """``muon_sr.SRAccumulator`` (muon_sr/muon_sr.py:28-80) on the CUDA engine: the first
    micro-batch clones the gradient into ``p.acc_grad``; later ones add with SR, seeded from
    torch's default generator (the reference draws its noise with ``torch.randint_like``)."""

    @staticmethod
    def stochastic_grad_accum(p):
        if hasattr(p, "acc_grad"):
            seed = int(torch.randint(0, 1 << 32, (1,), dtype=torch.int64).item())
            grad = p.grad.to(torch.bfloat16)
            K.grad_accum_(p.acc_grad, grad if grad.is_contiguous() else grad.contiguous(), seed)
            del p.grad
        else:
            p.acc_grad = p.grad.clone().to(torch.bfloat16)
            del p.grad

    @staticmethod
    def reassign_grad_buffer(model):
        for n, p in model.named_parameters():
            if p.requires_grad:
                p.grad = p.acc_grad
                del p.acc_grad

    @staticmethod
    def assign_hooks(model):
        hooks = []
        for n, p in model.named_parameters():
            if p.requires_grad:
                hooks.append(p.register_post_accumulate_grad_hook(SRAccumulator.stochastic_grad_accum))
        return hooks
