"""The reference's pure-PyTorch ``MuonSR`` / AdamW-SR step on CPU tensors.

This is the timed CPU baseline (``bench.py``'s ``cpu_baseline`` leg and its
``--impl reference`` arm). It restates, with the same torch ops in the same order:

* ``copy_stochastic_`` -- ``muon_sr/muon_sr.py:5-24`` (torch RNG noise, int32 add, mask);
* ``_muon_step_fp32`` -- ``muon_sr/muon_sr.py:101-109`` with the per-parameter loop of
  ``MuonSR.step`` (``batch_ns=False``) -- ``muon_sr/muon_sr.py:286-300``;
* the AdamW branch of ``MuonSRWithAuxAdam.step`` -- ``muon_sr/muon_sr.py:383-416``.
"""
import torch

from .newton_schulz import newton_schulz


def copy_stochastic_(target: torch.Tensor, source: torch.Tensor) -> None:
    with torch.no_grad():
        result = torch.randint_like(source, dtype=torch.int32, low=0, high=(1 << 16))
        result.add_(source.view(dtype=torch.int32))
        result.bitwise_and_(-65536)
        target.copy_(result.view(dtype=torch.float32))


def muon_step_fp32(grad, buf, p_fp32, beta, nesterov, ns_steps, lr, weight_decay):
    buf.lerp_(grad, 1 - beta)
    update = grad.lerp_(buf, beta) if nesterov else buf.clone()
    update = newton_schulz(update, steps=ns_steps, out_dtype=torch.float32)
    update *= max(1, update.size(-2) / update.size(-1)) ** 0.5
    if weight_decay != 0:
        p_fp32.mul_(1 - lr * weight_decay)
    p_fp32.add_(update, alpha=-lr)


@torch.no_grad()
def muon_sr_step(params, grads, bufs, lr=0.02, weight_decay=0.0, momentum=0.95,
                 nesterov=True, ns_steps=5):
    """One ``MuonSR.step()`` (batch_ns=False) over bf16 CPU tensors, updating in place."""
    for p, g, b in zip(params, grads, bufs):
        grad = g.to(torch.float32)
        p_fp32 = p.clone().to(torch.float32)
        buf = b.to(torch.float32)
        muon_step_fp32(grad, buf, p_fp32, momentum, nesterov, ns_steps, lr, weight_decay)
        copy_stochastic_(b, buf)
        copy_stochastic_(p, p_fp32)


@torch.no_grad()
def adamw_sr_step(params, grads, emas, ema_sqs, step, lr=3e-4, betas=(0.9, 0.95),
                  eps=1e-10, weight_decay=0.0):
    """The AdamW branch of ``MuonSRWithAuxAdam.step`` for one step number ``step``."""
    beta1, beta2 = betas
    for p, g, e, es in zip(params, grads, emas, ema_sqs):
        grad = g.to(torch.float32)
        p_fp32 = p.clone().to(torch.float32)
        ema = e.to(torch.float32)
        ema_sq = es.to(torch.float32)
        bias_correction = 1 - beta1 ** step
        bias_correction_sqrt = (1 - beta2 ** step) ** 0.5
        step_size = lr / bias_correction
        ema.mul_(beta1).add_(grad, alpha=1 - beta1)
        ema_sq.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)
        denom = (ema_sq.sqrt() / bias_correction_sqrt).add_(eps)
        if weight_decay != 0:
            p_fp32.mul_(1 - lr * weight_decay)
        p_fp32.addcdiv_(ema, denom, value=-step_size)
        copy_stochastic_(e, ema)
        copy_stochastic_(es, ema_sq)
        copy_stochastic_(p, p_fp32)
