"""The reference's fused elementwise kernels, restated in numpy fp32.

Every kernel below evaluates the same fp32 operations in the same order as the Triton
source it cites, with no fused multiply-add (the Triton interpreter evaluates the kernels
this way, which is how the golden vectors were produced). Inputs and outputs are bf16 bit
patterns (uint16 arrays).

Scalars: the interpreter keeps Python-float kernel arguments as Python floats, so a
subexpression made only of scalars (``1.0 - beta``, ``1.0 - lr * weight_decay``,
``lr / bias_correction``) is evaluated in double and rounded to fp32 once, where it meets
a tensor. ``host_coefficients``-style helpers below do exactly that; the CUDA engine's
host code computes the same coefficients the same way. (Compiled Triton would evaluate
them in fp32 and can differ from this by one fp32 ulp in a coefficient.)
"""
import numpy as np

from .philox import sr_noise, triton_key
from .sr import bf16_to_f32, rne_bf16, sr_bf16

f32 = np.float32


def counters(n: int, ctr_base: int = 0) -> np.ndarray:
    """Per-element Philox counters: the element offset truncated to 32 bits
    (``triton_muon_sr.py:44`` ``offsets.to(tl.int32)``; int32 offsets elsewhere)."""
    return (np.arange(n, dtype=np.uint64) + np.uint64(ctr_base)) & np.uint64(0xFFFFFFFF)


def sr_round(x, key64: int, ctr_base: int = 0, noise: str = "reference"):
    """The rounding of an SR store: stochastic with the noise stream ``noise`` ("reference":
    the reference's Philox words, "fast": the engine's opt-in stream) at counters
    ctr_base, ctr_base + 1, ..., or, for ``noise="none"`` (the engine's parity mode without
    noise), round to nearest even like a plain fp32 -> bf16 cast."""
    x = np.asarray(x, dtype=f32)
    if noise == "none":
        return rne_bf16(x)
    return sr_bf16(x, sr_noise(key64, x.size, ctr_base, noise))


def grad_accum(acc_bits, grad_bits, seed: int, noise: str = "reference"):
    """``_grad_accum_kernel`` -- ``muon_sr/triton_adamw.py:206-229``: acc <- SR(acc + g).
    ``noise`` selects the rounding (``sr_round``)."""
    acc = bf16_to_f32(acc_bits)
    g = bf16_to_f32(grad_bits)
    s = (acc + g).astype(f32)
    return sr_round(s, triton_key(seed), 0, noise)


def muon_prepare(g_bits, buf_bits, beta: float, nesterov: bool, seed: int, ctr_base: int = 0,
                 return_f32: bool = False, noise: str = "reference"):
    """``_muon_prepare_kernel`` -- ``muon_sr/triton_muon_sr.py:18-50``.

    new_buf = buf + (1 - beta) * (g - buf); update = g + beta * (new_buf - g) (Nesterov) or
    new_buf. Returns (SR(new_buf) bits, RNE(update) bits) and, with ``return_f32``, the
    fp32 update as well. ``ctr_base`` is the offset of element 0 within the launch (the
    whole stacked group in the batched path, ``triton_muon_sr.py:156-159``).

    The update store (``:50``) is a plain ``.to(bfloat16)``: round-to-nearest-even in
    compiled Triton and torch, which is what this returns. The Triton interpreter that
    produced the golden vectors truncates in that cast instead, so the golden ``update``
    bits equal ``truncate_bf16`` of the fp32 update returned here.
    """
    g = bf16_to_f32(g_bits)
    buf = bf16_to_f32(buf_bits)
    one_minus_beta = f32(1.0 - beta)
    new_buf = (buf + one_minus_beta * (g - buf)).astype(f32)
    if nesterov:
        update = (g + f32(beta) * (new_buf - g)).astype(f32)
    else:
        update = new_buf
    buf_bits = sr_round(new_buf, triton_key(seed), ctr_base, noise)
    if return_f32:
        return buf_bits, rne_bf16(update), update
    return buf_bits, rne_bf16(update)


def ns_scale(rows: int, cols: int) -> float:
    """``_ns_scale`` -- ``muon_sr/triton_muon_sr.py:101-102`` (computed in double, passed
    to the kernel as fp32)."""
    return max(1.0, rows / cols) ** 0.5


def muon_apply(p_bits, upd_bits, lr: float, weight_decay: float, scale: float, seed: int, noise: str = "reference"):
    """``_muon_apply_kernel`` -- ``muon_sr/triton_muon_sr.py:53-80``:
    p <- SR(p * (1 - lr * wd) - lr * (update * scale))."""
    p = bf16_to_f32(p_bits)
    upd = (bf16_to_f32(upd_bits) * f32(scale)).astype(f32)
    decay = f32(1.0 - lr * weight_decay)
    p = (p * decay).astype(f32)
    p = (p - f32(lr) * upd).astype(f32)
    return sr_round(p, triton_key(seed), 0, noise)


def adamw_coefficients(lr, beta1, beta2, eps, weight_decay, step):
    """Host side of ``_adamw_step`` (``muon_sr/triton_adamw.py:88-89``) plus the scalar-only
    subexpressions of ``_adamw_kernel`` (:37-45), each in double and rounded to fp32 once:
    (beta1, 1-beta1, beta2, 1-beta2, lr/bc1, bc2_sqrt, eps, 1-lr*wd)."""
    bc1 = 1.0 - beta1 ** step
    bc2s = (1.0 - beta2 ** step) ** 0.5
    return (f32(beta1), f32(1.0 - beta1), f32(beta2), f32(1.0 - beta2), f32(lr / bc1),
            f32(bc2s), f32(eps), f32(1.0 - lr * weight_decay))


def adamw_sr(p_bits, g_bits, m_bits, v_bits, lr, beta1, beta2, eps, weight_decay, step, seed, noise="reference"):
    """``_adamw_kernel`` -- ``muon_sr/triton_adamw.py:9-72``.

    Decay before the update; SR on ema (seed), ema_sq (seed + 1), p (seed + 2).
    Returns (p, ema, ema_sq) bf16 bits.
    """
    b1, omb1, b2, omb2, step_size, bc2s, eps, decay = adamw_coefficients(
        lr, beta1, beta2, eps, weight_decay, step)
    p = bf16_to_f32(p_bits)
    g = bf16_to_f32(g_bits)
    m = bf16_to_f32(m_bits)
    v = bf16_to_f32(v_bits)
    m = (b1 * m + omb1 * g).astype(f32)
    v = (b2 * v + omb2 * g * g).astype(f32)
    denom = (np.sqrt(v) / bc2s + eps).astype(f32)
    p = (p * decay).astype(f32)
    p = (p - step_size * m / denom).astype(f32)
    return (sr_round(p, triton_key(seed, 2), 0, noise), sr_round(m, triton_key(seed, 0), 0, noise),
            sr_round(v, triton_key(seed, 1), 0, noise))
