"""Tensor-level wrappers of the C ABI: each function validates torch tensors, fills the
C entry tables and enqueues the CUDA kernels on the current stream. No host syncs.

Scalars that the reference evaluates from Python floats (``1 - beta``, ``1 - lr * wd``,
``lr / bias_correction`` ...) are computed here in double and rounded to fp32 once, as the
reference's kernels see them.
"""
import contextlib
import ctypes
import math
import threading

import numpy as np
import torch

from . import _lib
from .seeds import triton_key

f32 = np.float32


def stream_handle(device=None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require(t: torch.Tensor, name: str, dtype=torch.bfloat16):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (muon_sr_b200 has no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


# ``recorder(rec)`` is entered by ``graph.StepGraph`` while it sizes, captures or refreshes a
# step on this thread: the multi-tensor launches below then go through ``rec`` (replayable
# launches whose scalars live in a device record), and in its passes that issue no kernels
# (``rec.launches`` False) the Newton-Schulz and centralisation calls return without launching.
_tls = threading.local()


@contextlib.contextmanager
def recorder(rec):
    _tls.rec = rec
    try:
        yield rec
    finally:
        _tls.rec = None


def _recorder():
    return getattr(_tls, "rec", None)


def _issuing():
    rec = _recorder()
    return rec is None or rec.launches


# Multicast addresses of the parameters this process updates, registered by a
# ``sharding.Sharder`` whose weights live in a symmetric allocation bound to an NVLink
# multicast object: data_ptr -> multicast address. The weight-updating launches (apply, AdamW,
# 8-bit AdamW) pass it as the entry's ``param_mc``, so the updated weight is stored once and
# reaches every rank's replica.
_multicast = {}


def register_multicast(mapping) -> None:
    """Add multicast parameter addresses (``{data_ptr: address}``) to the registry."""
    _multicast.update(mapping)


def unregister_multicast(data_ptrs) -> None:
    for ptr in data_ptrs:
        _multicast.pop(ptr, None)


def _mc(t):
    return _multicast.get(t.data_ptr()) if _multicast else None


# ---------------------------------------------------------------------------------------
def philox_fill(n: int, ctr_base: int, key: int, device) -> torch.Tensor:
    """Test hook: Philox words for counters ctr_base .. ctr_base + n - 1 (as int32)."""
    out = torch.empty(n, dtype=torch.int32, device=device)
    _lib.check(_lib.load().msr_philox_fill(out.data_ptr(), n, ctr_base, key, stream_handle(device)),
               "msr_philox_fill")
    return out


def grad_accum_(acc: torch.Tensor, grad: torch.Tensor, seed: int, first: bool = False) -> None:
    """acc <- SR(acc + grad) with the seed of one accumulator hook call; with ``first`` the
    accumulator's old contents are ignored (treated as zero) and only written."""
    _require(acc, "acc")
    _require(grad, "grad")
    if acc.numel() != grad.numel():
        raise ValueError("acc and grad sizes differ")
    _lib.check(_lib.load().msr_grad_accum_bf16(acc.data_ptr(), grad.data_ptr(), acc.numel(), triton_key(seed),
                                               int(bool(first)), stream_handle(acc.device)), "msr_grad_accum_bf16")


def muon_prepare(items, beta: float, nesterov: bool) -> None:
    """items: iterable of (grad, momentum, update, ctr_base, seed)."""
    items = list(items)
    if not items:
        return
    arr = (_lib.PrepareEntry * len(items))()
    for e, (g, buf, upd, ctr_base, seed) in zip(arr, items):
        e.grad = g.data_ptr()
        e.momentum = buf.data_ptr()
        e.update = upd.data_ptr()
        e.numel = g.numel()
        e.ctr_base = ctr_base & 0xFFFFFFFFFFFFFFFF
        e.key = triton_key(seed)
    dev = items[0][0].device
    rec = _recorder()
    if rec is not None:
        hdr = _lib.PrepareRecord(float(f32(beta)), float(f32(1.0 - beta)), int(bool(nesterov)), len(items))
        rec.launch("msr_muon_prepare_rec", hdr, arr, dev)
        return
    _lib.check(_lib.load().msr_muon_prepare(arr, len(items), float(f32(beta)), float(f32(1.0 - beta)),
                                            int(bool(nesterov)), stream_handle(dev)), "msr_muon_prepare")


def muon_apply(items, lr: float, weight_decay: float) -> None:
    """items: iterable of (param, update, scale, seed)."""
    items = list(items)
    if not items:
        return
    arr = (_lib.ApplyEntry * len(items))()
    for e, (p, upd, scale, seed) in zip(arr, items):
        e.param = p.data_ptr()
        e.update = upd.data_ptr()
        e.numel = p.numel()
        e.key = triton_key(seed)
        e.scale = float(f32(scale))
        e.param_mc = _mc(p)
    dev = items[0][0].device
    rec = _recorder()
    if rec is not None:
        hdr = _lib.ApplyRecord(float(f32(lr)), float(f32(1.0 - lr * weight_decay)), len(items), 0)
        rec.launch("msr_muon_apply_rec", hdr, arr, dev)
        return
    _lib.check(_lib.load().msr_muon_apply(arr, len(items), float(f32(lr)), float(f32(1.0 - lr * weight_decay)),
                                          stream_handle(dev)), "msr_muon_apply")


def adamw_sr(items, lr: float, beta1: float, beta2: float, eps: float, weight_decay: float) -> None:
    """items: iterable of (param, grad, exp_avg, exp_avg_sq, step, seed)."""
    items = list(items)
    if not items:
        return
    arr = (_lib.AdamWEntry * len(items))()
    for e, (p, g, m, v, step, seed) in zip(arr, items):
        e.param, e.grad, e.exp_avg, e.exp_avg_sq = p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr()
        e.numel = p.numel()
        e.key_m, e.key_v, e.key_p = triton_key(seed, 0), triton_key(seed, 1), triton_key(seed, 2)
        bc1 = 1.0 - beta1 ** step
        bc2s = (1.0 - beta2 ** step) ** 0.5
        e.step_size = float(f32(lr / bc1))
        e.bc2_sqrt = float(f32(bc2s))
        e.param_mc = _mc(p)
    hp = _lib.AdamWHparams(float(f32(beta1)), float(f32(1.0 - beta1)), float(f32(beta2)), float(f32(1.0 - beta2)),
                           float(f32(eps)), float(f32(1.0 - lr * weight_decay)))
    dev = items[0][0].device
    rec = _recorder()
    if rec is not None:
        rec.launch("msr_adamw_sr_rec", _lib.AdamWRecord(hp, len(items), 0), arr, dev)
        return
    _lib.check(_lib.load().msr_adamw_sr(arr, len(items), ctypes.byref(hp), stream_handle(dev)), "msr_adamw_sr")


_qtable_cache = {}


def quant_tables(qmap1: torch.Tensor, qmap2: torch.Tensor):
    """Device copy of the quantiser lookup tables for this codebook pair (built once per
    device and codebook contents), or None if the table rule is not exact for them."""
    from . import quant_tables as qt
    q1 = qmap1.detach().float().cpu().numpy()
    q2 = qmap2.detach().float().cpu().numpy()
    key = (qmap1.device.index, q1.tobytes(), q2.tobytes())
    if key not in _qtable_cache:
        b = qt.blob(q1, q2)
        _qtable_cache[key] = None if b is None else torch.from_numpy(b).to(qmap1.device)
    return _qtable_cache[key]


def adamw8bit(items, qmap1, qmap2, lr, beta1, beta2, eps, weight_decay, block_size, qtables=None) -> None:
    """items: iterable of (param, grad, state1, state2, absmax1, absmax2, step, seed, quantized).
    ``qtables``: the lookup-table blob of ``quant_tables`` (None runs the codebook walk)."""
    if _recorder() is not None:
        raise RuntimeError("8-bit AdamW launches cannot be captured in a StepGraph")
    items = list(items)
    if not items:
        return
    arr = (_lib.Adam8Entry * len(items))()
    lr32, eps32 = f32(lr), f32(eps)
    for e, (p, g, s1, s2, a1, a2, step, seed, quant) in zip(arr, items):
        e.param, e.grad, e.state1, e.state2 = p.data_ptr(), g.data_ptr(), s1.data_ptr(), s2.data_ptr()
        e.absmax1 = a1.data_ptr() if quant else None
        e.absmax2 = a2.data_ptr() if quant else None
        e.numel = p.numel()
        e.key_p, e.key_m, e.key_v = triton_key(seed, 0), triton_key(seed, 1), triton_key(seed, 2)
        bc1 = f32(1.0 - beta1 ** step)
        sq_bc2 = np.sqrt(f32(1.0 - beta2 ** step))
        e.coef = float(f32(f32(lr32 * sq_bc2) / bc1))
        e.sqrt_bc2_eps = float(f32(sq_bc2 * eps32))
        e.quantized = 1 if quant else 0
        e.param_mc = _mc(p)
    hp = _lib.Adam8Hparams(float(f32(beta1)), float(f32(1.0 - beta1)), float(f32(beta2)), float(f32(1.0 - beta2)),
                           float(f32(1.0 - lr * weight_decay)), int(block_size),
                           qtables.data_ptr() if qtables is not None else None)
    dev = items[0][0].device
    _lib.check(_lib.load().msr_adamw8bit(arr, len(items), _ptr(qmap1), _ptr(qmap2), ctypes.byref(hp),
                                         stream_handle(dev)), "msr_adamw8bit")


# ---------------------------------------------------------------------------------------
# Newton-Schulz
# ---------------------------------------------------------------------------------------
_workspaces = {}


def _workspace(device, nbytes: int) -> torch.Tensor:
    """Scratch buffer for the Newton-Schulz chain, one per (device, stream) and grown on
    demand: calls on one stream reuse it in stream order, calls on different streams never
    share it. A buffer used while a ``StepGraph`` captures is also held by that graph's
    recorder (``hold``), so growing the buffer later for an eager call never returns memory
    a captured graph still writes to."""
    device = torch.device(device)
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        _workspaces[key] = ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    rec = _recorder()
    if rec is not None and rec.launches:
        rec.hold(ws)
    return ws


def ns_workspace_bytes(batch: int, rows: int, cols: int) -> int:
    return int(_lib.load().msr_ns_workspace_bytes(batch, rows, cols))


NS_REFERENCE_ROUNDING = 0
NS_FUSED_ROUNDING = 1


def newton_schulz(x: torch.Tensor, steps: int = 5, norm_sq: torch.Tensor = None,
                  out: torch.Tensor = None, mode: int = NS_REFERENCE_ROUNDING) -> torch.Tensor:
    """bf16 Newton-Schulz over the last two dims of ``x`` (leading dims are a batch), as
    ``_newton_schulz(x, steps, out_dtype=None)`` of the reference (muon_sr.py:82-98).
    ``mode`` selects the reference's op-by-op bf16 rounding (default) or one rounding per
    GEMM (closer to exact arithmetic)."""
    _require(x, "x")
    if x.ndim < 2:
        raise ValueError("Newton-Schulz needs a tensor with ndim >= 2")
    rows, cols = x.shape[-2], x.shape[-1]
    batch = x.numel() // max(1, rows * cols)
    if not _issuing():
        return x if out is None else out  # a refresh pass: the captured graph computes it
    if out is None:
        out = torch.empty_like(x)
    if batch == 0:
        return out
    nbytes = ns_workspace_bytes(batch, rows, cols)
    ws = _workspace(x.device, nbytes)
    if norm_sq is not None:
        _require(norm_sq, "norm_sq", torch.float32)
    _lib.check(_lib.load().msr_newton_schulz_bf16(
        x.data_ptr(), out.data_ptr(), batch, rows, cols, int(steps), int(mode),
        norm_sq.data_ptr() if norm_sq is not None else None, ws.data_ptr(), ws.numel(),
        stream_handle(x.device)), "msr_newton_schulz_bf16")
    return out


def gemm_bf16(a, a_mn_major, b, b_mn_major, c=None, alpha=1.0, beta=0.0, scale=None, alpha_pow=0, beta_pow=0,
              ref_rounding=False, symmetric=False):
    """Test hook: batched tcgen05 GEMM with the Newton-Schulz epilogue (see the header)."""
    for t, n in ((a, "a"), (b, "b")):
        _require(t, n)
    batch = a.shape[0]
    if a_mn_major:
        K, M = a.shape[1], a.shape[2]
    else:
        M, K = a.shape[1], a.shape[2]
    N = b.shape[2] if b_mn_major else b.shape[1]
    d = torch.empty(batch, M, N, dtype=torch.bfloat16, device=a.device)
    _lib.check(_lib.load().msr_gemm_bf16(
        a.data_ptr(), int(a_mn_major), b.data_ptr(), int(b_mn_major), c.data_ptr() if c is not None else None,
        d.data_ptr(), batch, M, N, K, float(alpha), float(beta), scale.data_ptr() if scale is not None else None,
        int(alpha_pow), int(beta_pow), (1 if ref_rounding else 0) | (2 if symmetric else 0),
        stream_handle(a.device)), "msr_gemm_bf16")
    return d


def centralize(grad: torch.Tensor, centralization: float) -> torch.Tensor:
    """``bf16(g - c * g.mean(dim=trailing dims, keepdim=True))`` with the mean in fp32, as
    TritonAdamW's centralization (muon_sr/triton_adamw.py:179-187), in one fused kernel;
    returns a new bf16 tensor."""
    rec = _recorder()
    if rec is not None:
        rec.constant("centralization", float(centralization))
        if not rec.launches:
            return grad
    g = grad if grad.is_contiguous() else grad.contiguous()
    _require(g, "grad")
    out = torch.empty_like(g, memory_format=torch.contiguous_format)
    if g.numel() == 0:
        return out
    rows = g.shape[0] if g.dim() > 1 else 1
    _lib.check(_lib.load().msr_centralize_bf16(g.data_ptr(), out.data_ptr(), rows, g.numel() // rows,
                                               float(centralization), stream_handle(g.device)),
               "msr_centralize_bf16")
    return out


SR_NOISE_MODES = {"reference": 0, "fast": 1, "none": 2}


def set_sr_noise(mode: str = "reference") -> None:
    """Noise stream of every stochastic rounding (process-wide). ``"reference"`` (default):
    the reference's Philox stream, bit-identical results. ``"fast"``: one Philox4x32-10 call
    per 8 consecutive values (16 bits each) -- unbiased stochastic rounding at a fraction of
    the integer work, with different bits than the reference. ``"none"``: no stochastic
    rounding, every SR store rounds to nearest even (a parity mode for checking the updates'
    fp32 arithmetic, not for training). See ``msr_set_sr_noise``."""
    if mode not in SR_NOISE_MODES:
        raise ValueError(f"sr noise mode must be one of {sorted(SR_NOISE_MODES)}, got {mode!r}")
    _lib.check(_lib.load().msr_set_sr_noise(SR_NOISE_MODES[mode]), "msr_set_sr_noise")


def set_gemm_pairs(enable: bool) -> None:
    """Run the Newton-Schulz GEMMs on SM pairs (256 x 256 tiles, the default) or on single
    SMs (128 x 256 tiles). Both produce the same bits; process-wide."""
    _lib.load().msr_set_gemm_pairs(1 if enable else 0)


def device_error(clear: bool = True, device=None) -> int:
    """Synchronise the current stream and return (and clear) the library's device error code."""
    return int(_lib.load().msr_device_error(stream_handle(device), int(clear)))


def ns_scale(shape) -> float:
    """``_ns_scale`` -- muon_sr/triton_muon_sr.py:101-102."""
    return max(1.0, shape[-2] / shape[-1]) ** 0.5


def numel_of(shape) -> int:
    return int(math.prod(shape))
