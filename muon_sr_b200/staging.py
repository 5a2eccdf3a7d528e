"""Optimizer steps fed from host memory, with the copies overlapped with the step.

``HostStaging`` runs an optimizer step whose gradients come from pinned host buffers and
whose updated weights go back to pinned host buffers (a host-resident or offloaded training
loop). The optimizers of this package announce, while they issue a step, which parameters'
gradients the next launch reads (``need``) and which parameters the last launch finished
updating (``done``); they do so at the granularity of their launches: a Newton-Schulz chunk
of a batched Muon stack, one Muon matrix, an AdamW or 8-bit AdamW launch batch. HostStaging
turns the announcements into stream dependencies:

* ``need(params)`` -- the gradients of ``params`` not yet uploaded in this step are copied
  host -> device on an upload stream, and the step's stream waits for that copy only;
* ``done(params)`` -- a download stream waits for the step's stream at that point and copies
  ``params`` device -> host.

The host issues a whole step long before the GPU finishes it, so the uploads queue up in the
order the step consumes them and run on the host-to-device copy engine while earlier chunks
compute; the downloads run on the device-to-host engine behind them. A step ends with the
caller's stream waiting for both copy streams, and the next step's uploads start only after
that (its gradients may depend on the weights just downloaded), so steps never overlap each
other. The bits are those of ``upload; optimizer.step(); download``.

Without an active ``HostStaging`` the hooks do nothing.
"""
import threading

import torch

_tls = threading.local()

# Launch batches of the AdamW and 8-bit AdamW steps hold at most this many elements while a
# HostStaging step runs, so that the upload of one batch overlaps the update of the previous
# one (a parameter is never split).
BATCH_NUMEL = 1 << 28


def active():
    """Whether a HostStaging step is being issued on this thread."""
    return getattr(_tls, "io", None) is not None


def need(params):
    """Announce that the next launch reads the gradients of ``params``."""
    io = getattr(_tls, "io", None)
    if io is not None:
        io.need(params)


def done(params):
    """Announce that the launches issued so far finished updating ``params``."""
    io = getattr(_tls, "io", None)
    if io is not None:
        io.done(params)


def batches(items, numel_of):
    """``items`` cut into consecutive batches of at most BATCH_NUMEL elements (one item may
    exceed it alone) while a HostStaging step runs; otherwise one batch."""
    if getattr(_tls, "io", None) is None or not items:
        return [items] if items else []
    out, cur, size = [], [], 0
    for it in items:
        n = numel_of(it)
        if cur and size + n > BATCH_NUMEL:
            out.append(cur)
            cur, size = [], 0
        cur.append(it)
        size += n
    out.append(cur)
    return out


def _pinned_like(t, name):
    if t.device.type != "cpu" or not t.is_pinned():
        raise ValueError(f"{name} must be pinned host tensors")
    if t.dtype != torch.bfloat16 or not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous bfloat16 tensors")


class HostStaging:
    """Run ``optimizer.step()`` with gradients from ``host_grads`` and updated weights into
    ``host_params``, the copies overlapped with the step.

    Arguments:
        optimizer: an optimizer of this package over ``params`` (CUDA bf16 parameters)
        params: the parameters, in the order of the host buffers
        host_grads: one pinned bf16 host tensor per parameter (its shape), or None for a
            parameter without a gradient; the device gradients ``p.grad`` are allocated
            once and filled from these at every step
        host_params: optional pinned bf16 host tensors receiving every parameter the step
            updates on this device (with a ``Sharder``: the parameters this rank owns)

    ``step()`` returns after issuing the work, like ``optimizer.step()``; call
    ``synchronize()`` (or synchronize the device) before reading ``host_params`` or refilling
    ``host_grads``. ``h2d_bytes`` / ``d2h_bytes`` count the bytes copied by the last step.
    """

    def __init__(self, optimizer, params, host_grads, host_params=None):
        from .adamw import TritonAdamW
        from .adamw8bit import TritonAdamW8bit
        from .muon import _MuonBase
        if not isinstance(optimizer, (_MuonBase, TritonAdamW, TritonAdamW8bit)):
            raise TypeError("HostStaging needs an optimizer of muon_sr_b200 (they announce their launches)")
        params = list(params)
        host_grads = list(host_grads)
        if len(host_grads) != len(params):
            raise ValueError("host_grads must hold one entry per parameter")
        if host_params is not None:
            host_params = list(host_params)
            if len(host_params) != len(params):
                raise ValueError("host_params must hold one entry per parameter")
        if not params:
            raise ValueError("no parameters")
        device = params[0].device
        for i, p in enumerate(params):
            if not p.is_cuda or p.device != device or p.dtype != torch.bfloat16 or not p.is_contiguous():
                raise ValueError("parameters must be contiguous bfloat16 tensors on one CUDA device")
            for name, bufs in (("host_grads", host_grads), ("host_params", host_params)):
                h = None if bufs is None else bufs[i]
                if h is None:
                    continue
                _pinned_like(h, name)
                if h.shape != p.shape:
                    raise ValueError(f"{name}[{i}] has shape {tuple(h.shape)}, parameter {tuple(p.shape)}")
        self.optimizer = optimizer
        self._params = params
        self._index = {id(p): i for i, p in enumerate(params)}
        self._host_g = host_grads
        self._host_p = host_params
        self._device = device
        self._up = torch.cuda.Stream(device=device)
        self._down = torch.cuda.Stream(device=device)
        for p, h in zip(params, host_grads):
            if h is None:
                p.grad = None
            elif p.grad is None or p.grad.shape != p.shape or p.grad.dtype != torch.bfloat16 \
                    or not p.grad.is_contiguous():
                p.grad = torch.empty_like(p, memory_format=torch.contiguous_format)
        self._uploaded = {}
        self._downloaded = set()
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    # ---- hooks (called by the optimizers through need/done) ----
    def need(self, params):
        idx = [self._index[id(p)] for p in params if id(p) in self._index]
        idx = [i for i in idx if self._host_g[i] is not None]
        missing = [i for i in dict.fromkeys(idx) if i not in self._uploaded]
        if missing:
            with torch.cuda.stream(self._up):
                for i in missing:
                    self._params[i].grad.copy_(self._host_g[i], non_blocking=True)
                    self.h2d_bytes += self._host_g[i].numel() * 2
            ev = torch.cuda.Event()
            ev.record(self._up)
            for i in missing:
                self._uploaded[i] = ev
        cur = torch.cuda.current_stream(self._device)
        for ev in {id(self._uploaded[i]): self._uploaded[i] for i in idx}.values():
            cur.wait_event(ev)

    def done(self, params):
        if self._host_p is None:
            return
        idx = [self._index[id(p)] for p in params if id(p) in self._index]
        idx = [i for i in dict.fromkeys(idx) if self._host_p[i] is not None and i not in self._downloaded]
        if not idx:
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self._device))
        self._down.wait_event(ev)
        with torch.cuda.stream(self._down):
            for i in idx:
                self._host_p[i].copy_(self._params[i].detach(), non_blocking=True)
                self.d2h_bytes += self._host_p[i].numel() * 2
                self._downloaded.add(i)

    # ---- the step ----
    def step(self):
        if getattr(_tls, "io", None) is not None:
            raise RuntimeError("HostStaging steps do not nest")
        cur = torch.cuda.current_stream(self._device)
        start = torch.cuda.Event()
        start.record(cur)
        # the previous step (its update and its downloads) is complete before new gradients
        # overwrite the device buffers
        self._up.wait_event(start)
        self._down.wait_event(start)
        self._uploaded = {}
        self._downloaded = set()
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        _tls.io = self
        try:
            loss = self.optimizer.step()
        finally:
            _tls.io = None
        for s in (self._up, self._down):
            ev = torch.cuda.Event()
            ev.record(s)
            cur.wait_event(ev)
        return loss

    def synchronize(self):
        """Wait on the host until the last step, its uploads and its downloads are done."""
        for s in (self._up, self._down, torch.cuda.current_stream(self._device)):
            s.synchronize()
