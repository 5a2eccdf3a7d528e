"""Parameter-sharded optimizer work across the ranks of one node.

The reference is single-device; data-parallel replicas each run the whole optimizer step
and stay identical because the rounding seeds depend only on (step, index). Here each rank
runs the step for the parameters it owns and the updated bf16 weights are then shared over
NVLink / NVSwitch, so the step's work is divided by the number of ranks.

* Partition: whole tensors (Newton-Schulz needs each full matrix), longest-processing-time
  greedy on an estimated B200 time per tensor -- Newton-Schulz FLOPs at its measured
  effective rate for Muon matrices, bytes at the measured rate of each elementwise kernel.
* Seeds and Philox counters stay global, so every rank writes exactly the bits a single GPU
  would (Newton-Schulz computes each matrix independently of how the batch is chunked).
* Sharing: as soon as a segment of a shape stack (or a param group) is updated, its
  parameters travel from their owners (see ``transport``), so the transfers run under the
  remaining Newton-Schulz work; the step ends by waiting for all of them.
* Optimizer state (momentum, moments) stays with the owner; ``state_dict()`` on a rank holds
  valid values only for the parameters that rank owns until ``gather_state`` copies the
  owners' values over (for checkpoints).
* ``reduce_grads`` replaces the data-parallel all-reduce of the gradients: each gradient
  only has to reach its owner.
"""
import ctypes
import datetime
import heapq
import math
import os
import warnings

import torch
import torch.distributed as dist

# Rates that weigh the partition (measured on B200 inside the sharded step): Newton-Schulz at
# its effective rate on the algorithmic FLOP count (symmetric tiles skip ~29%), and the
# elementwise kernels at their achieved algorithmic bytes per second -- bound by the
# reference's Philox noise stream, well below the HBM copy rate.
TENSOR_FLOPS = 1.7e15
MUON_EW_BYTES = 2.0e12     # prepare (8 B) + apply (6 B) per element
ADAMW_BYTES = 1.2e12       # 14 B per element, three Philox streams (1.25e12 measured at 8 GPUs)
ADAMW8BIT_BYTES = 1.28e12  # 10.0625 B per element
SEGMENT_SECONDS = 4e-3  # per-rank Newton-Schulz time between two weight shares of a stack
COPY_STREAMS_PER_PEER = 2
HOST_BARRIER_TIMEOUT = datetime.timedelta(seconds=300)


def _ns_flops(shape, steps=5):
    r, c = shape[-2], shape[-1]
    m, n = min(r, c), max(r, c)
    batch = 1
    for s in shape[:-2]:
        batch *= s
    return batch * steps * (4 * m * m * n + 2 * m ** 3)


def _kind(group):
    """Kind of update a param group gets: Newton-Schulz (Muon), 8-bit AdamW or AdamW-SR."""
    if group.get("use_muon", "momentum" in group and "betas" not in group):
        return "muon"
    return "adamw8bit" if "optim_bits" in group else "adamw"


def _cost(p, kind, ns_steps):
    """Estimated B200 seconds of one parameter's update."""
    numel = p.numel()
    if kind == "muon" and p.ndim >= 2:
        return _ns_flops(tuple(p.shape), ns_steps) / TENSOR_FLOPS + 14 * numel / MUON_EW_BYTES
    if kind == "adamw8bit":
        return 10.0625 * numel / ADAMW8BIT_BYTES
    return 14 * numel / ADAMW_BYTES


class Sharder:
    """Spreads the per-parameter optimizer work of one optimizer over a process group.

    Weight sharing (``transport``):

    * ``"multicast"`` (chosen by the default ``"auto"`` when every rank's GPU supports NVLink
      multicast): on the first step every parameter is moved into one symmetric allocation
      (torch symmetric memory: every rank maps every rank's copy, bound to one NVLink
      multicast object) and becomes a view of its slot there. The owner's weight-updating
      kernels (apply, AdamW, 8-bit AdamW) then store each updated weight once through the
      multicast address and the NVSwitch writes it into every rank's replica: the update and
      the all-gather are one kernel, with no copies, no extra SMs and one outgoing write per
      element. Ordering: an interprocess event per rank and a host-only (gloo) barrier at the
      start of the step (no rank may still read weights an owner is about to overwrite) and at
      its end (every rank waits for every owner's writes). The parameters' storage changes
      once (``p.data`` is re-pointed); code that cached the old tensors must re-read them.
    * ``"p2p"`` (``"auto"`` without multicast): every rank maps, once, the device allocations that hold
      the parameters other ranks own (CUDA IPC) and pulls their updated values with
      copy-engine peer copies over NVLink on COPY_STREAMS_PER_PEER side streams per owner, so
      the transfers use no SMs and run under the Newton-Schulz GEMMs (the process needs
      CUDA_DEVICE_MAX_CONNECTIONS=32 so that these streams get their own hardware queues).
      Ordering: at each share point every
      rank records an interprocess event on its compute stream, a host-only (gloo) barrier
      makes sure all records are enqueued, and the copies wait on the owners' events; at the
      end of the step the compute stream waits for the copies and for the peers' copies of
      this rank's weights (another event + barrier), so the next step's updates cannot
      overwrite weights a peer is still reading. Falls back to ``"nccl"`` when the memory
      cannot be mapped (e.g. VMM / expandable-segment allocations).
    * ``"nccl"``: one NCCL broadcast per parameter from its owner.
    """

    def __init__(self, group=None, reserve_sms: int = 0, transport: str = "auto"):
        """``reserve_sms``: SMs the Newton-Schulz GEMMs leave free for concurrent NCCL
        kernels (pair it with NCCL_MAX_NCHANNELS <= reserve_sms); 0 keeps every SM.
        ``transport``: "auto" (multicast if every rank supports it, else p2p), "multicast",
        "p2p" or "nccl"."""
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("Sharder needs an initialised torch.distributed process group")
        if transport not in ("auto", "multicast", "p2p", "nccl"):
            raise ValueError("transport must be 'auto', 'multicast', 'p2p' or 'nccl'")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if reserve_sms > 0 and torch.cuda.is_available():
            from . import _lib
            sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
            _lib.load().msr_set_gemm_max_ctas(max(1, sms - int(reserve_sms)))
        self.transport = transport if torch.cuda.is_available() else "nccl"
        if self.transport in ("auto", "p2p") and int(os.environ.get("CUDA_DEVICE_MAX_CONNECTIONS", "8")) < 8 * COPY_STREAMS_PER_PEER:
            warnings.warn("Sharder(transport='p2p') runs several copy streams per peer next to the compute stream; "
                          "set CUDA_DEVICE_MAX_CONNECTIONS=32 before CUDA initialises, or copies waiting on peers "
                          "can delay compute kernels that share their hardware queue", RuntimeWarning)
        # host-only barriers for the p2p ordering (created collectively, same order on all ranks);
        # they only wait for the other ranks to issue their work, so a rank that failed ends
        # the others' wait with an error after HOST_BARRIER_TIMEOUT instead of torch's default
        self._host = dist.new_group(backend="gloo", timeout=HOST_BARRIER_TIMEOUT) if self.transport != "nccl" else None
        self._owner = None  # id(param) -> rank within the group
        self._order = None  # params in a fixed order
        self._p2p = None    # lazily built peer mappings
        self._mc = None     # lazily built multicast weights
        self._side = None   # stream of the weight updates under the multicast transport

    # -- plan -----------------------------------------------------------------------------
    def plan(self, param_groups):
        """Assign every parameter to a rank (same result on every rank)."""
        entries = []
        for gi, g in enumerate(param_groups):
            kind = _kind(g)
            for pi, p in enumerate(g["params"]):
                entries.append((_cost(p, kind, g.get("ns_steps", 5)), gi, pi, p))
        # Largest first; ties broken by position so that the plan is deterministic.
        entries.sort(key=lambda e: (-e[0], e[1], e[2]))
        heap = [(0.0, r) for r in range(self.world)]
        owner = {}
        for cost, gi, pi, p in entries:
            load, r = heapq.heappop(heap)
            owner[id(p)] = r
            heapq.heappush(heap, (load + cost, r))
        self._owner = owner
        self._order = [p for g in param_groups for p in g["params"]]
        self._index = {id(p): i for i, p in enumerate(self._order)}
        self._p2p = None
        if self._mc:
            self._mc.close()
            self._mc = None
            self.transport = "auto"
        return owner

    def loads(self, param_groups):
        """Estimated seconds of work per rank under the current plan."""
        out = [0.0] * self.world
        for g in param_groups:
            kind = _kind(g)
            for p in g["params"]:
                out[self._owner[id(p)]] += _cost(p, kind, g.get("ns_steps", 5))
        return out

    def _ensure(self, optimizer):
        if self._owner is None or any(id(p) not in self._owner for g in optimizer.param_groups for p in g["params"]):
            self.plan(optimizer.param_groups)

    # -- queries used by the optimizers -----------------------------------------------------
    def bind(self, optimizer):
        self._ensure(optimizer)
        self._groups = optimizer.param_groups
        if self.transport in ("auto", "multicast"):
            if self._mc and self._mc.stale():
                self._mc.close()
                self._mc = None  # parameters were replaced: build the shared weights again
            if self._mc is None:
                ok = _Multicast.possible(self)
                if not ok and self.transport == "multicast":
                    raise RuntimeError("Sharder(transport='multicast'): NVLink multicast is not available on every "
                                       "rank's GPU")
                self._mc = _Multicast(self) if ok else False
                self.transport = "multicast" if ok else "p2p"
        if self.transport == "p2p" and self._p2p and self._p2p.stale():
            self._p2p = None  # some owner's weights moved: every rank maps them again
        if self.transport == "p2p" and self._p2p is None:
            self._p2p = _PeerMaps(self) if _PeerMaps.possible(self) else False
            if self._p2p is False:
                self.transport = "nccl"
        self.begin_step()
        return self

    def segments(self, shape, n) -> int:
        """Number of consecutive segments a stack of ``n`` matrices of ``shape`` is shared
        in: about SEGMENT_SECONDS of Newton-Schulz per rank each, at least two matrices per
        rank per segment (so the batched GEMMs stay full), at most 8."""
        if self.transport == "multicast":
            return 1  # weights travel as the kernels write them: nothing to share in between
        per_rank = n * _ns_flops(tuple(shape)) / TENSOR_FLOPS / self.world
        return max(1, min(8, n // (2 * self.world), round(per_rank / SEGMENT_SECONDS)))

    @property
    def update_stream(self):
        """Under the multicast transport, the stream on which the optimizers run the weight
        updates (apply after each chunk's Newton-Schulz, the AdamW groups) so that their
        NVLink multicast stores overlap the Newton-Schulz GEMMs on the current stream; it
        starts after the step's start point and the step's end point waits for it. None with
        the other transports (their updates run in line and the copies overlap instead)."""
        return self._side if self.transport == "multicast" else None

    def owns(self, gi, pi) -> bool:
        return self._owner[id(self._groups[gi]["params"][pi])] == self.rank

    def muon_owner(self, gi, shape_groups):
        stacks = list(shape_groups.values())
        return lambda shape_idx, i: self._owner[id(stacks[shape_idx][i])] == self.rank

    # -- weight sharing ----------------------------------------------------------------------
    def begin_step(self):
        self._shared = set()
        self._pending = []
        self._point = 0
        if self.transport == "multicast":
            self._mc.begin()
            if self._side is None:
                self._side = torch.cuda.Stream(self._mc.device)
            self._side.wait_stream(torch.cuda.current_stream(self._mc.device))

    def share(self, params):
        """Start sharing each of ``params`` that has a gradient from its owner. Every rank
        must call this with the same tensors in the same order (the optimizers call it once
        per shape stack / param group, in a fixed order); the transfers run behind the
        kernels already issued on the current stream while later work proceeds, and
        ``sync_params`` waits for them."""
        todo = [p for p in params if p.grad is not None and id(p) not in self._shared]
        for p in todo:
            self._shared.add(id(p))
        if self.transport == "multicast":
            return  # the owners' kernels already wrote every replica
        if self.transport == "p2p":
            self._p2p.share(todo, self._point)
            self._point += 1
            return
        for p in todo:
            src = self._owner[id(p)]
            src_global = dist.get_global_rank(self.group, src) if self.group is not None else src
            self._pending.append(dist.broadcast(p.data, src=src_global, group=self.group, async_op=True))

    def sync_params(self, optimizer):
        """Share whatever was not shared yet, then make the current stream wait for all of
        this step's transfers."""
        self.share(self._order)
        if self.transport == "multicast":
            torch.cuda.current_stream(self._mc.device).wait_stream(self._side)
            self._mc.finish()
            return
        if self.transport == "p2p":
            self._p2p.finish()
            return
        for w in self._pending:
            w.wait()
        self._pending = []

    # -- gradients -----------------------------------------------------------------------
    def _src(self, r):
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def reduce_grads(self, optimizer, average: bool = True):
        """Collective replacing the data-parallel gradient all-reduce: every parameter's
        gradient is summed (or averaged) over the ranks onto its owner only, with ONE
        reduce-scatter per step over an owner-ordered packed gradient buffer -- half the
        bytes an all-reduce moves. The buffer holds rank r's parameters in chunk r (chunks
        padded to the largest one, slots aligned to 128 bytes); on the first call each
        gradient is copied into its slot and ``p.grad`` becomes a view of that slot, so later
        backward passes that accumulate into the existing ``.grad`` write straight into the
        buffer and need no copy (a gradient that was replaced, e.g. after
        ``zero_grad(set_to_none=True)``, is copied in again). Non-owners keep their local
        gradients (the step skips their parameters but still sees that they have one). Every
        rank calls it after backward with the same parameters holding gradients. Returns the
        packed buffer's layout: ``{"chunk_elements", "padding", "tensors"}``."""
        self._ensure(optimizer)
        params = [p for p in self._order if p.grad is not None]
        if not params:
            return None
        key = tuple((id(p), p.numel(), p.grad.dtype, p.grad.device, self._owner[id(p)]) for p in params)
        lay = getattr(self, "_grad_layout", None)
        if lay is None or lay["key"] != key:
            lay = self._grad_layout = self._pack_layout(params, key)
        buf, chunk = lay["buffer"], lay["chunk"]
        for p, off in lay["slots"]:
            view = buf[off:off + p.numel()].view_as(p)
            if p.grad.data_ptr() != view.data_ptr():
                view.copy_(p.grad)
                p.grad = view
        own = buf[self.rank * chunk:(self.rank + 1) * chunk]
        if dist.get_backend(self.group) == "nccl":
            # in place: the output is this rank's chunk of the input
            dist.reduce_scatter_tensor(own, buf, op=dist.ReduceOp.AVG if average else dist.ReduceOp.SUM,
                                       group=self.group)
        else:  # gloo (CPU tests) has no reduce-scatter: the same result through an all-reduce
            total = buf.clone()
            dist.all_reduce(total, group=self.group)
            mine = total[self.rank * chunk:(self.rank + 1) * chunk]
            own.copy_(mine / self.world if average else mine)
        return {"chunk_elements": chunk, "padding": lay["padding"], "tensors": len(params)}

    def _pack_layout(self, params, key):
        """Owner-ordered slots of the packed gradient buffer (same on every rank)."""
        align = 64  # elements: 128-byte slots keep every gradient 16-byte aligned
        per_rank = [[] for _ in range(self.world)]
        for p in params:
            per_rank[self._owner[id(p)]].append(p)
        sizes = []
        for lst in per_rank:
            sizes.append(sum((p.numel() + align - 1) // align * align for p in lst))
        chunk = max(align, max(sizes))
        slots = []
        for r, lst in enumerate(per_rank):
            off = r * chunk
            for p in lst:
                slots.append((p, off))
                off += (p.numel() + align - 1) // align * align
        g0 = params[0].grad
        buf = torch.zeros(self.world * chunk, dtype=g0.dtype, device=g0.device)
        used = sum(p.numel() for p in params)
        return {"key": key, "buffer": buf, "chunk": chunk, "slots": slots,
                "padding": 1.0 - used / (self.world * chunk)}

    # -- checkpoints -----------------------------------------------------------------------
    def gather_state(self, optimizer, dst=None):
        """Collective: copy every parameter's optimizer state from its owner to rank ``dst``
        (every rank when None), so that ``optimizer.state_dict()`` there holds the whole
        state with the reference's keys and dtypes (checkpoints stay interchangeable with
        the single-GPU classes). Each owner packs all the state tensors it holds into one
        byte buffer (16-byte aligned slots, any dtype), so the transfer is one broadcast per
        owner (``dst`` None) or one send/receive pair per owner (``dst`` given; ranks other
        than the owner and ``dst`` move nothing) -- not one collective per tensor. Loading
        needs no counterpart: every rank loads the full checkpoint and uses the part it owns."""
        self._ensure(optimizer)
        order = [p for g in optimizer.param_groups for p in g["params"]]
        meta = {}
        for i, p in enumerate(order):
            if self._owner[id(p)] != self.rank:
                continue
            meta[i] = {k: (("t", tuple(v.shape), str(v.dtype).split(".")[-1]) if torch.is_tensor(v) else ("v", v))
                       for k, v in optimizer.state.get(p, {}).items()}
        metas = [None] * self.world
        dist.all_gather_object(metas, meta, group=self.group)
        device = order[0].device if order else torch.device("cpu")
        for owner in range(self.world):
            receive = owner != self.rank and (dst is None or dst == self.rank)
            items, size = [], 0
            for i in sorted(metas[owner]):
                p = order[i]
                for k, spec in sorted(metas[owner][i].items()):
                    if spec[0] == "v":
                        if receive:
                            optimizer.state[p][k] = spec[1]
                        continue
                    shape, dtype = spec[1], getattr(torch, spec[2])
                    nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
                    items.append((p, k, shape, dtype, size, nbytes))
                    size = (size + nbytes + 15) // 16 * 16
            if size == 0 or (dst is not None and owner == dst):
                continue
            if self.rank == owner:
                buf = torch.empty(size, dtype=torch.uint8, device=device)
                for p, k, shape, dtype, off, nbytes in items:
                    buf[off:off + nbytes].copy_(optimizer.state[p][k].contiguous().view(-1).view(torch.uint8))
            elif dst is None or dst == self.rank:
                buf = torch.empty(size, dtype=torch.uint8, device=device)
            else:
                continue  # a point-to-point transfer between the owner and dst
            if dst is None:
                dist.broadcast(buf, src=self._src(owner), group=self.group)
            elif self.rank == owner:
                dist.send(buf, dst=self._src(dst), group=self.group)
            else:
                dist.recv(buf, src=self._src(owner), group=self.group)
            if not receive:
                continue
            for p, k, shape, dtype, off, nbytes in items:
                st = optimizer.state[p]
                t = st.get(k)
                if not (torch.is_tensor(t) and tuple(t.shape) == shape and t.dtype == dtype and t.is_contiguous()
                        and t.device == buf.device):
                    t = torch.empty(shape, dtype=dtype, device=buf.device)
                t.view(-1).view(torch.uint8).copy_(buf[off:off + nbytes])
                st[k] = t


def _event_set(sh, lib):
    """One interprocess event of this rank plus the opened events of every peer (collective
    over the host group). Returns (own event, {peer rank: event}, [handles to destroy])."""
    from . import _lib
    ev = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    _lib.check(lib.msr_ipc_event_create(ctypes.byref(ev), h), "msr_ipc_event_create")
    owned = [ev.value]
    handles = [None] * sh.world
    dist.all_gather_object(handles, bytes(h.raw), group=sh._host)
    peers = {}
    for r, hh in enumerate(handles):
        if r == sh.rank:
            continue
        pe = ctypes.c_void_p()
        _lib.check(lib.msr_ipc_event_open(hh, ctypes.byref(pe)), "msr_ipc_event_open")
        owned.append(pe.value)
        peers[r] = pe.value
    return ev.value, peers, owned


def _cross_rank_point(sh, lib, events, stream):
    """Every rank's ``stream`` continues only after every rank's stream reached this point:
    record this rank's event, a host barrier (all records are enqueued), wait for the peers'."""
    from . import _lib
    ev, peers, _ = events
    _lib.check(lib.msr_event_record(ctypes.c_void_p(ev), ctypes.c_void_p(stream.cuda_stream)), "msr_event_record")
    dist.barrier(group=sh._host)
    for e in peers.values():
        _lib.check(lib.msr_stream_wait_event(ctypes.c_void_p(stream.cuda_stream), ctypes.c_void_p(e)),
                   "msr_stream_wait_event")


class _Multicast:
    """Weights in one symmetric allocation bound to an NVLink multicast object (the
    ``multicast`` transport). Slots are 128-byte aligned, so every parameter keeps 16-byte
    alignment and an odd-length parameter is followed by padding the kernels may write."""

    ALIGN = 64  # elements (bf16): 128-byte slots

    @staticmethod
    def possible(sh) -> bool:
        """Collective (host group): every rank's GPU supports NVLink multicast and every
        parameter is a bf16 CUDA tensor."""
        ok = 0
        try:
            import torch.distributed._symmetric_memory  # noqa: F401
            from torch._C._autograd import DeviceType
            from torch._C._distributed_c10d import _SymmetricMemory
            params = sh._order
            ok = int(bool(params) and all(p.is_cuda and p.dtype == torch.bfloat16 for p in params)
                     and _SymmetricMemory.has_multicast_support(DeviceType.CUDA, torch.cuda.current_device()))
        except Exception:
            ok = 0
        flags = [None] * sh.world
        dist.all_gather_object(flags, ok, group=sh._host)
        return all(flags)

    def __init__(self, sh):
        import torch.distributed._symmetric_memory as symm
        from . import _lib
        from . import kernels as K
        self.sh = sh
        self.lib = _lib.load()
        self.device = torch.device("cuda", torch.cuda.current_device())
        slots, off = [], 0
        for p in sh._order:
            slots.append((p, off))
            off += (p.numel() + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        self.flat = symm.empty(max(off, self.ALIGN), dtype=torch.bfloat16, device=self.device)
        self.handle = symm.rendezvous(self.flat, sh.group if sh.group is not None else dist.group.WORLD)
        mc = int(self.handle.multicast_ptr)
        ok = torch.tensor([1 if mc else 0], dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=sh._host)
        if not int(ok.item()):
            raise RuntimeError("NVLink multicast address missing after the symmetric-memory rendezvous")
        base = self.flat.data_ptr()
        mapping = {}
        for p, o in slots:
            view = self.flat[o:o + p.numel()].view_as(p)
            view.copy_(p.detach())
            p.data = view
            if sh._owner[id(p)] == sh.rank:
                mapping[base + 2 * o] = mc + 2 * o
        torch.cuda.current_stream(self.device).synchronize()
        self.exported = [(p, p.data_ptr()) for p, _ in slots]
        self.registered = list(mapping)
        K.register_multicast(mapping)
        self.start = _event_set(sh, self.lib)
        self.done = _event_set(sh, self.lib)

    def stale(self) -> bool:
        """Collective (host group): True on every rank if any rank's parameters no longer are
        the views of the shared allocation (``p.data`` replaced, a module's
        ``load_state_dict`` that assigned new tensors ...), so all ranks rebuild together."""
        moved = any(p.data_ptr() != ptr for p, ptr in self.exported)
        flag = torch.tensor([1 if moved else 0], dtype=torch.int32)
        dist.all_reduce(flag, group=self.sh._host)
        return bool(flag.item())

    def begin(self):
        # no rank may still read (e.g. a backward pass) weights an owner is about to overwrite
        _cross_rank_point(self.sh, self.lib, self.start, torch.cuda.current_stream(self.device))

    def finish(self):
        # every owner's multicast writes (fenced at system scope by the kernels) are done
        _cross_rank_point(self.sh, self.lib, self.done, torch.cuda.current_stream(self.device))

    def close(self):
        from . import kernels as K
        K.unregister_multicast(self.registered)
        self.registered = []
        for ev in (self.start, self.done):
            for e in ev[2]:
                self.lib.msr_event_destroy(ctypes.c_void_p(e))
        self.start = self.done = (None, {}, [])


class _PeerMaps:
    """CUDA IPC mappings, side streams and interprocess events of the ``p2p`` transport."""

    @staticmethod
    def possible(sh):
        from . import _lib
        lib = _lib.load()
        ok = 1
        for p in sh._order:
            if sh._owner[id(p)] == sh.rank:
                h = ctypes.create_string_buffer(64)
                off = ctypes.c_uint64()
                if lib.msr_ipc_export(ctypes.c_void_p(p.data_ptr()), h, ctypes.byref(off)) != 0:
                    ok = 0
                    break
        flags = [None] * sh.world
        dist.all_gather_object(flags, ok, group=sh._host)
        return all(flags)

    def __init__(self, sh):
        from . import _lib
        self.sh = sh
        self.lib = _lib.load()
        self.device = torch.device("cuda", torch.cuda.current_device())
        mine = []
        self.exported = []  # (param, address at export): the peers' mappings point there
        for i, p in enumerate(sh._order):
            if sh._owner[id(p)] == sh.rank:
                h = ctypes.create_string_buffer(64)
                off = ctypes.c_uint64()
                _lib.check(self.lib.msr_ipc_export(ctypes.c_void_p(p.data_ptr()), h, ctypes.byref(off)),
                           "msr_ipc_export")
                mine.append((i, bytes(h.raw), off.value))
                self.exported.append((p, p.data_ptr()))
        lists = [None] * sh.world
        dist.all_gather_object(lists, mine, group=sh._host)
        self.bases = []
        opened = {}
        self.remote = {}
        for r, lst in enumerate(lists):
            if r == sh.rank:
                continue
            for i, h, off in lst:
                if (r, h) not in opened:
                    base = ctypes.c_void_p()
                    _lib.check(self.lib.msr_ipc_import(h, ctypes.byref(base)), "msr_ipc_import")
                    opened[(r, h)] = base.value
                    self.bases.append(base.value)
                self.remote[i] = opened[(r, h)] + off
        # several copy streams per owner spread the transfers over more copy engines
        self.streams = {r: [torch.cuda.Stream(self.device) for _ in range(COPY_STREAMS_PER_PEER)]
                        for r in range(sh.world) if r != sh.rank}
        self.next_stream = {r: 0 for r in self.streams}
        self.owned_events = []
        self.events = []      # per share point: (local event, {rank: peer event})
        self.done = self._event_set()

    def stale(self) -> bool:
        """Collective (host group): True on every rank if any rank's owned parameters no
        longer live where they were exported (``.to()``, a ``load_state_dict`` that
        replaced them, re-materialised tensors), so that all ranks rebuild their mappings
        together instead of copying from stale peer addresses."""
        moved = any(p.data_ptr() != ptr for p, ptr in self.exported)
        flag = torch.tensor([1 if moved else 0], dtype=torch.int32)
        dist.all_reduce(flag, group=self.sh._host)
        return bool(flag.item())

    def _event_set(self):
        """One interprocess event of this rank plus the opened events of every peer."""
        from . import _lib
        ev = ctypes.c_void_p()
        h = ctypes.create_string_buffer(64)
        _lib.check(self.lib.msr_ipc_event_create(ctypes.byref(ev), h), "msr_ipc_event_create")
        self.owned_events.append(ev.value)
        handles = [None] * self.sh.world
        dist.all_gather_object(handles, bytes(h.raw), group=self.sh._host)
        peers = {}
        for r, hh in enumerate(handles):
            if r == self.sh.rank:
                continue
            pe = ctypes.c_void_p()
            _lib.check(self.lib.msr_ipc_event_open(hh, ctypes.byref(pe)), "msr_ipc_event_open")
            self.owned_events.append(pe.value)
            peers[r] = pe.value
        return ev.value, peers

    def share(self, params, point):
        while len(self.events) <= point:
            self.events.append(self._event_set())
        ev, peers = self.events[point]
        main = torch.cuda.current_stream(self.device)
        self._check(self.lib.msr_event_record(ctypes.c_void_p(ev), ctypes.c_void_p(main.cuda_stream)))
        dist.barrier(group=self.sh._host)  # every owner's record of this point is enqueued
        waited = set()
        for p in params:
            r = self.sh._owner[id(p)]
            if r == self.sh.rank:
                continue
            if r not in waited:
                for s in self.streams[r]:
                    self._check(self.lib.msr_stream_wait_event(ctypes.c_void_p(s.cuda_stream),
                                                               ctypes.c_void_p(peers[r])))
                waited.add(r)
            s = self.streams[r][self.next_stream[r]]
            self.next_stream[r] = (self.next_stream[r] + 1) % len(self.streams[r])
            nbytes = p.numel() * p.element_size()
            self._check(self.lib.msr_copy_async(ctypes.c_void_p(p.data_ptr()),
                                                ctypes.c_void_p(self.remote[self.sh._index[id(p)]]), nbytes,
                                                ctypes.c_void_p(s.cuda_stream)))

    @staticmethod
    def _check(st):
        if st:
            from . import _lib
            _lib.check(st, "peer copy")

    def finish(self):
        main = torch.cuda.current_stream(self.device)
        for ss in self.streams.values():
            for s in ss:
                main.wait_stream(s)
        ev, peers = self.done
        # this rank's copies of its peers' weights are done ...
        self._check(self.lib.msr_event_record(ctypes.c_void_p(ev), ctypes.c_void_p(main.cuda_stream)))
        dist.barrier(group=self.sh._host)
        for e in peers.values():           # ... and no peer still reads this rank's weights
            self._check(self.lib.msr_stream_wait_event(ctypes.c_void_p(main.cuda_stream), ctypes.c_void_p(e)))

    def __del__(self):
        try:
            for e in self.owned_events:
                self.lib.msr_event_destroy(ctypes.c_void_p(e))
            for b in self.bases:
                self.lib.msr_ipc_close(ctypes.c_void_p(b))
        except Exception:
            pass
