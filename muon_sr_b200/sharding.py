"""Parameter-sharded optimizer work across the ranks of one node.

The reference is single-device; data-parallel replicas each run the whole optimizer step
and stay identical because the rounding seeds depend only on (step, index). Here each rank
runs the step for the parameters it owns and the updated bf16 weights are then shared over
NCCL (NVLink / NVSwitch), so the step's work is divided by the number of ranks.

* Partition: whole tensors (Newton-Schulz needs each full matrix), longest-processing-time
  greedy on an estimated B200 time per tensor -- Newton-Schulz FLOPs at the tensor-core rate
  for Muon matrices, bytes at the HBM rate for AdamW / 8-bit tensors.
* Seeds and Philox counters stay global, so every rank writes exactly the bits a single GPU
  would (Newton-Schulz computes each matrix independently of how the batch is chunked).
* Sharing: as soon as a shape stack (or param group) is updated, its parameters are
  broadcast from their owners on NCCL's stream, so the transfers run under the next
  stacks' Newton-Schulz work; the step ends by waiting for all of them.
* Optimizer state (momentum, moments) stays with the owner; ``state_dict()`` on a rank holds
  valid values only for the parameters that rank owns.
"""
import heapq

import torch
import torch.distributed as dist

TENSOR_FLOPS = 1.4e15   # sustained dense bf16 on B200, used only to weigh the partition
HBM_BYTES = 6.5e12


def _ns_flops(shape, steps=5):
    r, c = shape[-2], shape[-1]
    m, n = min(r, c), max(r, c)
    batch = 1
    for s in shape[:-2]:
        batch *= s
    return batch * steps * (4 * m * m * n + 2 * m ** 3)


def _cost(p, use_muon, ns_steps):
    numel = p.numel()
    if use_muon and p.ndim >= 2:
        return _ns_flops(tuple(p.shape), ns_steps) / TENSOR_FLOPS + 14 * numel / HBM_BYTES
    return 14 * numel / HBM_BYTES


class Sharder:
    """Spreads the per-parameter optimizer work of one optimizer over a process group."""

    def __init__(self, group=None, reserve_sms: int = 0):
        """``reserve_sms``: SMs the Newton-Schulz GEMMs leave free so that the weight
        broadcasts (NCCL kernels) run concurrently with them (pair it with
        NCCL_MAX_NCHANNELS <= reserve_sms); 0 keeps every SM for the GEMMs."""
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("Sharder needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if reserve_sms > 0 and torch.cuda.is_available():
            from . import _lib
            sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
            _lib.load().msr_set_gemm_max_ctas(max(1, sms - int(reserve_sms)))
        self._owner = None  # id(param) -> rank within the group
        self._order = None  # params in a fixed order for the broadcasts

    # -- plan -----------------------------------------------------------------------------
    def plan(self, param_groups):
        """Assign every parameter to a rank (same result on every rank)."""
        entries = []
        for gi, g in enumerate(param_groups):
            use_muon = g.get("use_muon", "momentum" in g and "betas" not in g)
            for pi, p in enumerate(g["params"]):
                entries.append((_cost(p, use_muon, g.get("ns_steps", 5)), gi, pi, p))
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
        return owner

    def loads(self, param_groups):
        """Estimated seconds of work per rank under the current plan."""
        out = [0.0] * self.world
        for g in param_groups:
            use_muon = g.get("use_muon", "momentum" in g and "betas" not in g)
            for p in g["params"]:
                out[self._owner[id(p)]] += _cost(p, use_muon, g.get("ns_steps", 5))
        return out

    def _ensure(self, optimizer):
        if self._owner is None or any(id(p) not in self._owner for g in optimizer.param_groups for p in g["params"]):
            self.plan(optimizer.param_groups)

    # -- queries used by the optimizers -----------------------------------------------------
    def bind(self, optimizer):
        self._ensure(optimizer)
        self._groups = optimizer.param_groups
        self.begin_step()
        return self

    def owns(self, gi, pi) -> bool:
        return self._owner[id(self._groups[gi]["params"][pi])] == self.rank

    def muon_owner(self, gi, shape_groups):
        stacks = list(shape_groups.values())
        return lambda shape_idx, i: self._owner[id(stacks[shape_idx][i])] == self.rank

    # -- weight sharing ----------------------------------------------------------------------
    def share(self, params):
        """Start broadcasting each of ``params`` that has a gradient from its owner. Every
        rank must call this with the same tensors in the same order (the optimizers call it
        once per shape stack / param group, in a fixed order). The broadcasts are enqueued
        behind the kernels already issued on the current stream and run while later work
        proceeds; ``sync_params`` waits for them."""
        if not hasattr(self, "_pending"):
            self._pending = []
        for p in params:
            if p.grad is None or id(p) in self._shared:
                continue
            self._shared.add(id(p))
            src = self._owner[id(p)]
            src_global = dist.get_global_rank(self.group, src) if self.group is not None else src
            self._pending.append(dist.broadcast(p.data, src=src_global, group=self.group, async_op=True))

    def begin_step(self):
        self._shared = set()
        self._pending = []

    def sync_params(self, optimizer):
        """Share whatever was not shared yet, then make the current stream wait for all of
        this step's broadcasts."""
        self.share(self._order)
        for w in self._pending:
            w.wait()
        self._pending = []
