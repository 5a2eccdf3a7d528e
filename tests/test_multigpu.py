"""Sharded optimizer steps on 2 GPUs produce exactly the single-GPU bits.

Each rank updates only the tensors the Sharder assigns to it and receives the others over
NVLink; seeds and Philox counters are global and Newton-Schulz computes each matrix on its
own, so the parameters after every step must equal a 1-GPU run bit for bit (also when
stacks are shared segment by segment, and for the random-seed classes). The gradients
start rank-local and reach their owners through ``reduce_grads``; after the steps
``gather_state`` must reproduce the single-GPU optimizer state (checkpoint interop).
Skipped on a box with fewer than 2 GPUs.
"""
import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES_MUON = [(256, 512)] * 9 + [(512, 256)] * 2 + [(128, 384)] * 2
SHAPES_ADAM = [(1000, 64), (64,), (64,), (67,)]  # 67: a ragged end (4-byte multicast pairs)


def _params(device):
    g = torch.Generator().manual_seed(3)
    mk = lambda s: torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16().to(device))
    return [mk(s) for s in SHAPES_MUON], [mk(s) for s in SHAPES_ADAM]


def _grads(step, device):
    g = torch.Generator().manual_seed(100 + step)
    return [(torch.randn(*s, generator=g) * 1e-3).bfloat16().to(device) for s in SHAPES_MUON + SHAPES_ADAM]


def _state_tensors(opt):
    """Every tensor of state_dict()["state"], in a fixed order."""
    sd = opt.state_dict()["state"]
    return [sd[i][k] for i in sorted(sd) for k in sorted(sd[i]) if torch.is_tensor(sd[i][k])]


def _run(device, shard, steps=3, batch_ns=True, rank=0):
    """Hybrid steps then 8-bit steps. With ``shard``: each rank starts from local gradients
    (2 g on rank 0, 0 elsewhere) that ``reduce_grads`` averages onto the owners, and the
    state is gathered from the owners before it is returned."""
    from muon_sr_b200 import TritonAdamW8bit, TritonMuonSRWithAuxAdam
    muon, adam = _params(device)
    sh = shard() if shard else None
    opt = TritonMuonSRWithAuxAdam([dict(params=muon, use_muon=True, weight_decay=0.01),
                                   dict(params=adam, use_muon=False, weight_decay=0.01)],
                                  batch_ns=batch_ns, shard=sh)

    def set_grads(params, grads):
        for p, g in zip(params, grads):
            p.grad = g if sh is None else (g * 2 if rank == 0 else torch.zeros_like(g))

    for k in range(steps):
        set_grads(muon + adam, _grads(k, device))
        if sh is not None:
            sh.reduce_grads(opt)
        opt.step()
    params8 = [torch.nn.Parameter(p.detach().clone()) for p in muon + adam]
    sh8 = shard() if shard else None
    opt8 = TritonAdamW8bit(params8, lr=1e-3, weight_decay=0.01, shard=sh8)
    for k in range(2):
        set_grads(params8, _grads(10 + k, device))
        if sh8 is not None:
            sh8.reduce_grads(opt8)
        opt8.step()
    # the random-seed variant: every process draws its seeds from an identically seeded
    # torch generator, ranks skip (but still draw) the seeds of tensors they do not own
    from muon_sr_b200 import MuonSRWithAuxAdam
    muon_r = [torch.nn.Parameter(p.detach().clone()) for p in muon]
    adam_r = [torch.nn.Parameter(p.detach().clone()) for p in adam]
    sh_r = shard() if shard else None
    opt_r = MuonSRWithAuxAdam([dict(params=muon_r, use_muon=True), dict(params=adam_r, use_muon=False)],
                              batch_ns=batch_ns, shard=sh_r)
    torch.manual_seed(1234)
    for k in range(2):
        for p, g in zip(muon_r + adam_r, _grads(20 + k, device)):
            p.grad = g
        opt_r.step()
    if sh is not None:
        sh.gather_state(opt)
        sh8.gather_state(opt8)
    torch.cuda.synchronize()
    state = _state_tensors(opt) + _state_tensors(opt8)
    return ([p.detach().cpu() for p in muon + adam + params8] + [t.detach().cpu() for t in state] +
            [p.detach().cpu() for p in muon_r + adam_r])


def _bits(t):
    """Raw bytes of a tensor of any dtype (bf16 weights/moments, uint8 codes, fp32 absmax)."""
    return t.contiguous().view(-1).view(torch.uint8).numpy()


def _worker(rank, world, port, q, transport):
    import functools

    import torch.distributed as dist
    from muon_sr_b200 import Sharder, sharding
    sharding.SEGMENT_SECONDS = 1e-9  # share the larger stacks in segments even at these sizes
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_DEVICE_MAX_CONNECTIONS="32")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        if transport == "multicast":
            probe = Sharder(transport="auto")
            probe._order = [torch.zeros(8, dtype=torch.bfloat16, device="cuda")]
            if not sharding._Multicast.possible(probe):
                if rank == 0:
                    q.put("no multicast")
                dist.barrier()
                return
        out = _run(torch.device("cuda", rank), functools.partial(Sharder, transport=transport), rank=rank)
        torch.cuda.synchronize()
        if rank == 0:
            q.put([_bits(t) for t in out])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "multicast"])
def test_two_gpu_sharded_step_equals_single_gpu(transport):
    """Weights shared by copy-engine peer pulls (p2p) or stored by the owners' kernels through
    an NVLink multicast address (multicast): the same bits as one GPU."""
    import numpy as np
    single = [_bits(t) for t in _run(torch.device("cuda", 0), None)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 500 + (7 if transport == "multicast" else 0)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, transport)) for r in range(2)]
    for p in procs:
        p.start()
    sharded = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    if sharded == "no multicast":
        pytest.skip("NVLink multicast is not available on these GPUs")
    for i, (a, b) in enumerate(zip(single, sharded)):
        assert np.array_equal(a, b), f"tensor {i} (parameters, then optimizer state) differs between 1 and 2 GPUs"
