"""Sharded optimizer steps on 2 GPUs (NCCL) produce exactly the single-GPU bits.

Each rank updates only the tensors the Sharder assigns to it and receives the others by
broadcast; seeds and Philox counters are global and Newton-Schulz computes each matrix on
its own, so the parameters after every step must equal a 1-GPU run bit for bit. Skipped on
a box with fewer than 2 GPUs.
"""
import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES_MUON = [(256, 512)] * 3 + [(512, 256)] * 2 + [(128, 384)] * 2
SHAPES_ADAM = [(1000, 64), (64,), (64,)]


def _params(device):
    g = torch.Generator().manual_seed(3)
    mk = lambda s: torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).bfloat16().to(device))
    return [mk(s) for s in SHAPES_MUON], [mk(s) for s in SHAPES_ADAM]


def _grads(step, device):
    g = torch.Generator().manual_seed(100 + step)
    return [(torch.randn(*s, generator=g) * 1e-3).bfloat16().to(device) for s in SHAPES_MUON + SHAPES_ADAM]


def _run(device, shard, steps=3, batch_ns=True):
    from muon_sr_b200 import TritonAdamW8bit, TritonMuonSRWithAuxAdam
    muon, adam = _params(device)
    opt = TritonMuonSRWithAuxAdam([dict(params=muon, use_muon=True, weight_decay=0.01),
                                   dict(params=adam, use_muon=False, weight_decay=0.01)],
                                  batch_ns=batch_ns, shard=shard() if shard else None)
    for k in range(steps):
        for p, g in zip(muon + adam, _grads(k, device)):
            p.grad = g
        opt.step()
    params8 = [torch.nn.Parameter(p.detach().clone()) for p in muon + adam]
    opt8 = TritonAdamW8bit(params8, lr=1e-3, weight_decay=0.01, shard=shard() if shard else None)
    for k in range(2):
        for p, g in zip(params8, _grads(10 + k, device)):
            p.grad = g
        opt8.step()
    torch.cuda.synchronize()
    return [p.detach().cpu() for p in muon + adam + params8]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from muon_sr_b200 import Sharder
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        out = _run(torch.device("cuda", rank), Sharder)
        if rank == 0:
            q.put([t.view(torch.int16).numpy() for t in out])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_step_equals_single_gpu():
    import numpy as np
    single = [t.view(torch.int16).numpy() for t in _run(torch.device("cuda", 0), None)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    sharded = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for i, (a, b) in enumerate(zip(single, sharded)):
        assert np.array_equal(a, b), f"tensor {i} differs between 1 and 2 GPUs"
