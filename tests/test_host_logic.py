"""Host-side logic that needs no GPU: seeds, Philox keys, the sharding plan, API errors."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muon_sr_b200 import TritonAdamW8bit, TritonMuonSRWithAuxAdam, create_dynamic_map, seeds
from muon_sr_b200.sharding import Sharder
from oracle import adamw8bit as o8
from oracle import philox as op
from tests._golden import load


def test_seed_formulas_match_oracle():
    for step in (1, 2, 999, 123456):
        for idx in (0, 5, 10002, 2**31 - 1):
            for salt in (0, 1):
                assert seeds.deterministic_seed(step, idx, salt) == op.deterministic_seed(step, idx, salt)


@pytest.mark.parametrize("seed", [0, 1, 2**31 - 2, 2**31 - 1, 2**31, 2**32 - 2, 2**32 - 1])
def test_triton_key(seed):
    for add in range(3):
        assert seeds.triton_key(seed, add) == op.triton_key(seed, add)


def test_wrapped_key_edge():
    # i32 seed + 2 wraps and is sign-extended into the high key word
    assert seeds.triton_key(2**31 - 1, 1) == 0xFFFFFFFF80000000
    assert seeds.triton_key(2**32 - 1, 1) == 1 << 32


def test_codebooks_equal_golden():
    d = load("adamw8bit.npz")
    assert np.array_equal(create_dynamic_map(True).numpy().view(np.uint32), d["qmap1"].view(np.uint32))
    assert np.array_equal(create_dynamic_map(False).numpy().view(np.uint32), d["qmap2"].view(np.uint32))


def test_hybrid_requires_use_muon_and_fills_defaults():
    p = torch.nn.Parameter(torch.zeros(4, 4, dtype=torch.bfloat16))
    with pytest.raises(AssertionError):
        TritonMuonSRWithAuxAdam([dict(params=[p])])
    opt = TritonMuonSRWithAuxAdam([dict(params=[p], use_muon=True)], batch_ns=True)
    g = opt.param_groups[0]
    assert (g["lr"], g["momentum"], g["nesterov"], g["ns_steps"], g["weight_decay"]) == (0.02, 0.95, True, 5, 0)
    q = torch.nn.Parameter(torch.zeros(4, dtype=torch.bfloat16))
    opt = TritonMuonSRWithAuxAdam([dict(params=[q], use_muon=False)])
    g = opt.param_groups[0]
    assert (g["lr"], g["betas"], g["eps"], g["weight_decay"]) == (3e-4, (0.9, 0.95), 1e-10, 0)


@pytest.mark.parametrize("kw,msg", [
    (dict(lr=-1.0), "lr must be"), (dict(eps=0.0), "eps must be positive"), (dict(betas=(0.9, 1.0)), "betas"),
    (dict(block_size=48), "block_size"), (dict(optim_bits=32), "optim_bits"), (dict(min_8bit_size=-1), "optim_bits"),
])
def test_adamw8bit_validation(kw, msg):
    p = torch.nn.Parameter(torch.zeros(4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match=msg):
        TritonAdamW8bit([p], **kw)


def test_adamw8bit_rejects_cpu_params_on_step():
    p = torch.nn.Parameter(torch.zeros(4096, dtype=torch.bfloat16))
    p.grad = torch.zeros_like(p)
    opt = TritonAdamW8bit([p])
    with pytest.raises(ValueError, match="CUDA BF16"):
        opt.step()


def test_for_model_groups():
    model = torch.nn.Sequential(torch.nn.Embedding(100, 64), torch.nn.Linear(64, 128), torch.nn.LayerNorm(128))
    opt = TritonAdamW8bit.for_model(model.to(torch.bfloat16))
    bits = {g["optim_bits"]: len(g["params"]) for g in opt.param_groups}
    assert bits == {8: 1, 16: 4}  # Linear weight 8-bit; embedding, bias, LN weight/bias 16-bit
    with pytest.raises(ValueError):
        TritonAdamW8bit.for_model(model, optim_bits=8)


def _llama_like_groups():
    mk = lambda *s: torch.nn.Parameter(torch.empty(*s, dtype=torch.bfloat16, device="meta"))
    muon, adam = [], [mk(1000, 64), mk(1000, 64)]
    for _ in range(4):
        muon += [mk(64, 64), mk(16, 64), mk(16, 64), mk(64, 64), mk(224, 64), mk(224, 64), mk(64, 224)]
        adam += [mk(64), mk(64)]
    return [dict(params=muon, use_muon=True, ns_steps=5), dict(params=adam, use_muon=False)]


def _plan_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        groups = _llama_like_groups()
        sh = Sharder()
        owner = sh.plan(groups)
        order = [owner[id(p)] for g in groups for p in g["params"]]
        loads = sh.loads(groups)
        # every rank computes the same plan; gather them to rank 0
        gathered = [None] * world
        dist.all_gather_object(gathered, order)
        # broadcast of owned CPU tensors: each rank writes its rank into the tensors it owns
        ts = [torch.full((3,), -1.0) for _ in order]
        for t, o in zip(ts, order):
            if o == rank:
                t.fill_(float(rank))
        for t, o in zip(ts, order):
            dist.broadcast(t, src=o)
        ok = all(float(t[0]) == o for t, o in zip(ts, order))
        if rank == 0:
            out.put((gathered, loads, ok))
    finally:
        dist.destroy_process_group()


def test_sharding_plan_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_plan_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, loads, ok = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert gathered[0] == gathered[1], "ranks disagree on the plan"
    assert set(gathered[0]) == {0, 1}
    assert max(loads) / min(loads) < 1.25, loads
    assert ok
