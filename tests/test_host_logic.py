"""Host-side logic that needs no GPU: seeds, Philox keys, the sharding plan, API errors."""
import ctypes
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muon_sr_b200 import TritonAdamW8bit, TritonMuonSRWithAuxAdam, create_dynamic_map, seeds
from muon_sr_b200.sharding import Sharder
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
    (dict(block_size=48), "block_size"), (dict(optim_bits=32), "optim_bits"), (dict(min_8bit_size=-1), "min_8bit_size"),
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


def _state_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mk = lambda *s: torch.nn.Parameter(torch.zeros(*s, dtype=torch.bfloat16))
        muon = [mk(8, 16), mk(8, 16), mk(16, 8), mk(8, 16), mk(4, 4)]
        adam = [mk(16), mk(5, 3), mk(7)]
        opt = TritonMuonSRWithAuxAdam([dict(params=muon, use_muon=True), dict(params=adam, use_muon=False)],
                                      batch_ns=True)
        sh = Sharder()
        sh.plan(opt.param_groups)
        order = [p for g in opt.param_groups for p in g["params"]]
        owner = [sh._owner[id(p)] for p in order]
        val = lambda i: float(2 * (i % 16) + owner[i])

        def fill():
            # what a sharded step leaves behind: every rank has every key, owners hold values
            for i, p in enumerate(order):
                mine = owner[i] == rank
                st = opt.state[p]
                st["step"] = 3 if mine else 0
                if i < len(muon):
                    st["momentum_buffer"] = torch.full(p.shape, val(i) if mine else -1.0, dtype=torch.bfloat16)
                else:
                    st["ema"] = torch.full(p.shape, val(i) if mine else -1.0, dtype=torch.bfloat16)
                    st["ema_squared"] = torch.full(p.shape, val(i) + 0.5 if mine else -1.0, dtype=torch.bfloat16)

        def complete():
            ok = True
            for i, p in enumerate(order):
                st = opt.state[p]
                ok &= st["step"] == 3
                if i < len(muon):
                    ok &= bool((st["momentum_buffer"].float() == val(i)).all())
                else:
                    ok &= bool((st["ema"].float() == val(i)).all()) and bool((st["ema_squared"].float() == val(i) + 0.5).all())
            return ok

        fill()
        sh.gather_state(opt)
        ok_all = complete()
        sd = opt.state_dict()
        keys = [sorted(sd["state"][i].keys()) for i in range(len(order))]
        fill()
        sh.gather_state(opt, dst=0)
        ok_dst = complete() if rank == 0 else not complete()

        for i, p in enumerate(order):
            p.grad = torch.full(p.shape, float(rank + 1 + i % 7), dtype=torch.bfloat16)
        lay = sh.reduce_grads(opt)
        ok_red = all(bool((p.grad.float() == ((i % 7) + 1.5 if owner[i] == rank else rank + 1 + i % 7)).all())
                     for i, p in enumerate(order))
        # the gradients are now views of the packed buffer: a backward pass accumulating into
        # them (here: an in-place fill) needs no copy; a replaced gradient is copied in again
        buf_ptr = sh._grad_layout["buffer"].data_ptr()
        ok_red &= all(buf_ptr <= p.grad.data_ptr() < buf_ptr + sh._grad_layout["buffer"].numel() * 2 for p in order)
        for i, p in enumerate(order):
            if i == 0:
                p.grad = torch.full(p.shape, float(2 * rank + 3), dtype=torch.bfloat16)
            else:
                p.grad.fill_(float(3 * rank + i % 5))
        sh.reduce_grads(opt)

        def local(r, i):
            return 2 * r + 3 if i == 0 else 3 * r + i % 5

        def want(i):
            return (local(0, i) + local(1, i)) / 2 if owner[i] == rank else local(rank, i)
        ok_red &= all(bool((p.grad.float() == want(i)).all()) for i, p in enumerate(order))
        ok_red &= lay["tensors"] == len(order) and 0.0 <= lay["padding"] < 1.0
        out.put((rank, ok_all, ok_dst, ok_red, keys, sorted(set(owner))))
    finally:
        dist.destroy_process_group()


def test_sharded_state_gather_and_grad_reduce_two_ranks_gloo():
    """Sharder.gather_state completes every rank's (or one rank's) optimizer state from the
    owners, state_dict() keeps the reference's keys; reduce_grads averages each gradient
    onto its owner and leaves the others' local gradients alone."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_state_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120), q.get(timeout=120)])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_all, ok_dst, ok_red, keys, owners in res:
        assert owners == [0, 1]
        assert ok_all and ok_dst and ok_red, (rank, ok_all, ok_dst, ok_red)
        assert keys[:5] == [["momentum_buffer", "step"]] * 5
        assert keys[5:] == [["ema", "ema_squared", "step"]] * 3


def test_segments_cover_each_stack_in_order():
    """A shape stack is shared in consecutive, non-empty, ordered segments that cover every
    row exactly once, whatever count is asked for."""
    from muon_sr_b200.muon import _segments
    for n in (1, 2, 7, 64):
        for count in (0, 1, 3, 8, 100):
            segs = _segments(n, count)
            rows = [r for s in segs for r in s]
            assert rows == list(range(n))
            assert all(len(s) > 0 for s in segs)
            assert len(segs) == max(1, min(n, count))


def test_sharder_segment_counts():
    """About 4 ms of per-rank Newton-Schulz per segment, at least two matrices per rank per
    segment, at most 8 segments; small stacks stay whole."""
    class Fake(Sharder):
        def __init__(self, world, transport="p2p"):  # no process group needed for the arithmetic
            self.world = world
            self.transport = transport
    # the multicast transport has nothing to share between segments: whole stacks
    assert all(Fake(8, "multicast").segments(shape, 64) == 1 for shape in ((4096, 4096), (14336, 4096)))
    expect = {2: {(4096, 4096): 8, (1024, 4096): 1, (14336, 4096): 8, (4096, 14336): 8},
              8: {(4096, 4096): 2, (1024, 4096): 1, (14336, 4096): 4, (4096, 14336): 2}}
    counts = {(4096, 4096): 64, (1024, 4096): 64, (14336, 4096): 64, (4096, 14336): 32}
    for world, table in expect.items():
        sh = Fake(world)
        for shape, want in table.items():
            n = counts[shape]
            got = sh.segments(shape, n)
            assert got == want, (world, shape, got)
            assert got == 1 or n // got >= 2 * world


def _record_batched_step(rank, world, random_seeds, drop_grad=None, segments=None):
    """Run muon.muon_batch_step on CPU tensors with recording fakes in place of the CUDA
    kernels; returns (per-matrix apply seeds, prepare calls, share calls)."""
    import muon_sr_b200.muon as M
    shapes = [(8, 16)] * 6 + [(16, 8)] * 3 + [(4, 4)] * 2
    params = [torch.nn.Parameter(torch.zeros(*s, dtype=torch.bfloat16)) for s in shapes]
    for i, p in enumerate(params):
        p.grad = None if i == drop_grad else torch.zeros_like(p)
    state = {p: {} for p in params}
    stacks = M._MomentumStacks(params, state)
    log = {"apply": {}, "prepare": [], "share": []}
    names = {id(p): i for i, p in enumerate(params)}

    def prepare(items, beta, nesterov):
        log["prepare"].append([(int(ctr), int(seed)) for _, _, _, ctr, seed in items])

    def ns(x, steps):
        return torch.zeros_like(x)

    def apply(items, lr, wd):
        for p, _, _, seed in items:
            log["apply"][names[id(p)]] = int(seed)

    saved = (M.K.muon_prepare, M.K.newton_schulz, M.K.muon_apply)
    M.K.muon_prepare, M.K.newton_schulz, M.K.muon_apply = prepare, ns, apply
    try:
        owner = (lambda s, r: (s * 7 + r) % world == rank) if world > 1 else None
        share = (lambda ps: log["share"].append([names[id(p)] for p in ps])) if world > 1 else None
        torch.manual_seed(99)
        M.muon_batch_step(stacks, 0.95, True, 5, 0.02, 0.0, 7, M._Seeder(random_seeds),
                          M._Work(owner, share, segments))
    finally:
        M.K.muon_prepare, M.K.newton_schulz, M.K.muon_apply = saved
    return log


@pytest.mark.parametrize("random_seeds", [False, True])
@pytest.mark.parametrize("drop_grad", [None, 7])
def test_batched_step_sharding_logic(random_seeds, drop_grad):
    """Two simulated ranks together update every matrix exactly once, with the seed the
    single-process step uses (deterministic or drawn from torch's generator, also in the
    partial-gradient fallback), and call the share hook with the same sequence; segmented
    sharing changes neither."""
    single = _record_batched_step(0, 1, random_seeds, drop_grad)
    seg = (lambda shape, n: 2)
    for segments in (None, seg):
        logs = [_record_batched_step(r, 2, random_seeds, drop_grad, segments) for r in range(2)]
        merged = {}
        for lg in logs:
            assert not set(merged) & set(lg["apply"]), "a matrix was updated by both ranks"
            merged.update(lg["apply"])
        assert merged == single["apply"]
        assert logs[0]["share"] == logs[1]["share"]
        if segments is not None and drop_grad is None:
            assert len(logs[0]["share"]) > len(_record_batched_step(0, 2, random_seeds, drop_grad)["share"])
    if drop_grad is None:
        # prepare counters run over each whole stack (row r starts at r * numel) on every rank
        ctrs = sorted(c for lg in (_record_batched_step(r, 2, random_seeds) for r in range(2))
                      for call in lg["prepare"] for c, _ in call)
        assert ctrs == sorted(c for call in single["prepare"] for c, _ in call)


class _RecordingIO:
    """Stands in for a HostStaging: records the announcements of a step."""

    def __init__(self, log, names):
        self.log, self.names = log, names

    def need(self, params):
        self.log.append(("need", [self.names[id(p)] for p in params]))

    def done(self, params):
        self.log.append(("done", [self.names[id(p)] for p in params]))


def test_batched_step_staging_hooks(monkeypatch):
    """A batched Muon step announces each Newton-Schulz chunk: its gradients are needed before
    the chunk's prepare, and its weights are done after the chunk's apply; every matrix with a
    gradient is announced exactly once, and the prepare counters are those of the whole stack."""
    import muon_sr_b200.muon as M
    import muon_sr_b200.staging as S
    shapes = [(8, 16)] * 5 + [(16, 8)] * 3
    params = [torch.nn.Parameter(torch.zeros(*s, dtype=torch.bfloat16)) for s in shapes]
    for p in params:
        p.grad = torch.zeros_like(p)
    names = {id(p): i for i, p in enumerate(params)}
    stacks = M._MomentumStacks(params, {p: {} for p in params})
    log = []
    monkeypatch.setattr(M, "NS_CHUNK_NUMEL", 256)   # 2 matrices per chunk
    monkeypatch.setattr(M.K, "muon_prepare", lambda items, b, n: log.append(
        ("prepare", [int(ctr) for _, _, _, ctr, _ in items])))
    monkeypatch.setattr(M.K, "newton_schulz", lambda x, steps: torch.zeros_like(x))
    monkeypatch.setattr(M.K, "muon_apply", lambda items, lr, wd: log.append(
        ("apply", [names[id(p)] for p, _, _, _ in items])))
    monkeypatch.setattr(S._tls, "io", _RecordingIO(log, names), raising=False)
    M.muon_batch_step(stacks, 0.95, True, 5, 0.02, 0.0, 3, M._Seeder(False))
    kinds = [k for k, _ in log]
    assert kinds == ["need", "prepare", "apply", "done"] * 5   # chunks: 2+2+1 and 2+1 matrices
    needs = [v for k, v in log if k == "need"]
    assert needs == [v for k, v in log if k == "apply"] == [v for k, v in log if k == "done"]
    assert sorted(i for v in needs for i in v) == list(range(8))
    ctrs = [c for k, v in log if k == "prepare" for c in v]
    assert ctrs == [r * 128 for r in range(5)] + [r * 128 for r in range(3)]


@pytest.mark.parametrize("adam_first", [False, True])
def test_hybrid_staging_order(monkeypatch, adam_first):
    """Under HostStaging a deterministic-seed hybrid step runs its AdamW group once, right
    after the first Muon stack (so the AdamW weights download under the later stacks);
    without staging, and for the classes seeded from torch's generator, the group order
    stands."""
    import muon_sr_b200.muon as M
    import muon_sr_b200.staging as S
    from muon_sr_b200 import MuonSRWithAuxAdam, TritonMuonSRWithAuxAdam
    shapes = [(8, 16)] * 3 + [(16, 8)] * 2 + [(4,), (6,)]
    params = [torch.nn.Parameter(torch.zeros(*s, dtype=torch.bfloat16)) for s in shapes]
    for p in params:
        p.grad = torch.zeros_like(p)
    names = {id(p): i for i, p in enumerate(params)}
    log = []
    monkeypatch.setattr(M, "NS_CHUNK_NUMEL", 256)   # 2 matrices per chunk
    monkeypatch.setattr(M.K, "muon_prepare", lambda items, b, n: None)
    monkeypatch.setattr(M.K, "newton_schulz", lambda x, steps: torch.zeros_like(x))
    monkeypatch.setattr(M.K, "muon_apply", lambda items, lr, wd: None)
    import muon_sr_b200.adamw as A
    monkeypatch.setattr(A.K, "adamw_sr", lambda batch, *a: log.append(("adamw", [names[id(e[0])] for e in batch])))
    muon = dict(params=params[:5], use_muon=True, lr=0.02)
    adam = dict(params=params[5:], use_muon=False, lr=3e-4)

    def run(cls, staged):
        log.clear()
        opt = cls([adam, muon] if adam_first else [muon, adam], batch_ns=True)
        if staged:
            monkeypatch.setattr(S._tls, "io", _RecordingIO(log, names), raising=False)
        try:
            opt.step()
        finally:
            monkeypatch.setattr(S._tls, "io", None, raising=False)
        return [(k, v) for k, v in log if k != "need"]

    staged = run(TritonMuonSRWithAuxAdam, True)
    # first stack (3 matrices: chunks 2 + 1), then the AdamW group, then the second stack
    assert staged == [("done", [0, 1]), ("done", [2]), ("adamw", [5, 6]), ("done", [5, 6]),
                      ("done", [3, 4])]
    plain = run(TritonMuonSRWithAuxAdam, False)
    assert plain == [("adamw", [5, 6])]
    seeded = run(MuonSRWithAuxAdam, True)
    adam_at = seeded.index(("adamw", [5, 6]))
    assert adam_at == (0 if adam_first else len(seeded) - 2)
    assert [v for k, v in seeded if k == "adamw"] == [[5, 6]]


def test_staging_batches():
    """Launch batches are cut only while a staging step runs, at whole items."""
    import muon_sr_b200.staging as S
    items = [1 << 27, 1 << 27, 1 << 27, 1 << 29, 5]
    assert S.batches(items, lambda n: n) == [items]
    assert S.batches([], lambda n: n) == []
    S._tls.io = object()
    try:
        got = S.batches(items, lambda n: n)
    finally:
        S._tls.io = None
    assert got == [[1 << 27, 1 << 27], [1 << 27], [1 << 29], [5]]
    assert [x for b in got for x in b] == items


def test_step_graph_record_refresh():
    """A refresh rewrites a captured record's scalars (header and per-entry keys / scales)
    but keeps the captured pointers, and refuses a launch whose structure differs."""
    from muon_sr_b200 import _lib
    from muon_sr_b200 import graph as G
    m = G._Recorder("measure")
    arr = (_lib.ApplyEntry * 2)()
    arr[0].numel, arr[1].numel = 10, 20
    m.launch("msr_muon_apply_rec", _lib.ApplyRecord(0.5, 0.9, 2, 0), arr, None)
    esz = ctypes.sizeof(_lib.ApplyEntry)
    assert m.size == 16 + 2 * esz and len(m.plan) == 1
    host = torch.zeros(m.size, dtype=torch.uint8)
    cap = (_lib.ApplyEntry * 2)()
    cap[0].param, cap[0].update, cap[0].numel = 0x1000, 0x3000, 10
    cap[1].param, cap[1].update, cap[1].numel = 0x2000, 0x4000, 20
    plan = [G._Launch("msr_muon_apply_rec", 0, _lib.ApplyRecord(0.0, 0.0, 2, 0), cap)]
    new = (_lib.ApplyEntry * 2)()
    new[0].param, new[0].numel, new[0].key, new[0].scale = 0xDEAD, 10, 7, 1.5
    new[1].param, new[1].numel, new[1].key, new[1].scale = 0xBEEF, 20, 8, 2.0
    r = G._Recorder("refresh", host, None, plan=plan, constants=[])
    r.launch("msr_muon_apply_rec", _lib.ApplyRecord(0.25, 0.99, 2, 0), new, None)
    assert r.complete()
    raw = host.numpy().tobytes()
    hdr = _lib.ApplyRecord.from_buffer_copy(raw[:16])
    ents = (_lib.ApplyEntry * 2).from_buffer_copy(raw[16:16 + 2 * esz])
    assert (hdr.lr, hdr.count) == (0.25, 2)
    assert [(e.param, e.update, e.numel, e.key, e.scale) for e in ents] == \
        [(0x1000, 0x3000, 10, 7, 1.5), (0x2000, 0x4000, 20, 8, 2.0)]
    bad = (_lib.ApplyEntry * 1)()
    bad[0].numel = 10
    with pytest.raises(RuntimeError, match="captured graph"):
        G._Recorder("refresh", host, None, plan=plan, constants=[]).launch(
            "msr_muon_apply_rec", _lib.ApplyRecord(0.25, 0.99, 1, 0), bad, None)
    c = G._Recorder("refresh", host, None, plan=[], constants=[("centralization", 0.5)])
    with pytest.raises(RuntimeError, match="captured graph"):
        c.constant("centralization", 0.25)


def test_step_graph_snapshot_restore():
    """Passes that size or capture a step leave step counters, the global step and torch's
    generator as they found them; tensors in the state are the same objects."""
    from muon_sr_b200 import TritonMuonSR
    from muon_sr_b200 import graph as G
    p = torch.nn.Parameter(torch.zeros(4, 4, dtype=torch.bfloat16))
    opt = TritonMuonSR([p], batch_ns=True)
    buf = torch.zeros(4, 4, dtype=torch.bfloat16)
    opt.state[p].update(step=3, momentum_buffer=buf)
    opt._clock.value = 3
    snap = G._snapshot(opt)
    draw = torch.randint(0, 1 << 30, (1,)).item()
    opt.state[p]["step"] = 4
    opt.state[p]["extra"] = 1
    opt._clock.value = 4
    torch.randint(0, 1 << 30, (1,))
    G._restore(opt, snap)
    assert opt.state[p]["step"] == 3 and "extra" not in opt.state[p]
    assert opt.state[p]["momentum_buffer"] is buf and opt._clock.value == 3
    assert torch.randint(0, 1 << 30, (1,)).item() == draw
