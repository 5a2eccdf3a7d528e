"""StepGraph: whole optimizer steps captured once as CUDA graphs and replayed.

Twin optimizers from the same weights take the same gradients: one steps eagerly, the other
replays its captured graph (after the one eager step a capture needs). Weights and optimizer
state must agree bit for bit after every step, also when the learning rate changes between
replays, with seeds drawn from torch's generator, with several Newton-Schulz chunks per stack
and with gradient centralisation; a step whose structure changed is refused."""
import pytest
import torch

import muon_sr_b200.muon as M
from muon_sr_b200 import (MuonSRWithAuxAdam, StepGraph, TritonAdamW, TritonAdamW8bit, TritonMuonSR,
                          TritonMuonSRWithAuxAdam)

pytestmark = pytest.mark.gpu
DEV = "cuda"
MUON = [(24, 40)] * 5 + [(40, 24)] * 3 + [(16, 16)] * 2
ADAM = [(30, 16), (16,), (4096, 512), (16,)]


def _bits(t):
    return t.detach().contiguous().view(torch.int16)


def _twins(shapes, seed=0):
    g = torch.Generator().manual_seed(seed)
    init = [(torch.randn(s, generator=g) * 0.02).to(torch.bfloat16) for s in shapes]
    a = [torch.nn.Parameter(t.to(DEV)) for t in init]
    b = [torch.nn.Parameter(t.to(DEV)) for t in init]
    for p in a + b:
        p.grad = torch.empty_like(p)
    return a, b


def _fill(grads_a, grads_b, shapes, seed):
    g = torch.Generator().manual_seed(seed)
    for ga, gb, s in zip(grads_a, grads_b, shapes):
        x = (torch.randn(s, generator=g) * 1e-3).to(torch.bfloat16)
        ga.copy_(x)
        gb.copy_(x)


def _same(pa, pb, opt_a, opt_b, what):
    for i, (a, b) in enumerate(zip(pa, pb)):
        assert torch.equal(_bits(a), _bits(b)), (what, "weights", i)
        sa, sb = opt_a.state[a], opt_b.state[b]
        assert sa.keys() == sb.keys(), (what, i)
        for k in sa:
            if torch.is_tensor(sa[k]):
                assert torch.equal(sa[k].view(torch.uint8), sb[k].view(torch.uint8)), (what, k, i)
            else:
                assert sa[k] == sb[k], (what, k, i)


def _run(make, shapes, steps=4, random_seeds=False, lr_change=None, after_capture=None):
    pa, pb = _twins(shapes)
    opt_a, opt_b = make(pa), make(pb)
    ga, gb = [p.grad for p in pa], [p.grad for p in pb]
    _fill(ga, gb, shapes, 100)
    for opt in (opt_a, opt_b):          # the eager step a capture needs
        if random_seeds:
            torch.manual_seed(7)
        opt.step()
    _same(pa, pb, opt_a, opt_b, "eager")
    graph = StepGraph(opt_b)
    _same(pa, pb, opt_a, opt_b, "after capture")  # capturing does not step
    if after_capture is not None:
        after_capture()
    for step in range(steps):
        _fill(ga, gb, shapes, 200 + step)
        if lr_change is not None and step == 2:
            lr_change(opt_a)
            lr_change(opt_b)
        if random_seeds:
            torch.manual_seed(step)
        opt_a.step()
        if random_seeds:
            torch.manual_seed(step)
        graph.step()
        torch.cuda.synchronize()
        _same(pa, pb, opt_a, opt_b, f"replay {step}")
    return graph, opt_b, pb


@pytest.fixture
def small_chunks(monkeypatch):
    monkeypatch.setattr(M, "NS_CHUNK_NUMEL", 2 * 24 * 40)   # 2 matrices per Newton-Schulz chunk


def _halve_lr(opt):
    for g in opt.param_groups:
        g["lr"] *= 0.5


@pytest.mark.parametrize("batch_ns", [True, False])
def test_hybrid_graph_matches_eager(small_chunks, batch_ns):
    nm = len(MUON)

    def make(params):
        return TritonMuonSRWithAuxAdam([
            dict(params=params[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=params[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=batch_ns)
    _run(make, MUON + ADAM, lr_change=_halve_lr)


def test_graph_keeps_its_workspaces_when_eager_calls_grow_them(small_chunks):
    """Newton-Schulz scratch a captured graph writes to stays the graph's: after capture, larger
    eager Newton-Schulz calls on the side streams and on the current stream replace those
    streams' workspaces; tensors allocated afterwards on the same streams (where the caching
    allocator would hand out a freed workspace block) must not be touched by the replays, and
    the replays still give the eager steps' bits."""
    import muon_sr_b200.kernels as KK
    nm = len(MUON)
    fillers = []

    def make(params):
        return TritonMuonSRWithAuxAdam([
            dict(params=params[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=params[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=True)

    def grow():
        dev = torch.device(DEV, torch.cuda.current_device())
        streams = list(M._side_streams(dev)[0]) + [torch.cuda.current_stream(dev)]
        big = (torch.randn(2, 512, 768, device=DEV) * 1e-3).bfloat16()
        for s in streams:
            s.wait_stream(torch.cuda.current_stream(dev))
            old = KK._workspaces.get((dev.index, s.cuda_stream))
            size = old.numel() if old is not None else 1 << 20
            with torch.cuda.stream(s):
                KK.newton_schulz(big, 5)     # grows (replaces) this stream's workspace
                del old
                for _ in range(4):           # candidates for the freed block
                    fillers.append(torch.full((size,), 0x5A, dtype=torch.uint8, device=DEV))
            torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()

    _run(make, MUON + ADAM, after_capture=grow)
    torch.cuda.synchronize()
    for f in fillers:
        assert bool((f == 0x5A).all()), "a replay wrote into memory the graph no longer owns"


def test_random_seed_hybrid_graph_matches_eager(small_chunks):
    nm = len(MUON)

    def make(params):
        return MuonSRWithAuxAdam([
            dict(params=params[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=params[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=True)
    _run(make, MUON + ADAM[:2], random_seeds=True)


def test_adamw_centralized_graph_matches_eager():
    graph, opt, params = _run(lambda ps: TritonAdamW(ps, lr=1e-3, weight_decay=0.01, centralization=0.5), ADAM,
                              lr_change=_halve_lr)
    # a constant baked into the graph (the centralisation strength) may not change
    opt.param_groups[0]["centralization"] = 0.25
    before = {p: dict(opt.state[p]) for p in params}
    with pytest.raises(RuntimeError, match="captured graph"):
        graph.step()
    assert all(opt.state[p]["step"] == before[p]["step"] for p in params)  # a refused step is undone


def test_graph_refuses_changed_structure(small_chunks):
    graph, opt, params = _run(lambda ps: TritonMuonSR(ps, lr=0.02, weight_decay=0.01, batch_ns=True), MUON, steps=1)
    params[0].grad = torch.zeros_like(params[0])     # another tensor behind a .grad
    with pytest.raises(RuntimeError, match="captured graph"):
        graph.step()
    graph, opt, params = _run(lambda ps: TritonMuonSR(ps, lr=0.02, weight_decay=0.01, batch_ns=True), MUON, steps=1)
    opt.load_state_dict(opt.state_dict())            # new state tensors: the graph's pointers are stale
    with pytest.raises(RuntimeError, match="captured graph"):
        graph.step()


def test_graph_argument_errors():
    p = torch.nn.Parameter(torch.zeros(64, 64, dtype=torch.bfloat16, device=DEV))
    p.grad = torch.zeros_like(p)
    with pytest.raises(TypeError):
        StepGraph(TritonAdamW8bit([p]))
    with pytest.raises(RuntimeError, match="eager"):
        StepGraph(TritonMuonSR([p]))


@pytest.mark.parametrize("batch_ns,fname", [(True, "traj_hybrid_batch.npz"), (False, "traj_hybrid_nobatch.npz")])
def test_graph_replays_follow_reference_trajectory(batch_ns, fname):
    """Replayed steps against the reference's own hybrid trajectories (golden vectors from
    muon_sr's TritonMuonSRWithAuxAdam, muon_sr/triton_muon_sr.py:258-373): step 0 runs eagerly
    (a capture needs one), steps 1 and 3 are replays of the captured graph, step 2 -- where two
    parameters have no gradient, a structure the graph refuses -- runs eagerly. Every step is
    checked with the eager trajectory test's gates (momentum, AdamW tensors and step counters
    bit-exact)."""
    from tests._golden import bits_of, load, to_bf16
    from tests.test_optim_gpu import check_hybrid_step, hybrid_from_golden
    d = load(fname)
    params, opt = hybrid_from_golden(d, batch_ns)
    grads = [torch.empty_like(p) for p in params]  # the tensors behind .grad, kept for the replays
    graph = None
    replays = 0
    for step in range(4):
        mine_prev = [bits_of(p).ravel() for p in params]
        full = all(d[f"g{step}_{i}"].size for i in range(len(params)))
        for i, p in enumerate(params):
            g = d[f"g{step}_{i}"]
            if g.size:
                grads[i].copy_(to_bf16(g, DEV).view(p.shape))
                p.grad = grads[i]
            else:
                p.grad = None
        if graph is not None and full:
            graph.step()
            replays += 1
        else:
            opt.step()
        torch.cuda.synchronize()
        check_hybrid_step(d, step, params, opt, mine_prev)
        if graph is None:
            graph = StepGraph(opt)
    assert replays == 2


def test_graph_adamw_replays_follow_reference_trajectory():
    """TritonAdamW with centralisation (muon_sr/triton_adamw.py:130-203): step 0 eager, steps 1
    and 2 replayed, each against the reference's golden trajectory (1 ulp on < 5% of elements,
    as the eager test allows for the fp32 mean's last bit)."""
    from tests._golden import bits_of, load, to_bf16
    from tests.test_optim_gpu import _ulp_diff
    d = load("traj_adamw_central.npz")
    shapes = [(12, 20), (20,)]
    params = [torch.nn.Parameter(to_bf16(d[f"init_{i}"], DEV).view(*s)) for i, s in enumerate(shapes)]
    grads = [torch.empty_like(p) for p in params]
    opt = TritonAdamW(params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, centralization=0.5)
    graph = None
    for step in range(3):
        for i, p in enumerate(params):
            grads[i].copy_(to_bf16(d[f"g{step}_{i}"], DEV).view(p.shape))
            p.grad = grads[i]
        (graph.step if graph is not None else opt.step)()
        torch.cuda.synchronize()
        for i, p in enumerate(params):
            for got, want in ((bits_of(p), d[f"p{step}_{i}"]), (bits_of(opt.state[p]["ema"]), d[f"ema{step}_{i}"])):
                ud = _ulp_diff(got.ravel(), want.ravel())
                assert ud.max() <= 1.0 + 1e-9 and (ud > 0).mean() < 0.05, (step, i, ud.max())
        if graph is None:
            graph = StepGraph(opt)

