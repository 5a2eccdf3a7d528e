"""HostStaging: optimizer steps fed from pinned host memory, copies overlapped with the step.

Each case runs twin parameter sets from the same initial weights: one through the plain
``p.grad = g.cuda(); opt.step(); p.cpu()`` sequence, one through ``HostStaging``, with the
launch batches cut small so that every step has several uploads and downloads in flight.
Weights, host copies and optimizer state must agree bit for bit. One AdamW tensor is large
(128 MiB) so that a missing stream dependency (an update reading a gradient still being
uploaded, a download taken before the update) would show up as a mismatch."""
import pytest
import torch

import muon_sr_b200.muon as M
import muon_sr_b200.staging as S
from muon_sr_b200 import (HostStaging, MuonSRWithAuxAdam, TritonAdamW, TritonAdamW8bit, TritonMuonSR,
                          TritonMuonSRWithAuxAdam)

pytestmark = pytest.mark.gpu
DEV = "cuda"
MUON = [(24, 40)] * 5 + [(40, 24)] * 3 + [(16, 16)] * 2
ADAM = [(30, 16), (16,), (8192, 8192), (16,)]


def _bits(t):
    return t.detach().contiguous().view(torch.int16)


def _init(shapes, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(s, generator=g) * 0.02).to(torch.bfloat16) for s in shapes]


def _grads(shapes, seed, drop):
    g = torch.Generator().manual_seed(seed)
    return [None if i in drop else (torch.randn(s, generator=g) * 1e-3).to(torch.bfloat16)
            for i, s in enumerate(shapes)]


def _run(make_opt, shapes, drop=(), steps=3, random_seeds=False):
    init = _init(shapes, 0)
    pa = [torch.nn.Parameter(t.to(DEV)) for t in init]
    pb = [torch.nn.Parameter(t.to(DEV)) for t in init]
    opt_a, opt_b = make_opt(pa), make_opt(pb)
    host_g = [None if i in drop else torch.empty(s, dtype=torch.bfloat16).pin_memory() for i, s in enumerate(shapes)]
    host_p = [torch.empty(s, dtype=torch.bfloat16).pin_memory() for s in shapes]
    stg = HostStaging(opt_b, pb, host_g, host_p)
    for step in range(steps):
        grads = _grads(shapes, 100 + step, drop)
        for p, g in zip(pa, grads):
            p.grad = None if g is None else g.to(DEV)
        if random_seeds:
            torch.manual_seed(step)
        opt_a.step()
        for h, g in zip(host_g, grads):
            if h is not None:
                h.copy_(g)
        if random_seeds:
            torch.manual_seed(step)
        stg.step()
        stg.synchronize()
        want_h2d = sum(g.numel() * 2 for g in grads if g is not None)
        assert stg.h2d_bytes == want_h2d
        assert stg.d2h_bytes == want_h2d
        for i, (a, b) in enumerate(zip(pa, pb)):
            assert torch.equal(_bits(a), _bits(b)), ("weights", step, i)
            if i not in drop:
                assert torch.equal(_bits(a).cpu(), _bits(host_p[i])), ("host copy", step, i)
    for a, b in zip(pa, pb):
        sa, sb = opt_a.state[a], opt_b.state[b]
        assert sa.keys() == sb.keys()
        for k in sa:
            if torch.is_tensor(sa[k]):
                assert torch.equal(sa[k].view(torch.uint8), sb[k].view(torch.uint8)), k
            else:
                assert sa[k] == sb[k], k


@pytest.fixture
def small_batches(monkeypatch):
    monkeypatch.setattr(M, "NS_CHUNK_NUMEL", 2 * 24 * 40)   # 2 matrices per Newton-Schulz chunk
    monkeypatch.setattr(S, "BATCH_NUMEL", 1024)             # AdamW batches of one or two tensors


@pytest.mark.parametrize("batch_ns", [True, False])
@pytest.mark.parametrize("drop", [(), (3,)])
def test_hybrid_staged(small_batches, batch_ns, drop):
    shapes = MUON + ADAM
    nm = len(MUON)

    def make(params):
        return TritonMuonSRWithAuxAdam([
            dict(params=params[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=params[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=batch_ns)
    _run(make, shapes, drop)


def test_random_seed_hybrid_staged(small_batches):
    shapes = MUON + ADAM[:2]
    nm = len(MUON)

    def make(params):
        return MuonSRWithAuxAdam([
            dict(params=params[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=params[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=True)
    _run(make, shapes, random_seeds=True)


def test_muon_single_staged(small_batches):
    _run(lambda params: TritonMuonSR(params, lr=0.02, weight_decay=0.01, batch_ns=False), MUON, drop=(1,))


def test_adamw_centralized_staged(small_batches):
    _run(lambda params: TritonAdamW(params, lr=1e-3, weight_decay=0.01, centralization=0.5), ADAM)


def test_adamw8bit_staged(small_batches):
    shapes = [(64, 256), (128,), (64, 256), (4096, 4096), (33, 129)]
    _run(lambda params: TritonAdamW8bit(params, lr=1e-3, weight_decay=0.01, block_size=256), shapes)


def test_staging_argument_errors():
    p = torch.nn.Parameter(torch.zeros(4, 8, dtype=torch.bfloat16, device=DEV))
    pinned = torch.zeros(4, 8, dtype=torch.bfloat16).pin_memory()
    with pytest.raises(TypeError):
        HostStaging(torch.optim.SGD([p], lr=0.1), [p], [pinned])
    opt = TritonAdamW([p])
    with pytest.raises(ValueError, match="pinned"):
        HostStaging(opt, [p], [torch.zeros(4, 8, dtype=torch.bfloat16)])
    with pytest.raises(ValueError, match="shape"):
        HostStaging(opt, [p], [torch.zeros(8, 4, dtype=torch.bfloat16).pin_memory()])
    with pytest.raises(ValueError, match="one entry"):
        HostStaging(opt, [p], [pinned, pinned])
    with pytest.raises(ValueError, match="bfloat16"):
        HostStaging(opt, [p], [torch.zeros(4, 8, dtype=torch.float32).pin_memory()])
