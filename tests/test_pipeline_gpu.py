"""Pipelined chunk loop (``muon.PIPELINE_CHUNKS``): the prepare of the next Newton-Schulz
chunk and the apply of the previous one run on a second stream. The bits must equal the
sequential loop's -- eagerly, replayed from a StepGraph and under HostStaging."""
import pytest
import torch

import muon_sr_b200.muon as M
from muon_sr_b200 import HostStaging, StepGraph, TritonMuonSRWithAuxAdam
from tests.test_graph_gpu import _fill, _same, _twins

pytestmark = pytest.mark.gpu
MUON = [(64, 96)] * 7 + [(96, 64)] * 5
ADAM = [(30, 16), (16,)]
SHAPES = MUON + ADAM


@pytest.fixture
def chunked(monkeypatch):
    monkeypatch.setattr(M, "NS_CHUNK_NUMEL", 2 * 64 * 96)  # 2 matrices per chunk: 4 and 3 chunks
    monkeypatch.setattr(M, "CONCURRENT_MAX_DIM", 0)        # every stack on the step's stream
    return monkeypatch


def _make(params):
    nm = len(MUON)
    return TritonMuonSRWithAuxAdam([
        dict(params=params[:nm], use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
        dict(params=params[nm:], use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
    ], batch_ns=True)


def _step(mp, opt, pipelined):
    mp.setattr(M, "PIPELINE_CHUNKS", pipelined)
    opt.step()


def test_pipelined_chunks_equal_sequential(chunked):
    pa, pb = _twins(SHAPES)
    oa, ob = _make(pa), _make(pb)
    for step in range(3):
        _fill([p.grad for p in pa], [p.grad for p in pb], SHAPES, 300 + step)
        _step(chunked, oa, False)
        _step(chunked, ob, True)
        torch.cuda.synchronize()
        _same(pa, pb, oa, ob, f"step {step}")


def test_pipelined_chunks_in_graph(chunked):
    pa, pb = _twins(SHAPES)
    oa, ob = _make(pa), _make(pb)
    _fill([p.grad for p in pa], [p.grad for p in pb], SHAPES, 400)
    _step(chunked, oa, False)
    _step(chunked, ob, True)
    chunked.setattr(M, "PIPELINE_CHUNKS", True)
    graph = StepGraph(ob)
    for step in range(3):
        _fill([p.grad for p in pa], [p.grad for p in pb], SHAPES, 500 + step)
        _step(chunked, oa, False)
        chunked.setattr(M, "PIPELINE_CHUNKS", True)
        graph.step()
        torch.cuda.synchronize()
        _same(pa, pb, oa, ob, f"replay {step}")


def test_pipelined_chunks_under_staging(chunked):
    pa, pb = _twins(SHAPES)
    oa, ob = _make(pa), _make(pb)
    host_g = [torch.empty(s, dtype=torch.bfloat16).pin_memory() for s in SHAPES]
    host_p = [torch.empty(s, dtype=torch.bfloat16).pin_memory() for s in SHAPES]
    staged = HostStaging(ob, pb, host_g, host_p)
    for step in range(3):
        _fill([p.grad for p in pa], host_g, SHAPES, 600 + step)
        _step(chunked, oa, False)
        chunked.setattr(M, "PIPELINE_CHUNKS", True)
        staged.step()
        staged.synchronize()
        _same(pa, pb, oa, ob, f"staged {step}")
        for a, h in zip(pa, host_p):
            assert torch.equal(a.detach().cpu().view(torch.int16), h.view(torch.int16))
