"""Round-to-nearest parity mode (``set_sr_noise("none")``): every SR store rounds to the
nearest bf16 instead, which isolates the fp32 arithmetic of the updates from the noise.

The north-star gate "with SR swapped for round-to-nearest, updates within 1 bf16 ulp" is
checked two ways: every rounding kernel bit-exact against the oracle's fp32 restatement of
the reference's formulas cast to bf16, and whole optimizer steps through the public API
within 1 ulp of the same formulas written as torch fp32 ops on the GPU.
"""
import numpy as np
import pytest
import torch

from muon_sr_b200 import TritonAdamW, TritonMuonSR
from muon_sr_b200 import kernels as K
from oracle import adamw8bit as o8
from oracle import elementwise as ew
from oracle.sr import rne_bf16
from tests._golden import assert_bits_equal, bits_of, to_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def gpu(bits):
    return to_bf16(bits, DEV)


@pytest.fixture
def rtn():
    K.set_sr_noise("none")
    try:
        yield
    finally:
        K.set_sr_noise("reference")


def _bf16(rng, n, std):
    return rne_bf16((rng.standard_normal(n) * std).astype(np.float32))


def _ulps(a, b):
    """Distance in bf16 ulps between two bf16 tensors (ordered sign-magnitude bits)."""
    def key(t):
        u = t.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        return torch.where(u >= 0x8000, -(u & 0x7FFF), u)
    return (key(a) - key(b)).abs()


def test_rtn_kernels_match_oracle(rtn):
    rng = np.random.default_rng(21)
    for n in (8192 * 3 + 5, 1003, 16):
        acc, g = _bf16(rng, n, 1e-3), _bf16(rng, n, 1e-3)
        a = gpu(acc)
        K.grad_accum_(a, gpu(g), 77)
        assert_bits_equal(bits_of(a), ew.grad_accum(acc, g, 77, noise="none"), f"grad_accum n={n}")

        p, u = _bf16(rng, n, 0.02), _bf16(rng, n, 0.1)
        pg = gpu(p)
        K.muon_apply([(pg, gpu(u), 1.5, 91)], 0.02, 0.01)
        assert_bits_equal(bits_of(pg), ew.muon_apply(p, u, 0.02, 0.01, 1.5, 91, noise="none"), f"apply n={n}")

        m = _bf16(rng, n, 1e-3)
        v = rne_bf16(np.abs(rng.standard_normal(n) * 1e-6).astype(np.float32))
        pg, mg, vg = gpu(p), gpu(m), gpu(v)
        K.adamw_sr([(pg, gpu(g), mg, vg, 3, 5)], 3e-4, 0.9, 0.95, 1e-10, 0.01)
        wp, wm, wv = ew.adamw_sr(p, g, m, v, 3e-4, 0.9, 0.95, 1e-10, 0.01, 3, 5, noise="none")
        assert_bits_equal(bits_of(pg), wp, f"adamw p n={n}")
        assert_bits_equal(bits_of(mg), wm, f"adamw m n={n}")
        assert_bits_equal(bits_of(vg), wv, f"adamw v n={n}")

        bufs, upd = gpu(m), torch.empty(n, dtype=torch.bfloat16, device=DEV)
        K.muon_prepare([(gpu(g), bufs, upd, 3 * n, 4242)], 0.95, True)
        ob, ou = ew.muon_prepare(g, m, 0.95, True, 4242, ctr_base=3 * n, noise="none")
        assert_bits_equal(bits_of(bufs), ob, f"prepare momentum n={n}")
        assert_bits_equal(bits_of(upd), ou, f"prepare update n={n}")


@pytest.mark.parametrize("quant,block", [(True, 256), (True, 4096), (False, 256)])
def test_rtn_adamw8bit_matches_oracle(rtn, quant, block):
    rng = np.random.default_rng(23)
    n = 3 * block + 77 if quant else 5000
    p, g = _bf16(rng, n, 0.02), _bf16(rng, n, 1e-3)
    q1, q2 = o8.create_dynamic_map(True), o8.create_dynamic_map(False)
    nblk = (n + block - 1) // block
    if quant:
        s1, s2 = np.full(n, 127, np.uint8), np.zeros(n, np.uint8)
        a1, a2 = np.zeros(nblk, np.float32), np.zeros(nblk, np.float32)
        ts1, ts2 = torch.from_numpy(s1).to(DEV), torch.from_numpy(s2).to(DEV)
        ta1, ta2 = torch.from_numpy(a1).to(DEV), torch.from_numpy(a2).to(DEV)
    else:
        s1, s2 = np.zeros(n, np.uint16), np.zeros(n, np.uint16)
        a1 = a2 = None
        ts1, ts2 = gpu(s1), gpu(s2)
        ta1 = ta2 = None
    tq1, tq2 = torch.from_numpy(q1).to(DEV), torch.from_numpy(q2).to(DEV)
    tp = gpu(p)
    for step in (1, 2):
        gg = g if step == 1 else _bf16(rng, n, 1e-3)
        K.adamw8bit([(tp, gpu(gg), ts1, ts2, ta1, ta2, step, 99 + step, quant)], tq1, tq2, 1e-3, 0.9, 0.999,
                    1e-8, 0.01, block, qtables=K.quant_tables(tq1, tq2))
        p, s1, s2, a1, a2 = o8.adamw8bit(p, gg, s1, s2, a1, a2, q1, q2, 1e-3, 0.9, 0.999, 1e-8, 0.01, step,
                                         99 + step, block, quant, noise="none")
        assert_bits_equal(bits_of(tp), p, f"8-bit p step {step}")
        if quant:
            assert_bits_equal(ts1.cpu().numpy(), s1, "codes1")
            assert_bits_equal(ts2.cpu().numpy(), s2, "codes2")
        else:
            assert_bits_equal(bits_of(ts1), s1, "bf16 m")
            assert_bits_equal(bits_of(ts2), s2, "bf16 v")


def _f32(x):
    return torch.tensor(float(np.float32(x)), dtype=torch.float32, device=DEV)


def test_rtn_adamw_steps_within_one_ulp_of_torch(rtn):
    """TritonAdamW steps against the reference's update (muon_sr/triton_adamw.py:37-72) as
    torch fp32 ops cast to bf16: weights and both moments within 1 ulp after every step."""
    torch.manual_seed(0)
    shapes = [(257, 129), (4096,), (3, 5, 7)]
    lr, (b1, b2), eps, wd = 1e-3, (0.9, 0.95), 1e-8, 0.01
    params = [torch.nn.Parameter((torch.randn(s, device=DEV) * 0.02).to(torch.bfloat16)) for s in shapes]
    opt = TritonAdamW(params, lr=lr, betas=(b1, b2), eps=eps, weight_decay=wd)
    ref = [(p.detach().clone(), torch.zeros_like(p), torch.zeros_like(p)) for p in params]
    for step in range(1, 4):
        grads = [(torch.randn(s, device=DEV) * 1e-3).to(torch.bfloat16) for s in shapes]
        for p, g in zip(params, grads):
            p.grad = g
        opt.step()
        new_ref = []
        for (rp, rm, rv), g in zip(ref, grads):
            gf = g.float()
            m = _f32(b1) * rm.float() + _f32(1 - b1) * gf
            v = _f32(b2) * rv.float() + (_f32(1 - b2) * gf) * gf
            denom = torch.sqrt(v) / _f32((1 - b2 ** step) ** 0.5) + _f32(eps)
            p = rp.float() * _f32(1 - lr * wd)
            p = p - (_f32(lr / (1 - b1 ** step)) * m) / denom
            new_ref.append((p.to(torch.bfloat16), m.to(torch.bfloat16), v.to(torch.bfloat16)))
        ref = new_ref
        for i, (p, (rp, rm, rv)) in enumerate(zip(params, ref)):
            st = opt.state[p]
            assert int(_ulps(p.detach(), rp).max()) <= 1, ("p", step, i)
            assert int(_ulps(st["ema"], rm).max()) <= 1, ("m", step, i)
            assert int(_ulps(st["ema_squared"], rv).max()) <= 1, ("v", step, i)
            # keep the reference on the engine's bits so that the next step compares one update
            ref[i] = (p.detach().clone(), st["ema"].clone(), st["ema_squared"].clone())


@pytest.mark.parametrize("shape", [(96, 64), (64, 160)])
def test_rtn_muon_step_within_one_ulp_of_torch(rtn, shape):
    """TritonMuonSR steps against the reference's prepare and apply (triton_muon_sr.py:18-80)
    as torch fp32 ops cast to bf16, around the engine's Newton-Schulz of the same update:
    momentum and weights within 1 ulp after every step."""
    torch.manual_seed(1)
    lr, wd, beta = 0.02, 0.01, 0.95
    p = torch.nn.Parameter((torch.randn(shape, device=DEV) * 0.02).to(torch.bfloat16))
    opt = TritonMuonSR([p], lr=lr, weight_decay=wd, momentum=beta, nesterov=True, ns_steps=5)
    buf = torch.zeros_like(p)
    scale = max(1.0, shape[0] / shape[1]) ** 0.5
    for step in range(3):
        g = (torch.randn(shape, device=DEV) * 1e-3).to(torch.bfloat16)
        p.grad = g
        p0 = p.detach().clone()
        opt.step()
        gf, bf = g.float(), buf.float()
        nb = bf + _f32(1 - beta) * (gf - bf)
        upd = (gf + _f32(beta) * (nb - gf)).to(torch.bfloat16)
        ns = K.newton_schulz(upd.unsqueeze(0), 5)[0]
        want = p0.float() * _f32(1 - lr * wd) - _f32(lr) * (ns.float() * _f32(scale))
        mom = opt.state[p]["momentum_buffer"]
        assert int(_ulps(mom, nb.to(torch.bfloat16)).max()) <= 1, ("momentum", step)
        assert int(_ulps(p.detach(), want.to(torch.bfloat16)).max()) <= 1, ("weights", step)
        buf = mom.clone()
