"""The opt-in fast noise stream (``set_sr_noise("fast")``): every rounding kernel bit-exact
against the oracle's restatement of that stream, and the north-star SR gate (each output one
of the two bracketing bf16 values, mean over 256 seeds within 3 sigma of the fp32 value).
The default stream is the reference's; the golden-vector tests cover it.
"""
import numpy as np
import pytest
import torch

from muon_sr_b200 import kernels as K
from oracle import adamw8bit as o8
from oracle import elementwise as ew
from oracle.sr import bf16_to_f32, rne_bf16
from tests._golden import assert_bits_equal, bits_of, to_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def gpu(bits):
    return to_bf16(bits, DEV)


@pytest.fixture
def fast():
    K.set_sr_noise("fast")
    try:
        yield
    finally:
        K.set_sr_noise("reference")


def _bf16(rng, n, std):
    return rne_bf16((rng.standard_normal(n) * std).astype(np.float32))


def test_fast_noise_kernels_match_oracle(fast):
    rng = np.random.default_rng(11)
    for n in (8192 * 3 + 5, 1003, 16):
        acc, g = _bf16(rng, n, 1e-3), _bf16(rng, n, 1e-3)
        a = gpu(acc)
        K.grad_accum_(a, gpu(g), 77)
        assert_bits_equal(bits_of(a), ew.grad_accum(acc, g, 77, noise="fast"), f"grad_accum n={n}")

        p, u = _bf16(rng, n, 0.02), _bf16(rng, n, 0.1)
        pg = gpu(p)
        K.muon_apply([(pg, gpu(u), 1.5, 91)], 0.02, 0.01)
        assert_bits_equal(bits_of(pg), ew.muon_apply(p, u, 0.02, 0.01, 1.5, 91, noise="fast"), f"apply n={n}")

        m = _bf16(rng, n, 1e-3)
        v = rne_bf16(np.abs(rng.standard_normal(n) * 1e-6).astype(np.float32))
        pg, mg, vg = gpu(p), gpu(m), gpu(v)
        K.adamw_sr([(pg, gpu(g), mg, vg, 3, 5)], 3e-4, 0.9, 0.95, 1e-10, 0.01)
        wp, wm, wv = ew.adamw_sr(p, g, m, v, 3e-4, 0.9, 0.95, 1e-10, 0.01, 3, 5, noise="fast")
        assert_bits_equal(bits_of(pg), wp, f"adamw p n={n}")
        assert_bits_equal(bits_of(mg), wm, f"adamw m n={n}")
        assert_bits_equal(bits_of(vg), wv, f"adamw v n={n}")


def test_fast_noise_prepare_unaligned_stack_rows(fast):
    """Stack rows whose counters do not start on a multiple of 8 (numel 1003) and a base
    beyond 2^32: the fast stream uses 64-bit counters and straddles generator calls."""
    rng = np.random.default_rng(12)
    numel = 1003
    bases = [0, numel, 2 * numel, 5 * 2**32 + 11]
    gs = [_bf16(rng, numel, 1e-3) for _ in bases]
    bs = [_bf16(rng, numel, 1e-3) for _ in bases]
    bufs = [gpu(b) for b in bs]
    upds = [torch.empty_like(x) for x in bufs]
    K.muon_prepare([(gpu(g), b, u, base, 4242) for g, b, u, base in zip(gs, bufs, upds, bases)], 0.95, True)
    for g, b, buf, upd, base in zip(gs, bs, bufs, upds, bases):
        ob, ou = ew.muon_prepare(g, b, 0.95, True, 4242, ctr_base=base, noise="fast")
        assert_bits_equal(bits_of(buf), ob, f"momentum base {base}")
        assert_bits_equal(bits_of(upd), ou, f"update base {base}")


@pytest.mark.parametrize("quant,block", [(True, 256), (True, 4096), (False, 256)])
def test_fast_noise_adamw8bit_matches_oracle(fast, quant, block):
    rng = np.random.default_rng(13)
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
        K.adamw8bit([(tp, gpu(gg), ts1, ts2, ta1, ta2, step, 1234 + step, quant)], tq1, tq2, 1e-3, 0.9, 0.999,
                    1e-8, 0.01, block, qtables=K.quant_tables(tq1, tq2))
        p, s1, s2, a1, a2 = o8.adamw8bit(p, gg, s1, s2, a1, a2, q1, q2, 1e-3, 0.9, 0.999, 1e-8, 0.01, step,
                                         1234 + step, block, quant, noise="fast")
        assert_bits_equal(bits_of(tp), p, f"8-bit p step {step}")
        if quant:
            assert_bits_equal(ts1.cpu().numpy(), s1, "codes1")
            assert_bits_equal(ts2.cpu().numpy(), s2, "codes2")
        else:
            assert_bits_equal(bits_of(ts1), s1, "bf16 m")
            assert_bits_equal(bits_of(ts2), s2, "bf16 v")


def test_fast_noise_sr_statistics(fast):
    """North-star SR gate on the fast stream (AdamW p output): every output is one of the
    two bracketing bf16 values; the mean over 256 seeds is within 3 sigma of the fp32 value."""
    rng = np.random.default_rng(4)
    n = 4096
    p0 = _bf16(rng, n, 0.02)
    g = _bf16(rng, n, 1e-3)
    m0 = np.zeros(n, np.uint16)
    outs = []
    for s in range(256):
        p, m, v = gpu(p0), gpu(m0), gpu(m0)
        K.adamw_sr([(p, gpu(g), m, v, 1, s * 7919)], 3e-4, 0.9, 0.95, 1e-10, 0.0)
        outs.append(bf16_to_f32(bits_of(p)))
    outs = np.stack(outs).astype(np.float64)
    b1, omb1, b2, omb2, ss, bc2s, eps, decay = ew.adamw_coefficients(3e-4, 0.9, 0.95, 1e-10, 0.0, 1)
    gf, pf = bf16_to_f32(g), bf16_to_f32(p0)
    mm = (omb1 * gf).astype(np.float32)
    vv = ((omb2 * gf) * gf).astype(np.float32)
    x = (pf * decay - ss * mm / (np.sqrt(vv) / bc2s + eps)).astype(np.float32).astype(np.float64)
    xb = x.astype(np.float32).view(np.uint32)
    trunc = (xb & 0xFFFF0000).view(np.float32).astype(np.float64)
    ulp = np.abs((((xb & 0xFFFF0000) + 0x10000).astype(np.uint32)).view(np.float32) - trunc)
    other = trunc + np.sign(x) * ulp
    assert ((outs == trunc) | (outs == other)).all()
    frac = np.abs(x - trunc) / ulp
    sigma = ulp * np.sqrt(frac * (1 - frac) / 256) + 1e-30
    z = np.abs(outs.mean(0) - x) / sigma
    exact = frac == 0
    assert (z[~exact] < 3.0).mean() > 0.99
    assert np.all(outs.mean(0)[exact] == x[exact])


def test_reference_stream_is_restored():
    K.set_sr_noise("fast")
    K.set_sr_noise("reference")
    rng = np.random.default_rng(5)
    acc, g = _bf16(rng, 4096, 1e-3), _bf16(rng, 4096, 1e-3)
    a = gpu(acc)
    K.grad_accum_(a, gpu(g), 3)
    assert_bits_equal(bits_of(a), ew.grad_accum(acc, g, 3), "reference stream")
    with pytest.raises(ValueError):
        K.set_sr_noise("xoshiro")
