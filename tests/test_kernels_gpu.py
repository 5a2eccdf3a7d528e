"""Elementwise and 8-bit kernels through the C ABI on the GPU, against the reference's golden
vectors (bit-exact) and the CPU oracle (ragged, multi-tensor, unaligned and large-counter
cases), plus the stochastic-rounding statistics the north-star gates on."""
import numpy as np
import pytest
import torch

from muon_sr_b200 import kernels as K
from muon_sr_b200.seeds import deterministic_seed, triton_key
from oracle import adamw8bit as o8
from oracle import elementwise as ew
from oracle.philox import philox_randint
from oracle.sr import bf16_to_f32, rne_bf16
from tests._golden import assert_bits_equal, bits_of, load, to_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def gpu(bits):
    return to_bf16(bits, DEV)


def test_philox_matches_golden():
    d = load("philox.npz")
    for i, s in enumerate(d["seeds"].tolist()):
        for add in range(3):
            for j, b in enumerate(d["bases"].tolist()):
                got = K.philox_fill(32, int(b), triton_key(int(s), add), DEV).cpu().numpy().view(np.uint32)
                assert_bits_equal(got, d["words"][i, add, j], f"seed {s} add {add} base {b}")


def test_philox_large_launch_matches_oracle():
    n = 1 << 20
    got = K.philox_fill(n, 2**32 - 1000, 0x123456789ABC, DEV).cpu().numpy().view(np.uint32)
    ctr = (np.arange(n, dtype=np.uint64) + np.uint64(2**32 - 1000)) & np.uint64(0xFFFFFFFF)
    assert_bits_equal(got, philox_randint(0x123456789ABC, ctr), "philox 1M")


def test_grad_accum_golden():
    d = load("grad_accum.npz")
    for k, s in enumerate(d["seeds"].tolist()):
        acc = gpu(d["acc"])
        K.grad_accum_(acc, gpu(d["grad"]), int(s))
        assert_bits_equal(bits_of(acc), d["out"][k], "grad_accum")


def test_grad_accum_first_is_zero_fill_plus_accumulate():
    g = torch.randn(10007, device=DEV).bfloat16()
    g[::97] = -0.0
    acc = torch.full_like(g, 3.0)
    K.grad_accum_(acc, g, 1234, first=True)
    ref = torch.zeros_like(g)
    K.grad_accum_(ref, g, 1234)
    assert_bits_equal(bits_of(acc), bits_of(ref), "first micro-batch")


@pytest.mark.parametrize("offset", [0, 3])
def test_grad_accum_ragged_unaligned(offset):
    rng = np.random.default_rng(1)
    n = 8192 * 3 + 13
    a = (rng.standard_normal(n + 8) * 1e-3).astype(np.float32)
    b = (rng.standard_normal(n + 8) * 1e-3).astype(np.float32)
    ab, bb = rne_bf16(a), rne_bf16(b)
    acc = gpu(ab)[offset:offset + n]
    K.grad_accum_(acc, gpu(bb)[offset:offset + n], 77)
    assert_bits_equal(bits_of(acc), ew.grad_accum(ab[offset:offset + n], bb[offset:offset + n], 77), "ragged")


@pytest.mark.parametrize("nest", [0, 1])
def test_muon_prepare_golden(nest):
    d = load("muon_prepare.npz")
    for k, s in enumerate(d["seeds"].tolist()):
        buf = gpu(d["buf"])
        upd = torch.empty_like(buf)
        K.muon_prepare([(gpu(d["grad"]), buf, upd, 0, int(s))], float(d["beta"]), bool(nest))
        assert_bits_equal(bits_of(buf), d[f"buf_{nest}_{k}"], "momentum")
        obuf, oupd = ew.muon_prepare(d["grad"], d["buf"], float(d["beta"]), bool(nest), int(s))
        assert_bits_equal(bits_of(upd), oupd, "update (RNE)")


def test_muon_prepare_stack_counters_and_multi_entry():
    """Stacked prepare: counters run over the whole stack (ctr_base = i * numel), including
    a base beyond 2^32 that must wrap like the reference's int32 cast."""
    rng = np.random.default_rng(2)
    numel = 5000
    bases = [0, numel, 2 * numel, 2**32 - 3000, 5 * 2**32 + 11]
    gs = [rne_bf16((rng.standard_normal(numel) * 1e-3).astype(np.float32)) for _ in bases]
    bs = [rne_bf16((rng.standard_normal(numel) * 1e-3).astype(np.float32)) for _ in bases]
    seed = deterministic_seed(12, 3, 0)
    bufs = [gpu(b) for b in bs]
    upds = [torch.empty_like(x) for x in bufs]
    K.muon_prepare([(gpu(g), b, u, base, seed) for g, b, u, base in zip(gs, bufs, upds, bases)], 0.9, True)
    for g, b, buf, upd, base in zip(gs, bs, bufs, upds, bases):
        ob, ou = ew.muon_prepare(g, b, 0.9, True, seed, ctr_base=base)
        assert_bits_equal(bits_of(buf), ob, f"momentum base {base}")
        assert_bits_equal(bits_of(upd), ou, f"update base {base}")


def test_muon_apply_golden():
    d = load("muon_apply.npz")
    for k, s in enumerate(d["seeds"].tolist()):
        p = gpu(d["p"])
        K.muon_apply([(p, gpu(d["upd"]), float(d["scale"][k]), int(s))], float(d["lr"][k]), float(d["wd"][k]))
        assert_bits_equal(bits_of(p), d["out"][k], "apply")


def test_muon_apply_many_entries():
    rng = np.random.default_rng(3)
    sizes = [1, 7, 8, 9, 8191, 8192, 8193, 70000] * 10  # 80 entries > one launch's 64
    ps = [rne_bf16((rng.standard_normal(n) * 0.02).astype(np.float32)) for n in sizes]
    us = [rne_bf16((rng.standard_normal(n) * 0.1).astype(np.float32)) for n in sizes]
    pg = [gpu(p) for p in ps]
    K.muon_apply([(p, gpu(u), 1.7, 1000 + i) for i, (p, u) in enumerate(zip(pg, us))], 0.02, 0.01)
    for i, (p, pb, ub) in enumerate(zip(pg, ps, us)):
        assert_bits_equal(bits_of(p), ew.muon_apply(pb, ub, 0.02, 0.01, 1.7, 1000 + i), f"entry {i}")


def test_launch_packing_with_empty_entries():
    """More than one launch's worth of entries with empty tensors among them: every non-empty
    entry is updated exactly once (the packer resumes where the previous launch stopped)."""
    rng = np.random.default_rng(31)
    sizes = [0, 0, 5] + [3, 0, 7] * 30  # 93 entries, 32 of them empty
    ps = [rne_bf16((rng.standard_normal(n) * 0.02).astype(np.float32)) for n in sizes]
    us = [rne_bf16((rng.standard_normal(n) * 0.1).astype(np.float32)) for n in sizes]
    pg = [gpu(p) for p in ps]
    K.muon_apply([(p, gpu(u), 1.3, 500 + i) for i, (p, u) in enumerate(zip(pg, us))], 0.02, 0.01)
    for i, (p, pb, ub) in enumerate(zip(pg, ps, us)):
        assert_bits_equal(bits_of(p), ew.muon_apply(pb, ub, 0.02, 0.01, 1.3, 500 + i), f"apply entry {i}")
    gs = [rne_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32)) for n in sizes]
    pg, mg, vg = [gpu(p) for p in ps], [gpu(np.zeros(n, np.uint16)) for n in sizes], \
        [gpu(np.zeros(n, np.uint16)) for n in sizes]
    K.adamw_sr([(p, gpu(g), m, v, 2, 900 + i) for i, (p, g, m, v) in enumerate(zip(pg, gs, mg, vg))],
               3e-4, 0.9, 0.95, 1e-10, 0.01)
    for i, (p, pb, g) in enumerate(zip(pg, ps, gs)):
        z = np.zeros(len(pb), np.uint16)
        want = ew.adamw_sr(pb, g, z, z, 3e-4, 0.9, 0.95, 1e-10, 0.01, 2, 900 + i)[0]
        assert_bits_equal(bits_of(p), want, f"adamw entry {i}")
    n8 = [0] + [300] * 70  # 8-bit launcher: 64 entries per launch
    q1, q2 = torch.from_numpy(o8.create_dynamic_map(True)).to(DEV), torch.from_numpy(o8.create_dynamic_map(False)).to(DEV)
    p8 = [rne_bf16((rng.standard_normal(n) * 0.02).astype(np.float32)) for n in n8]
    g8 = [rne_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32)) for n in n8]
    tp = [gpu(p) for p in p8]
    st = [(gpu(np.zeros(n, np.uint16)), gpu(np.zeros(n, np.uint16))) for n in n8]
    K.adamw8bit([(p, gpu(g), s1, s2, None, None, 1, 40 + i, False) for i, (p, g, (s1, s2)) in
                 enumerate(zip(tp, g8, st))], q1, q2, 1e-3, 0.9, 0.999, 1e-8, 0.01, 256)
    for i, (p, pb, g) in enumerate(zip(tp, p8, g8)):
        z = np.zeros(len(pb), np.uint16)
        want = o8.adamw8bit(pb, g, z, z, None, None, None, None, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1, 40 + i, 256,
                            False)[0]
        assert_bits_equal(bits_of(p), want, f"8-bit entry {i}")


def test_adamw_golden():
    d = load("adamw.npz")
    for k, (step, idx) in enumerate(zip(d["steps"].tolist(), d["idx"].tolist())):
        p, m, v = gpu(d["p"]), gpu(d["m"]), gpu(d["v"])
        K.adamw_sr([(p, gpu(d["g"]), m, v, step, deterministic_seed(step, idx))], 3e-4, 0.9, 0.95, 1e-10, 0.01)
        assert_bits_equal(bits_of(p), d[f"p_{k}"], "p")
        assert_bits_equal(bits_of(m), d[f"m_{k}"], "m")
        assert_bits_equal(bits_of(v), d[f"v_{k}"], "v")
    for k, s in enumerate(d["edge_seeds"].tolist()):
        p, m, v = gpu(d["p"]), gpu(d["m"]), gpu(d["v"])
        K.adamw_sr([(p, gpu(d["g"]), m, v, 3, int(s))], 3e-4, 0.9, 0.95, 1e-10, 0.01)
        assert_bits_equal(bits_of(p), d[f"ep_{k}"], f"p edge seed {s}")
        assert_bits_equal(bits_of(m), d[f"em_{k}"], "m edge")
        assert_bits_equal(bits_of(v), d[f"ev_{k}"], "v edge")


def _adam8_run(case, tables):
    d = load("adamw8bit.npz")
    n, block, quant = d[f"c{case}_meta"].tolist()
    q1, q2 = torch.from_numpy(d["qmap1"]).to(DEV), torch.from_numpy(d["qmap2"]).to(DEV)
    qt = K.quant_tables(q1, q2) if tables else None
    if tables:
        assert qt is not None
    p = gpu(d[f"c{case}_p0"])
    if quant:
        s1 = torch.full((n,), 127, dtype=torch.uint8, device=DEV)
        s2 = torch.zeros(n, dtype=torch.uint8, device=DEV)
        a1 = torch.zeros((n + block - 1) // block, device=DEV)
        a2 = torch.zeros_like(a1)
    else:
        s1 = torch.zeros(n, dtype=torch.bfloat16, device=DEV)
        s2 = torch.zeros_like(s1)
        a1 = a2 = None
    for step in (1, 2, 3):
        seed = int(d[f"c{case}_seed{step}"])
        K.adamw8bit([(p, gpu(d[f"c{case}_g{step}"]), s1, s2, a1, a2, step, seed, bool(quant))], q1, q2,
                    1e-3, 0.9, 0.999, 1e-8, 0.01, block, qtables=qt)
        assert_bits_equal(bits_of(p), d[f"c{case}_p{step}"], f"p step {step}")
        if quant:
            assert_bits_equal(s1.cpu().numpy(), d[f"c{case}_s1_{step}"], f"codes1 step {step}")
            assert_bits_equal(s2.cpu().numpy(), d[f"c{case}_s2_{step}"], f"codes2 step {step}")
            assert_bits_equal(a1.cpu().numpy().view(np.uint32), d[f"c{case}_a1_{step}"].view(np.uint32), "absmax1")
            assert_bits_equal(a2.cpu().numpy().view(np.uint32), d[f"c{case}_a2_{step}"].view(np.uint32), "absmax2")
        else:
            assert_bits_equal(bits_of(s1), d[f"c{case}_s1_{step}"], f"m step {step}")
            assert_bits_equal(bits_of(s2), d[f"c{case}_s2_{step}"], f"v step {step}")


@pytest.mark.parametrize("tables", [False, True])
@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_adamw8bit_golden(case, tables):
    _adam8_run(case, tables)


@pytest.mark.parametrize("tables", [False, True])
@pytest.mark.parametrize("block", [32, 64, 128, 256, 512, 1024, 2048, 4096])
def test_adamw8bit_block_sizes_vs_oracle(block, tables):
    rng = np.random.default_rng(block)
    Q1, Q2 = o8.create_dynamic_map(True), o8.create_dynamic_map(False)
    q1, q2 = torch.from_numpy(Q1).to(DEV), torch.from_numpy(Q2).to(DEV)
    qt = K.quant_tables(q1, q2) if tables else None
    for n in (block * 3 + 5, 9000):
        pb = rne_bf16((rng.standard_normal(n) * 0.02).astype(np.float32))
        s1 = np.full(n, 127, np.uint8); s2 = np.zeros(n, np.uint8)
        a1 = np.zeros((n + block - 1) // block, np.float32); a2 = a1.copy()
        P, S1, S2 = gpu(pb), torch.from_numpy(s1).to(DEV), torch.from_numpy(s2).to(DEV)
        A1, A2 = torch.from_numpy(a1).to(DEV), torch.from_numpy(a2).to(DEV)
        for step in (1, 2):
            gb = rne_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32))
            seed = deterministic_seed(step, 9)
            pb, s1, s2, a1, a2 = o8.adamw8bit(pb, gb, s1, s2, a1, a2, Q1, Q2, 1e-3, 0.9, 0.999, 1e-8, 0.01, step,
                                              seed, block, True)
            K.adamw8bit([(P, gpu(gb), S1, S2, A1, A2, step, seed, True)], q1, q2, 1e-3, 0.9, 0.999, 1e-8, 0.01, block,
                        qtables=qt)
            assert_bits_equal(bits_of(P), pb, f"p block {block} n {n}")
            assert_bits_equal(S1.cpu().numpy(), s1, "codes1")
            assert_bits_equal(S2.cpu().numpy(), s2, "codes2")
            assert_bits_equal(A1.cpu().numpy().view(np.uint32), a1.view(np.uint32), "absmax1")


def test_sr_statistics_256_seeds():
    """North-star SR gate: every output is one of the two bracketing bf16 values and the
    mean over 256 seeds is within 3 sigma of the fp32 value (on the AdamW p output)."""
    rng = np.random.default_rng(4)
    n = 4096
    p0 = rne_bf16((rng.standard_normal(n) * 0.02).astype(np.float32))
    g = rne_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32))
    m0 = np.zeros(n, np.uint16)
    outs = []
    for s in range(256):
        p, m, v = gpu(p0), gpu(m0), gpu(m0)
        K.adamw_sr([(p, gpu(g), m, v, 1, s * 7919)], 3e-4, 0.9, 0.95, 1e-10, 0.0)
        outs.append(bf16_to_f32(bits_of(p)))
    outs = np.stack(outs).astype(np.float64)
    # exact fp32 value before rounding, from the oracle with SR removed
    b1, omb1, b2, omb2, ss, bc2s, eps, decay = ew.adamw_coefficients(3e-4, 0.9, 0.95, 1e-10, 0.0, 1)
    gf, pf = bf16_to_f32(g), bf16_to_f32(p0)
    mm = (omb1 * gf).astype(np.float32)
    vv = ((omb2 * gf) * gf).astype(np.float32)
    x = (pf * decay - ss * mm / (np.sqrt(vv) / bc2s + eps)).astype(np.float32).astype(np.float64)
    # bracketing values: truncation toward -inf / +inf in bf16 steps
    xb = x.astype(np.float32).view(np.uint32)
    trunc = (xb & 0xFFFF0000).view(np.float32).astype(np.float64)
    ulp = np.abs((((xb & 0xFFFF0000) + 0x10000).astype(np.uint32)).view(np.float32) - trunc)
    other = trunc + np.sign(x) * ulp
    ok = (outs == trunc) | (outs == other)
    assert ok.all(), "SR produced a value outside the two bracketing bf16 values"
    mean = outs.mean(0)
    frac = np.abs(x - trunc) / ulp
    sigma = ulp * np.sqrt(frac * (1 - frac) / 256) + 1e-30
    z = np.abs(mean - x) / sigma
    exact = frac == 0
    assert (z[~exact] < 3.0).mean() > 0.99, "SR mean drifts from the fp32 value"
    assert np.all(mean[exact] == x[exact])


@pytest.mark.parametrize("shape", [(1000, 768), (37, 100), (5000,), (3, 4, 5), (2, 8)])
def test_centralize_matches_reference_ops(shape):
    """The fused centralisation kernel against the reference's torch ops
    (muon_sr/triton_adamw.py:179-187) on the same GPU: bf16(g - c * mean_row) with the mean in
    fp32. Only the fp32 mean's summation order differs (a few fp32 ulps of the row's mean), so
    an element may differ by one bf16 ulp of the result plus that difference -- which is
    several bf16 ulps where g - c * mean nearly cancels -- on a small fraction of elements."""
    gen = torch.Generator(device="cuda").manual_seed(sum(shape))
    g = (torch.randn(*shape, device="cuda", generator=gen) * 1e-3).bfloat16()
    g[..., 0] += 5e-3  # rows with a clear nonzero mean
    g0 = g.clone()
    got = K.centralize(g, 0.5)
    dims = tuple(range(1, g.dim()))
    g32 = g.to(torch.float32)
    g32.sub_(g32.mean(dim=dims, keepdim=True).mul_(0.5))
    want = g32.to(torch.bfloat16)
    gi = got.view(torch.int16).int()
    wi = want.view(torch.int16).int()
    diff = (gi - wi).abs()
    assert float((diff > 0).float().mean()) < 0.02
    wf = want.float()
    ulp = ((wi + 1).to(torch.int16).view(torch.bfloat16).float() - wf).abs()
    row_mag = g.float().abs().mean(dim=dims, keepdim=True) if dims else g.float().abs().mean()
    bound = ulp + 0.5 * 2.0 ** -18 * row_mag
    assert bool(((got.float() - wf).abs() <= bound).all())
    assert torch.equal(g, g0)  # the gradient itself is not modified


def test_muon_prepare_gate_up_matrix_counters_cross_2_32():
    """One full gate/up matrix (14336 x 4096 = 58.7M elements) at the stack position whose
    Philox counters run through 2^32 (row 73 of a stack: counters 73 * numel ...), where the
    reference's int32 offset wraps (muon_sr/triton_muon_sr.py:44,156-164). The oracle checks
    the elements around the wrap and both ends of the matrix bit for bit."""
    numel = 14336 * 4096
    base = 73 * numel
    assert base < 2**32 < base + numel
    g = torch.Generator(device=DEV).manual_seed(73)
    grad = (torch.randn(numel, device=DEV, generator=g) * 1e-3).bfloat16()
    buf = (torch.randn(numel, device=DEV, generator=g) * 1e-3).bfloat16()
    b0 = bits_of(buf)
    upd = torch.empty_like(buf)
    seed = deterministic_seed(5, 4, 0)
    K.muon_prepare([(grad, buf, upd, base, seed)], 0.95, True)
    wrap = 2**32 - base
    gb, ob, ou = bits_of(grad), bits_of(buf), bits_of(upd)
    for lo, hi in ((0, 1 << 16), (wrap - (1 << 19), wrap + (1 << 19)), (numel - (1 << 16), numel)):
        eb, eu = ew.muon_prepare(gb[lo:hi], b0[lo:hi], 0.95, True, seed, ctr_base=base + lo)
        assert_bits_equal(ob[lo:hi], eb, f"momentum [{lo}, {hi})")
        assert_bits_equal(ou[lo:hi], eu, f"update [{lo}, {hi})")
