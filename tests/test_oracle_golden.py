"""The CPU oracle against the golden vectors produced by the reference itself."""
import numpy as np
import pytest

from oracle import adamw8bit as o8
from oracle import elementwise as ew
from oracle.newton_schulz import newton_schulz
from oracle.philox import deterministic_seed, philox_randint, triton_key
from oracle.sr import rne_bf16, truncate_bf16
from tests._golden import assert_bits_equal, bits_of, load, to_bf16


def test_philox_words():
    d = load("philox.npz")
    for i, s in enumerate(d["seeds"].tolist()):
        for add in range(3):
            for j, b in enumerate(d["bases"].tolist()):
                ctr = (np.arange(32, dtype=np.uint64) + np.uint64(b)) & np.uint64(0xFFFFFFFF)
                got = philox_randint(triton_key(int(s), add), ctr)
                assert_bits_equal(got, d["words"][i, add, j], f"seed={s} add={add} base={b}")


def test_grad_accum():
    d = load("grad_accum.npz")
    for k, s in enumerate(d["seeds"].tolist()):
        assert_bits_equal(ew.grad_accum(d["acc"], d["grad"], int(s)), d["out"][k], "grad_accum")


@pytest.mark.parametrize("nest", [0, 1])
def test_muon_prepare(nest):
    d = load("muon_prepare.npz")
    for k, s in enumerate(d["seeds"].tolist()):
        buf, upd, upd32 = ew.muon_prepare(d["grad"], d["buf"], float(d["beta"]), bool(nest), int(s),
                                          return_f32=True)
        assert_bits_equal(buf, d[f"buf_{nest}_{k}"], "buf")
        # the interpreter's fp32->bf16 cast truncates; the fp32 value itself must agree
        assert_bits_equal(truncate_bf16(upd32), d[f"upd_{nest}_{k}"], "update (truncated)")
        # and the engine's RNE store is the nearest bf16 of that same fp32 value
        assert_bits_equal(upd, rne_bf16(upd32), "update (RNE)")


def test_muon_apply():
    d = load("muon_apply.npz")
    for k, s in enumerate(d["seeds"].tolist()):
        out = ew.muon_apply(d["p"], d["upd"], float(d["lr"][k]), float(d["wd"][k]), float(d["scale"][k]), int(s))
        assert_bits_equal(out, d["out"][k], "apply")


def test_adamw():
    d = load("adamw.npz")
    for k, (step, idx) in enumerate(zip(d["steps"].tolist(), d["idx"].tolist())):
        seed = deterministic_seed(step, idx)
        p, m, v = ew.adamw_sr(d["p"], d["g"], d["m"], d["v"], 3e-4, 0.9, 0.95, 1e-10, 0.01, step, seed)
        assert_bits_equal(p, d[f"p_{k}"], "p")
        assert_bits_equal(m, d[f"m_{k}"], "m")
        assert_bits_equal(v, d[f"v_{k}"], "v")
    for k, s in enumerate(d["edge_seeds"].tolist()):
        p, m, v = ew.adamw_sr(d["p"], d["g"], d["m"], d["v"], 3e-4, 0.9, 0.95, 1e-10, 0.01, 3, int(s))
        assert_bits_equal(p, d[f"ep_{k}"], f"p edge seed {s}")
        assert_bits_equal(m, d[f"em_{k}"], "m edge")
        assert_bits_equal(v, d[f"ev_{k}"], "v edge")


def test_dynamic_maps():
    d = load("adamw8bit.npz")
    assert_bits_equal(o8.create_dynamic_map(True).view(np.uint32), d["qmap1"].view(np.uint32), "qmap1")
    assert_bits_equal(o8.create_dynamic_map(False).view(np.uint32), d["qmap2"].view(np.uint32), "qmap2")


def test_quantize():
    d = load("adamw8bit.npz")
    assert_bits_equal(o8.quantize(d["qs_x"], d["qmap1"], True), d["qs_code"], "signed")
    assert_bits_equal(o8.quantize(d["qu_x"], d["qmap2"], False), d["qu_code"], "unsigned")


@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_adamw8bit(case):
    d = load("adamw8bit.npz")
    n, block, quant = d[f"c{case}_meta"].tolist()
    p = d[f"c{case}_p0"]
    if quant:
        s1 = np.full(n, 127, np.uint8); s2 = np.zeros(n, np.uint8)
        a1 = np.zeros((n + block - 1) // block, np.float32); a2 = a1.copy()
    else:
        s1 = np.zeros(n, np.uint16); s2 = np.zeros(n, np.uint16); a1 = a2 = None
    for step in (1, 2, 3):
        seed = int(d[f"c{case}_seed{step}"])
        p, s1, s2, a1, a2 = o8.adamw8bit(p, d[f"c{case}_g{step}"], s1, s2, a1, a2, d["qmap1"], d["qmap2"],
                                         1e-3, 0.9, 0.999, 1e-8, 0.01, step, seed, block, quant)
        assert_bits_equal(p, d[f"c{case}_p{step}"], f"p step {step}")
        assert_bits_equal(s1, d[f"c{case}_s1_{step}"], f"state1 step {step}")
        assert_bits_equal(s2, d[f"c{case}_s2_{step}"], f"state2 step {step}")
        if quant:
            assert_bits_equal(a1.view(np.uint32), d[f"c{case}_a1_{step}"].view(np.uint32), "absmax1")
            assert_bits_equal(a2.view(np.uint32), d[f"c{case}_a2_{step}"].view(np.uint32), "absmax2")


def test_newton_schulz_cpu_matches_reference_bits():
    d = load("newton_schulz.npz")
    for k in range(int(d["count"])):
        shp = tuple(d[f"shape{k}"].tolist())
        x = to_bf16(d[f"x{k}"]).view(*shp)
        y = newton_schulz(x, 5, None)
        assert_bits_equal(bits_of(y), d[f"y{k}"], f"NS shape {shp}")


def test_fast_noise_stream_layout():
    """The engine's fast stream is built from the same (golden-checked) Philox4x32-10: word
    0 of the 4-word generator equals the reference's word for 32-bit counters, and counter c
    takes 16-bit half c & 1 of word (c >> 1) & 3 at generator counter c >> 3."""
    from oracle.philox import fast_noise, philox4, philox_randint
    key = 0x0123456789ABCDEF
    ctr = np.arange(0, 5000, 7, dtype=np.uint64)
    assert np.array_equal(philox4(key, ctr)[:, 0], philox_randint(key, ctr))
    c = np.arange(64, dtype=np.uint64) + np.uint64(3 * 2**32 + 5)
    words = philox4(key, c >> np.uint64(3))
    want = [(int(words[i, (int(x) >> 1) & 3]) >> (16 * (int(x) & 1))) & 0xFFFF for i, x in enumerate(c)]
    assert fast_noise(key, c).tolist() == want
    vals = fast_noise(key, np.arange(1 << 16, dtype=np.uint64))
    assert vals.max() < 1 << 16
    hist = np.bincount(vals >> 12, minlength=16)  # 16 bins of a uniform 16-bit value
    assert hist.min() > 0.9 * (1 << 12) and hist.max() < 1.1 * (1 << 12)


def test_round_to_nearest_mode_is_the_fp32_formula_cast():
    """noise="none" (the engine's parity mode) is the reference formula in fp32 rounded to
    nearest even -- the same fp32 values the SR modes round stochastically."""
    from oracle.sr import bf16_to_f32
    rng = np.random.default_rng(9)
    n = 4096
    a, g = rne_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32)), \
        rne_bf16((rng.standard_normal(n) * 1e-3).astype(np.float32))
    want = rne_bf16((bf16_to_f32(a) + bf16_to_f32(g)).astype(np.float32))
    assert_bits_equal(ew.grad_accum(a, g, 5, noise="none"), want, "grad_accum rtn")
    sr = ew.grad_accum(a, g, 5)
    # SR lands on one of the two bf16 neighbours of the fp32 sum; RTN on the nearer one
    s = (bf16_to_f32(a) + bf16_to_f32(g)).astype(np.float32)
    lo = truncate_bf16(s)
    assert np.all((sr == lo) | (sr == lo + 1) | (s == 0))
    assert np.all((want == lo) | (want == lo + 1) | (s == 0))
