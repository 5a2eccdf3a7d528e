"""The 8-bit quantiser's lookup tables (CPU): the table rule reproduces the reference's
7-step codebook walk (restated in the oracle) bit for bit."""
import numpy as np
import pytest

from muon_sr_b200 import quant_tables as qt
from oracle import adamw8bit as o8
from tests._golden import load


@pytest.mark.parametrize("signed", [True, False])
def test_tables_match_walk_on_random_and_special_values(signed):
    Q = o8.create_dynamic_map(signed)
    codes, T = qt.build(Q, signed)
    rng = np.random.default_rng(1)
    mids = ((Q[1:] + Q[:-1]) * np.float32(0.5)).astype(np.float32)
    xs = np.concatenate([
        rng.uniform(-1, 1, 400_000), rng.standard_normal(200_000) * 1e-4, rng.standard_normal(200_000) * 1e-6,
        Q, mids, np.nextafter(mids, np.float32(2)), np.nextafter(mids, np.float32(-2)),
        np.nextafter(Q, np.float32(2)), np.nextafter(Q, np.float32(-2)),
        [0.0, -0.0, 1.0, -1.0, 1e-40, -1e-40, 2.7e-7, -2.7e-7]]).astype(np.float32)
    xs = np.clip(xs if signed else np.abs(xs), -1, 1).astype(np.float32)
    want = o8.quantize(xs, Q, signed).astype(np.int32)
    assert np.array_equal(qt.lookup(xs, codes, T, signed), want)


@pytest.mark.parametrize("signed", [True, False])
@pytest.mark.parametrize("e", [-1, -21])
def test_tables_match_walk_on_whole_binades(signed, e):
    """Every float of [2^e, 2^(e+1)] (the densest codebook region and the smallest codes)."""
    Q = o8.create_dynamic_map(signed)
    codes, T = qt.build(Q, signed)
    lo, hi = np.float32(2.0 ** e).view(np.uint32), np.float32(2.0 ** (e + 1)).view(np.uint32)
    x = np.arange(lo, hi + 1, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for sgn in ((1, -1) if signed else (1,)):
        xx = np.clip(x * np.float32(sgn), -1, 1).astype(np.float32)
        assert np.array_equal(qt.lookup(xx, codes, T, signed), o8.quantize(xx, Q, signed).astype(np.int32))


def test_blob_layout_matches_header_constants():
    import re, os
    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "include", "muon_sr_b200.h")).read()
    val = lambda name: int(re.search(rf"#define {name} (\d+)", hdr).group(1))
    assert val("MSR_QT_NB") == qt.NB and val("MSR_QT_BASE") == qt.BASE and val("MSR_QT_T_OFFSET") == qt.T_OFFSET
    d = load("adamw8bit.npz")
    b = qt.blob(d["qmap1"], d["qmap2"])
    assert b is not None and b.size == qt.BLOB_BYTES


def test_unsorted_codebook_falls_back_to_the_walk():
    Q = o8.create_dynamic_map(True).copy()
    Q[[10, 11]] = Q[[11, 10]]
    assert qt.build(Q, True) is None
