"""Helpers shared by the tests: fixture loading and bf16 bit conversions."""
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def to_bf16(bits, device="cpu"):
    t = torch.from_numpy(np.ascontiguousarray(np.asarray(bits, dtype=np.uint16)).view(np.int16).copy())
    return t.view(torch.bfloat16).to(device)


def bits_of(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()


def assert_bits_equal(got, want, what=""):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, f"{what}: {bad.size} of {want.size} differ, first at {bad[:5]}: got {got.flat[bad[:5]]} want {want.flat[bad[:5]]}"
