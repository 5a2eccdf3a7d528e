"""Exhaustive check of the 8-bit quantiser lookup tables against the reference's 7-step
codebook walk (the oracle's restatement, pinned by the golden vectors), over every fp32 value
the 8-bit kernel can quantise. The kernel quantises x = m / absmax of its block, so |x| <= 1:
all 2^30 + 1 fp32 magnitudes from 0 to 1.0, on each side of each codebook (about 3.2e9
quantisations, several minutes of CPU). Opt-in with MSR_EXHAUSTIVE=1; the regular suite
checks every bucket edge (quant_tables.build) and random values."""
import os

import numpy as np
import pytest

from muon_sr_b200 import quant_tables as qt
from oracle import adamw8bit as o8

pytestmark = pytest.mark.skipif(os.environ.get("MSR_EXHAUSTIVE") != "1",
                                reason="exhaustive: set MSR_EXHAUSTIVE=1 (several minutes of CPU)")
CHUNK = 1 << 23
ONE = 0x3F800000  # bit pattern of 1.0f


@pytest.mark.parametrize("signed,negative", [(True, False), (True, True), (False, False)])
def test_tables_equal_walk_for_every_input(signed, negative):
    Q = o8.create_dynamic_map(signed)
    codes, T = qt.build(Q, signed)
    for start in range(0, ONE + 1, CHUNK):
        x = np.arange(start, min(start + CHUNK, ONE + 1), dtype=np.uint32).view(np.float32)
        if negative:
            x = -x
        got = qt.lookup(x, codes, T, signed)
        want = o8.quantize(x, Q, signed).astype(np.int32)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (float(x[bad[0]]), int(got[bad[0]]), int(want[bad[0]]))
