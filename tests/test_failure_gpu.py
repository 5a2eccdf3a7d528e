"""Failure detection on the GPU without a fault: a bounded device-side wait runs out.

Every wait in this library's kernels (the GEMM's copy, MMA and epilogue roles) gives up after
a time limit, records a code that ``msr_device_error`` returns, drains and returns. The test
hook waits with that same routine on a barrier nothing arrives on; the host must read the
code, and the context must stay usable for the next kernels. Nothing traps, faults or hangs.
"""
import time

import pytest
import torch

from muon_sr_b200 import _lib
from muon_sr_b200 import kernels as K

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    lib = _lib.load()
    K.device_error(clear=True)
    t0 = time.perf_counter()
    _lib.check(lib.msr_test_wait_timeout(20_000_000, K.stream_handle()), "msr_test_wait_timeout")  # 20 ms
    code = K.device_error(clear=True)
    elapsed = time.perf_counter() - t0
    assert code == 0x1FF
    assert 0.015 < elapsed < 5.0, elapsed
    assert K.device_error() == 0, "the code is cleared"
    # the context still runs kernels: a GEMM and a Newton-Schulz call after the timeout
    a = torch.randn(2, 256, 128, device="cuda").bfloat16()
    d = K.gemm_bf16(a, 0, a, 0)
    ref = a.float() @ a.float().transpose(1, 2)
    assert float((d.float() - ref).norm() / ref.norm()) < 1e-2
    y = K.newton_schulz(a, 5)
    assert torch.isfinite(y.float()).all()
    assert K.device_error() == 0


def test_wait_timeout_rejects_bad_limits():
    lib = _lib.load()
    assert lib.msr_test_wait_timeout(0, K.stream_handle()) == 1          # MSR_ERR_INVALID
    assert lib.msr_test_wait_timeout(20_000_000_000, K.stream_handle()) == 1
