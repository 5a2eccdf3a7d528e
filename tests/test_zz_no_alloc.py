"""Newton-Schulz through the entry point that allocates nothing.

msr_newton_schulz_bf16_noalloc serves callers that cannot allocate device memory (a plugin
whose host program owns all device allocations, a C / FFI caller without a device
allocator): it takes its scratch from a fixed 64 MiB area inside the library instead of a
caller-provided workspace. These tests call it through the C ABI and check that two calls
in a row give the same result as msr_newton_schulz_bf16 with a workspace, within the
Newton-Schulz tolerance used everywhere else (and, since the arithmetic is the same, bit for
bit), and that a request larger than the area is refused. This file is named to be
collected last.
"""
import ctypes

import pytest
import torch

from muon_sr_b200 import _lib
from muon_sr_b200 import kernels as K
from oracle.newton_schulz import rel_frobenius

pytestmark = pytest.mark.gpu
NS_TOL = 1e-2


def _noalloc(x, out, steps=5, mode=K.NS_REFERENCE_ROUNDING, norm_sq=None):
    rows, cols = x.shape[-2], x.shape[-1]
    batch = x.numel() // (rows * cols)
    return _lib.load().msr_newton_schulz_bf16_noalloc(
        x.data_ptr(), out.data_ptr(), batch, rows, cols, steps, mode,
        norm_sq.data_ptr() if norm_sq is not None else None,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("shape", [(3, 256, 512), (2, 512, 256), (2, 100, 300), (1, 2048, 2048)])
@pytest.mark.parametrize("mode", [K.NS_REFERENCE_ROUNDING, K.NS_FUSED_ROUNDING])
def test_noalloc_matches_workspace_entry_on_two_calls(shape, mode):
    g = torch.Generator(device="cuda").manual_seed(shape[1] + shape[2] + mode)
    x = (torch.randn(*shape, device="cuda", generator=g) * 1e-3).bfloat16()
    want = K.newton_schulz(x, 5, mode=mode)
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        st = _noalloc(x, out, mode=mode)
        assert st == 0, _lib.load().msr_last_error().decode()
        torch.cuda.synchronize()
        assert rel_frobenius(out, want) < NS_TOL, (call, shape)
        assert torch.equal(out.view(torch.int16), want.view(torch.int16)), (call, shape)


def test_noalloc_with_given_norm():
    x = (torch.randn(4, 256, 384, device="cuda") * 1e-2).bfloat16()
    nsq = (x.float() ** 2).sum(dim=(1, 2)).contiguous()
    want = K.newton_schulz(x, 5, norm_sq=nsq)
    out = torch.empty_like(x)
    assert _noalloc(x, out, norm_sq=nsq) == 0
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))


def test_noalloc_refuses_requests_beyond_its_area():
    x = torch.zeros(1, 4096, 4096, device="cuda", dtype=torch.bfloat16)  # needs 96 MiB of scratch
    out = torch.empty_like(x)
    st = _noalloc(x, out)
    assert st == 4  # MSR_ERR_WORKSPACE
    assert b"fixed" in _lib.load().msr_last_error()
    assert _noalloc(x, out, steps=-1) == 1  # MSR_ERR_INVALID, before any GPU work
