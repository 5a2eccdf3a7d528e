"""The C-ABI library loads and exports every entry point the public header declares
(CPU only: nothing here launches a kernel)."""
import ctypes
import os
import re

import pytest


from muon_sr_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "muon_sr_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(msr_\w+)\s*\(", text)))


def test_library_exists_and_loads():
    assert os.path.exists(_lib.LIB_PATH), "build the library first: python -m muon_sr_b200.build"
    lib = _lib.load()
    assert lib.msr_abi_version() == _lib.ABI_VERSION == 2


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 12
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert bound == set(declared_functions())


def test_status_strings_and_argument_errors_without_gpu():
    lib = _lib.load()
    assert lib.msr_status_string(0) == b"ok"
    assert lib.msr_status_string(4) == b"workspace too small"
    # argument validation happens before any CUDA call
    assert lib.msr_grad_accum_bf16(None, None, -1, 0, 0, None) == 1
    assert b"negative" in lib.msr_last_error()
    assert lib.msr_newton_schulz_bf16(None, None, 1, 8, 8, 5, 0, None, None, 0, None) == 1
    assert lib.msr_ns_workspace_bytes(0, 8, 8) == 0


def test_ns_workspace_accounts_for_padding():
    lib = _lib.load()
    plain = lib.msr_ns_workspace_bytes(4, 64, 128)
    padded = lib.msr_ns_workspace_bytes(4, 63, 127)
    assert plain > 0 and padded > plain  # padded shapes need two more staging buffers


def test_more_argument_errors_without_gpu():
    """Every entry point rejects bad arguments with MSR_ERR_INVALID (1) and a message before
    it touches a device."""
    lib = _lib.load()
    assert lib.msr_set_sr_noise(7) == 1 and b"unknown mode" in lib.msr_last_error()
    assert lib.msr_set_sr_noise(-1) == 1
    for mode in (1, 2, 0):  # fast, none, back to the reference's stream
        assert lib.msr_set_sr_noise(mode) == 0
    assert lib.msr_test_wait_timeout(0, None) == 1
    assert lib.msr_centralize_bf16(None, None, 4, 4, 0.5, None) == 1
    assert lib.msr_gemm_bf16(None, 0, None, 0, None, None, 1, 8, 8, 8, 1.0, 0.0, None, 0, 0, 0, None) == 1
    assert lib.msr_newton_schulz_bf16(None, None, 1, 8, 8, 5, 9, None, None, 0, None) == 1
    assert lib.msr_newton_schulz_bf16_noalloc(None, None, 1, 8, 8, 5, 0, None, None) == 1
    assert lib.msr_muon_prepare(None, -1, 0.9, 0.1, 1, None) == 1
    assert lib.msr_muon_apply(None, -1, 0.02, 1.0, None) == 1
    assert lib.msr_adamw_sr(None, -1, None, None) == 1
    assert lib.msr_adamw8bit(None, -1, None, None, None, None) == 1
    assert lib.msr_copy_async(None, None, 16, None) == 1
    assert lib.msr_ipc_export(None, None, None) == 1
    assert lib.msr_ipc_import(None, None) == 1
    assert lib.msr_ipc_event_create(None, None) == 1
    assert lib.msr_ipc_event_open(None, None) == 1
    # zero-length and empty requests are no-ops
    assert lib.msr_copy_async(None, None, 0, None) == 0
    assert lib.msr_muon_prepare(None, 0, 0.9, 0.1, 1, None) == 0


def test_env_knobs_apply_at_load():
    """MSR_SR_NOISE and MSR_GEMM_PAIRS are applied once, when the library loads; a bad value
    is refused with a message naming the variable."""
    import subprocess
    import sys
    code = ("from muon_sr_b200 import _lib; l = _lib.load(); "
            "print(l.msr_get_sr_noise(), l.msr_get_gemm_pairs())")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

    def run(env):
        return subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True,
                              env=dict(os.environ, **env), timeout=300)
    assert run({}).stdout.split() == ["0", "1"]
    assert run({"MSR_SR_NOISE": "none", "MSR_GEMM_PAIRS": "0"}).stdout.split() == ["2", "0"]
    assert run({"MSR_SR_NOISE": "fast"}).stdout.split() == ["1", "1"]
    bad = run({"MSR_SR_NOISE": "xoshiro"})
    assert bad.returncode != 0 and "MSR_SR_NOISE" in bad.stderr


def _tile_map(M, N, batch, sym, pairs):
    lib = _lib.load()
    n = ctypes.c_int64()
    assert lib.msr_gemm_tile_map(M, N, batch, sym, pairs, None, 0, ctypes.byref(n)) == 0
    out = (ctypes.c_int64 * (3 * n.value))()
    assert lib.msr_gemm_tile_map(M, N, batch, sym, pairs, out, 3 * n.value, ctypes.byref(n)) == 0
    return [tuple(out[3 * i:3 * i + 3]) for i in range(n.value)]


@pytest.mark.parametrize("pairs", [0, 1])
def test_gemm_tile_schedule_covers_each_tile_once(pairs):
    """The persistent GEMM's tile decoding, run on the host: every output tile of every matrix
    exactly once (full GEMMs), and in symmetric mode exactly the tiles that hold an element
    on or above the diagonal -- whose mirror-writes then cover the rest."""
    tm, bn = (256 if pairs else 128), 256
    sizes = [1, 100, 128, 129, 255, 256, 257, 768, 1000, 1024, 2049, 4096]
    for M in sizes:
        for N in sizes[::3] + [M]:
            for batch in (1, 3):
                got = _tile_map(M, N, batch, 0, pairs)
                want = [(b, i * tm, k * bn) for b in range(batch) for i in range(-(-M // tm))
                        for k in range(-(-N // bn))]
                assert sorted(got) == sorted(want) and len(got) == len(want), (M, N, batch)
        for batch in (1, 2):
            got = _tile_map(M, M, batch, 1, pairs)
            want = [(b, i * tm, k * bn) for b in range(batch) for i in range(-(-M // tm))
                    for k in range(-(-M // bn)) if k * bn + bn > i * tm]  # tile reaches the diagonal
            assert sorted(got) == sorted(want) and len(got) == len(set(got)), (M, batch)
    # grouped rasterisation: consecutive tiles stay within bands of 8 row-blocks
    got = _tile_map(4096, 14336, 1, 0, pairs)
    band = [m // (8 * tm) for _, m, _ in got]
    assert band == sorted(band)


def test_gemm_tile_map_argument_errors():
    lib = _lib.load()
    n = ctypes.c_int64()
    assert lib.msr_gemm_tile_map(0, 8, 1, 0, 0, None, 0, ctypes.byref(n)) == 1
    assert lib.msr_gemm_tile_map(8, 16, 1, 1, 0, None, 0, ctypes.byref(n)) == 1  # symmetric needs M == N
    assert lib.msr_gemm_tile_map(300, 300, 1, 0, 0, None, 0, ctypes.byref(n)) == 0
    out = (ctypes.c_int64 * 3)()
    assert lib.msr_gemm_tile_map(300, 300, 1, 0, 0, out, 3, ctypes.byref(n)) == 1  # too small
