"""ctypes binding of the engine's C ABI (``include/muon_sr_b200.h``).

The shared library ``libmuon_sr_b200.so`` is built in-tree by ``muon_sr_b200.build``. There
is no fallback: if the library is missing or cannot load, every optimizer step raises.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmuon_sr_b200.so")
# msr_abi_version() of the library these bindings describe (the entry structs below)
ABI_VERSION = 2

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_uint64 = ctypes.c_uint64
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t


class PrepareEntry(ctypes.Structure):
    _fields_ = [("grad", c_void_p), ("momentum", c_void_p), ("update", c_void_p),
                ("numel", c_int64), ("ctr_base", c_uint64), ("key", c_uint64)]


class ApplyEntry(ctypes.Structure):
    _fields_ = [("param", c_void_p), ("update", c_void_p), ("numel", c_int64), ("key", c_uint64),
                ("scale", c_float), ("reserved", c_float), ("param_mc", c_void_p)]


class AdamWEntry(ctypes.Structure):
    _fields_ = [("param", c_void_p), ("grad", c_void_p), ("exp_avg", c_void_p), ("exp_avg_sq", c_void_p),
                ("numel", c_int64), ("key_m", c_uint64), ("key_v", c_uint64), ("key_p", c_uint64),
                ("step_size", c_float), ("bc2_sqrt", c_float), ("param_mc", c_void_p)]


class AdamWHparams(ctypes.Structure):
    _fields_ = [("beta1", c_float), ("one_minus_beta1", c_float), ("beta2", c_float),
                ("one_minus_beta2", c_float), ("eps", c_float), ("decay", c_float)]


class PrepareRecord(ctypes.Structure):
    _fields_ = [("beta", c_float), ("one_minus_beta", c_float), ("nesterov", c_int32), ("count", c_int32)]


class ApplyRecord(ctypes.Structure):
    _fields_ = [("lr", c_float), ("decay", c_float), ("count", c_int32), ("reserved", c_int32)]


class AdamWRecord(ctypes.Structure):
    _fields_ = [("hp", AdamWHparams), ("count", c_int32), ("reserved", c_int32)]


class Adam8Entry(ctypes.Structure):
    _fields_ = [("param", c_void_p), ("grad", c_void_p), ("state1", c_void_p), ("state2", c_void_p),
                ("absmax1", c_void_p), ("absmax2", c_void_p), ("numel", c_int64), ("key_p", c_uint64),
                ("key_m", c_uint64), ("key_v", c_uint64), ("coef", c_float), ("sqrt_bc2_eps", c_float),
                ("quantized", c_int32), ("reserved", c_int32), ("param_mc", c_void_p)]


class Adam8Hparams(ctypes.Structure):
    _fields_ = [("beta1", c_float), ("one_minus_beta1", c_float), ("beta2", c_float),
                ("one_minus_beta2", c_float), ("decay", c_float), ("block_size", c_int32),
                ("qtables", c_void_p)]


# (name, restype, argtypes) of every exported symbol, in header order.
SIGNATURES = [
    ("msr_abi_version", c_int, []),
    ("msr_set_sr_noise", c_int, [c_int]),
    ("msr_get_sr_noise", c_int, []),
    ("msr_status_string", ctypes.c_char_p, [c_int]),
    ("msr_last_error", ctypes.c_char_p, []),
    ("msr_device_error", c_int, [c_void_p, c_int]),
    ("msr_test_wait_timeout", c_int, [c_uint64, c_void_p]),
    ("msr_launch_count", c_uint64, []),
    ("msr_set_gemm_max_ctas", None, [c_int]),
    ("msr_set_gemm_pairs", None, [c_int]),
    ("msr_get_gemm_pairs", c_int, []),
    ("msr_philox_fill", c_int, [c_void_p, c_int64, c_uint64, c_uint64, c_void_p]),
    ("msr_grad_accum_bf16", c_int, [c_void_p, c_void_p, c_int64, c_uint64, c_int, c_void_p]),
    ("msr_muon_prepare", c_int, [ctypes.POINTER(PrepareEntry), c_int, c_float, c_float, c_int, c_void_p]),
    ("msr_muon_apply", c_int, [ctypes.POINTER(ApplyEntry), c_int, c_float, c_float, c_void_p]),
    ("msr_adamw_sr", c_int, [ctypes.POINTER(AdamWEntry), c_int, ctypes.POINTER(AdamWHparams), c_void_p]),
    ("msr_muon_prepare_rec", c_int, [ctypes.POINTER(PrepareEntry), c_int, c_void_p, c_void_p]),
    ("msr_muon_apply_rec", c_int, [ctypes.POINTER(ApplyEntry), c_int, c_void_p, c_void_p]),
    ("msr_adamw_sr_rec", c_int, [ctypes.POINTER(AdamWEntry), c_int, c_void_p, c_void_p]),
    ("msr_centralize_bf16", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    ("msr_adamw8bit", c_int, [ctypes.POINTER(Adam8Entry), c_int, c_void_p, c_void_p,
                              ctypes.POINTER(Adam8Hparams), c_void_p]),
    ("msr_ns_workspace_bytes", c_size_t, [c_int64, c_int64, c_int64]),
    ("msr_newton_schulz_bf16", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int, c_void_p,
                                       c_void_p, c_size_t, c_void_p]),
    ("msr_newton_schulz_bf16_noalloc", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int,
                                               c_void_p, c_void_p]),
    ("msr_ipc_export", c_int, [c_void_p, c_void_p, ctypes.POINTER(c_uint64)]),
    ("msr_ipc_import", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    ("msr_ipc_close", c_int, [c_void_p]),
    ("msr_copy_async", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("msr_ipc_event_create", c_int, [ctypes.POINTER(c_void_p), c_void_p]),
    ("msr_ipc_event_open", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    ("msr_event_record", c_int, [c_void_p, c_void_p]),
    ("msr_stream_wait_event", c_int, [c_void_p, c_void_p]),
    ("msr_event_destroy", c_int, [c_void_p]),
    ("msr_gemm_bf16", c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                              c_int64, c_float, c_float, c_void_p, c_int, c_int, c_int, c_void_p]),
    ("msr_gemm_tile_map", c_int, [c_int64, c_int64, c_int64, c_int, c_int, ctypes.POINTER(c_int64), c_int64,
                                  ctypes.POINTER(c_int64)]),
]

_lib = None
_lock = threading.Lock()


def load():
    """Load (once) and return the shared library; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"muon_sr_b200: CUDA library {LIB_PATH} is missing; build it with "
                    "`python -m muon_sr_b200.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, restype, argtypes in SIGNATURES:
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _apply_env(lib)
            _lib = lib
    return _lib


# Process-wide debug knobs read once, when the library loads: MSR_SR_NOISE selects the
# stochastic-rounding noise ("none" = round to nearest, the parity mode), MSR_GEMM_PAIRS=0
# the single-SM GEMM tiles. Both give the same API; see msr_set_sr_noise / msr_set_gemm_pairs.
ENV_SR_NOISE = {"reference": 0, "fast": 1, "none": 2}


def _apply_env(lib):
    noise = os.environ.get("MSR_SR_NOISE")
    if noise:
        if noise not in ENV_SR_NOISE:
            raise ValueError(f"MSR_SR_NOISE must be one of {sorted(ENV_SR_NOISE)}, got {noise!r}")
        lib.msr_set_sr_noise(ENV_SR_NOISE[noise])
    pairs = os.environ.get("MSR_GEMM_PAIRS")
    if pairs:
        if pairs not in ("0", "1"):
            raise ValueError(f"MSR_GEMM_PAIRS must be 0 or 1, got {pairs!r}")
        lib.msr_set_gemm_pairs(int(pairs))


def check(status: int, what: str) -> None:
    if status != 0:
        lib = load()
        raise RuntimeError(f"{what} failed: {lib.msr_status_string(status).decode()}: "
                           f"{lib.msr_last_error().decode()}")
