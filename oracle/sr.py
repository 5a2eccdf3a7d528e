"""fp32 / bf16 bit helpers and the two roundings the reference uses.

Stochastic rounding: ``muon_sr/triton_adamw.py:57-67`` (and the identical blocks in
``triton_muon_sr.py:44-47,75-78``, ``triton_adamw_8bit.py:77-79,92-97``): take the fp32
bits as int32, add the low 16 bits of a Philox word, clear the low 16 bits (int32
wrap-around arithmetic), reinterpret as fp32 and store as bf16 (exact, low bits are 0).
Round-to-nearest-even: Triton's ``.to(tl.bfloat16)`` on a value with nonzero low bits
(``triton_muon_sr.py:50``).
"""
import numpy as np


def bf16_to_f32(bits) -> np.ndarray:
    """bf16 bit patterns (uint16) -> fp32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_bits(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).view(np.uint32)


def sr_bf16(x, rand_u32) -> np.ndarray:
    """Stochastically round fp32 ``x`` with Philox words ``rand_u32`` -> bf16 bits."""
    bits = f32_bits(x).astype(np.uint64)
    noise = np.asarray(rand_u32, dtype=np.uint64) & np.uint64(0xFFFF)
    out = ((bits + noise) & np.uint64(0xFFFF0000)) >> np.uint64(16)
    return out.astype(np.uint16)


def rne_bf16(x) -> np.ndarray:
    """Round fp32 ``x`` to the nearest bf16 (ties to even) -> bf16 bits."""
    bits = f32_bits(x).astype(np.uint64)
    lsb = (bits >> np.uint64(16)) & np.uint64(1)
    out = ((bits + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) & np.uint64(0xFFFF)
    return _canon_nan(out.astype(np.uint16), x)


def truncate_bf16(x) -> np.ndarray:
    """Round fp32 ``x`` toward zero to bf16 bits (the Triton interpreter's fp32->bf16 cast)."""
    return (f32_bits(x) >> np.uint32(16)).astype(np.uint16)


def _canon_nan(out, x):
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        out = out.copy()
        out[nan] = 0x7FC0
    return out
