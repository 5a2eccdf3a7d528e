"""Philox4x32-10 exactly as Triton's ``tl.randint`` uses it, plus the reference's seeds.

Third-party arithmetic: Triton 3.6.0 ``triton/language/random.py:12-110`` (unpinned in the
reference's ``pyproject.toml:15-18``). The algorithm is the published Philox4x32 counter
generator (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
SC 2011) with 10 rounds, multipliers 0xD2511F53 / 0xCD9E8D57 and Weyl key increments
0x9E3779B9 / 0xBB67AE85. Triton's layout: counter = (offset_lo32, offset_hi32, 0, 0),
key = (seed_lo32, seed_hi32); ``randint`` returns the first output word.
"""
import numpy as np

_M32 = np.uint64(0xFFFFFFFF)
_MUL_A = np.uint64(0xD2511F53)
_MUL_B = np.uint64(0xCD9E8D57)
_KEY_A = np.uint64(0x9E3779B9)
_KEY_B = np.uint64(0xBB67AE85)


def philox_randint(key64: int, counters) -> np.ndarray:
    """First Philox4x32-10 output word for each 32-bit counter.

    ``key64`` is the 64-bit key (seed after Triton's scalar typing, see ``triton_key``);
    ``counters`` are the per-element offsets already truncated to 32 bits, as every
    reference kernel passes them (e.g. ``triton_muon_sr.py:44``, ``triton_adamw.py:52``).
    """
    c0 = np.asarray(counters).astype(np.uint64) & _M32
    c1 = np.zeros_like(c0)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint64(key64 & 0xFFFFFFFF)
    k1 = np.uint64((key64 >> 32) & 0xFFFFFFFF)
    for _ in range(10):
        p0 = _MUL_A * c0
        p2 = _MUL_B * c2
        n0 = ((p2 >> np.uint64(32)) ^ c1 ^ k0) & _M32
        n2 = ((p0 >> np.uint64(32)) ^ c3 ^ k1) & _M32
        c1 = p2 & _M32
        c3 = p0 & _M32
        c0, c2 = n0, n2
        k0 = (k0 + _KEY_A) & _M32
        k1 = (k1 + _KEY_B) & _M32
    return c0.astype(np.uint32)


def triton_key(seed: int, add: int = 0) -> int:
    """64-bit Philox key that a Triton kernel derives from the Python int ``seed`` + ``add``.

    Triton types an int argument in [-2^31, 2^31) as i32 and a larger one as i64. The
    reference adds small constants inside the kernel (``seed + 1``, ``seed + 2`` at
    ``triton_adamw.py:53-54`` and ``triton_adamw_8bit.py:94-95``), so for an i32 seed the
    sum wraps in 32 bits and is then sign-extended to the 64-bit key
    (``triton/language/random.py:49``: ``seed.to(tl.uint64)``). Checked against the
    interpreter for seeds 2^31-1 (wraps) and 2^32-1 (does not).
    """
    if -(1 << 31) <= seed < (1 << 31):
        v = (seed + add + (1 << 31)) % (1 << 32) - (1 << 31)
    else:
        v = seed + add
    return v & 0xFFFFFFFFFFFFFFFF


def deterministic_seed(step: int, param_idx: int, salt: int = 0) -> int:
    """``_deterministic_seed`` -- ``muon_sr/triton_muon_sr.py:83-85``; AdamW uses salt 0
    (``triton_adamw.py:97``) and so does the 8-bit optimizer (``triton_adamw_8bit.py:197``)."""
    return (step * 2654435761 ^ param_idx * 1234567891 ^ salt) & 0xFFFFFFFF


def philox4(key64: int, counters64) -> np.ndarray:
    """All four Philox4x32-10 output words for 64-bit counters (ctr_lo32, ctr_hi32, 0, 0);
    shape (n, 4), uint32."""
    c = np.asarray(counters64).astype(np.uint64)
    c0 = c & _M32
    c1 = c >> np.uint64(32)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint64(key64 & 0xFFFFFFFF)
    k1 = np.uint64((key64 >> 32) & 0xFFFFFFFF)
    for _ in range(10):
        p0 = _MUL_A * c0
        p2 = _MUL_B * c2
        n0 = ((p2 >> np.uint64(32)) ^ c1 ^ k0) & _M32
        n2 = ((p0 >> np.uint64(32)) ^ c3 ^ k1) & _M32
        c1 = p2 & _M32
        c3 = p0 & _M32
        c0, c2 = n0, n2
        k0 = (k0 + _KEY_A) & _M32
        k1 = (k1 + _KEY_B) & _M32
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def fast_noise(key64: int, counters64) -> np.ndarray:
    """The engine's opt-in fast noise stream (not the reference's): counter c takes the
    16-bit half (c & 1) of output word ((c >> 1) & 3) of Philox4x32-10 at counter c >> 3."""
    c = np.asarray(counters64).astype(np.uint64)
    words = philox4(key64, c >> np.uint64(3))
    k = (c & np.uint64(7)).astype(np.int64)
    w = words[np.arange(c.size), k >> 1].astype(np.uint32)
    return (w >> (16 * (k & 1)).astype(np.uint32)) & np.uint32(0xFFFF)


def sr_noise(key64: int, n: int, ctr_base: int = 0, mode: str = "reference") -> np.ndarray:
    """Noise words of ``n`` consecutive elements from ``ctr_base``: the reference's stream
    (Philox word 0 at the offset truncated to 32 bits) or the fast one (64-bit counters)."""
    ctr = np.arange(n, dtype=np.uint64) + np.uint64(ctr_base)
    if mode == "reference":
        return philox_randint(key64, ctr & _M32)
    if mode == "fast":
        return fast_noise(key64, ctr)
    raise ValueError(f"unknown noise mode {mode!r}")
