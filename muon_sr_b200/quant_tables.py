"""Lookup tables that let the 8-bit kernel quantise with two shared-memory reads.

The reference quantiser (muon_sr/triton_adamw_8bit.py:27-53: a 7-step pivot walk over the
sorted 256-entry codebook, midpoint tie rules against the bracketing values, and a sign fix
for the signed map) is, for a sorted codebook, a step function of x: as |x| grows the code
moves one entry at a time at fixed fp32 thresholds. The tables encode that function exactly:

* buckets: |x| split by its fp32 bit pattern into 2^15-float buckets (exponent and top 8
  mantissa bits, relative width 2^-8), from 2^-30 up to 1.0; bucket 0 holds everything
  smaller. ``code[bucket]`` is the code at the bucket's smallest |x|.
* thresholds: ``T[c]`` is the smallest |x| at which code c is left (c -> c + 1 for x >= 0,
  c -> c - 1 for x < 0), +inf if never.
* kernel: ``c = code[bucket(|x|)]; c += (|x| >= T[c])`` (or ``-=`` on the negative side).

That is exact as long as no bucket holds two transitions; ``build`` checks this (and the
whole function at every bucket edge) against a restatement of the reference walk and
returns None when it does not hold, in which case the kernel runs the walk itself.
"""
import numpy as np

BUCKET_SHIFT = 15
EMIN = -30                                                # buckets start at 2^EMIN
BASE = (((127 + EMIN) << 23) >> BUCKET_SHIFT) - 1         # bucket 0: |x| < 2^EMIN
NB = ((127 << 23) >> BUCKET_SHIFT) - BASE + 1             # up to and including 1.0
INF_BITS = np.uint32(0x7F800000)


def _walk(x, Q, signed):
    """The reference pivot walk with its tie and sign rules, vectorised (fp32)."""
    x = np.asarray(x, np.float32)
    pivot = np.full(x.shape, 127, np.int32)
    lo_p = np.zeros(x.shape, np.int32)
    up_p = np.full(x.shape, 255, np.int32)
    lower = np.full(x.shape, -1.0 if signed else 0.0, np.float32)
    upper = np.full(x.shape, 1.0, np.float32)
    val = Q[pivot]
    for shift in range(7):
        d = 64 >> shift
        right = x > val
        lo_p = np.where(right, pivot, lo_p)
        up_p = np.where(right, up_p, pivot)
        lower = np.where(right, val, lower)
        upper = np.where(right, upper, val)
        pivot = pivot + np.where(right, d, -d).astype(np.int32)
        val = Q[pivot]
    mid_up = ((upper + val) * np.float32(0.5)).astype(np.float32)
    mid_lo = ((lower + val) * np.float32(0.5)).astype(np.float32)
    r = np.where(x > val, np.where(x > mid_up, up_p, pivot), np.where(x < mid_lo, lo_p, pivot)).astype(np.int32)
    if signed:
        dec = Q[r]
        r = r + np.where((dec < 0) != (x < 0), np.where(x > 0, 1, -1), 0)
    return r


def _side(Q, signed, negative):
    """(code per bucket uint8[NB], threshold per code float32[256]) for one sign, or None."""
    idx = np.arange(NB, dtype=np.int64)
    lo_bits = np.where(idx == 0, 0, (idx + BASE) << BUCKET_SHIFT).astype(np.uint32)
    hi_bits = np.where(idx == 0, ((BASE + 1) << BUCKET_SHIFT) - 1,
                       ((idx + BASE + 1) << BUCKET_SHIFT) - 1).astype(np.uint32)
    hi_bits = np.minimum(hi_bits, np.uint32(0x3F800000))  # |x| <= 1
    sign = np.float32(-1.0 if negative else 1.0)
    f = lambda b: sign * b.view(np.float32)
    if negative:  # x < 0 strictly: the smallest |x| of bucket 0 is the smallest subnormal
        lo_bits = np.where(idx == 0, np.uint32(1), lo_bits)
    c_lo = _walk(f(lo_bits), Q, signed)
    c_hi = _walk(f(hi_bits), Q, signed)
    step = 1 if not negative else -1
    diff = (c_hi - c_lo) * step
    if np.any(diff < 0) or np.any(diff > 1):
        return None
    T = np.full(256, np.inf, np.float32)
    moving = np.nonzero(diff == 1)[0]
    if moving.size:
        lo = lo_bits[moving].astype(np.int64)
        hi = hi_bits[moving].astype(np.int64)
        target = c_hi[moving]
        # smallest bit pattern in (lo, hi] whose code is the bucket's upper code
        for _ in range(BUCKET_SHIFT + 2):
            mid = (lo + hi) // 2
            cm = _walk(f(mid.astype(np.uint32)), Q, signed)
            at = cm == target
            hi = np.where(at, mid, hi)
            lo = np.where(at, lo, mid)
        starts = c_lo[moving]
        if np.unique(starts).size != starts.size:
            return None
        T[starts] = hi.astype(np.uint32).view(np.float32)
    # every bucket edge must reproduce the walk through the table rule
    for bits in (lo_bits, hi_bits):
        ax = bits.view(np.float32)
        got = c_lo + step * (ax >= T[c_lo]).astype(np.int32)
        if not np.array_equal(got, _walk(f(bits), Q, signed)):
            return None
    if np.any(c_lo < 0) or np.any(c_lo > 255):
        return None
    return c_lo.astype(np.uint8), T


def build(Q: np.ndarray, signed: bool):
    """Tables for codebook Q (float32[256]) or None if the table rule is not exact for it.

    Returns (codes uint8[k, NB], thresholds float32[k, 256]) with k = 2 (x >= 0, x < 0)
    for a signed codebook and k = 1 for an unsigned one.
    """
    Q = np.asarray(Q, np.float32)
    if Q.shape != (256,) or not np.all(np.diff(Q) > 0):
        return None
    sides = [_side(Q, signed, False)] + ([_side(Q, signed, True)] if signed else [])
    if any(s is None for s in sides):
        return None
    return np.stack([s[0] for s in sides]), np.stack([s[1] for s in sides])


T_OFFSET = (3 * NB + 15) // 16 * 16
BLOB_BYTES = T_OFFSET + 3 * 256 * 4


def blob(qmap1, qmap2):
    """The kernel's table blob for (signed qmap1, unsigned qmap2) as uint8[BLOB_BYTES], or None
    when the table rule is not exact for these codebooks (layout in muon_sr_b200.h)."""
    s = build(np.asarray(qmap1, np.float32), True)
    u = build(np.asarray(qmap2, np.float32), False)
    if s is None or u is None:
        return None
    out = np.zeros(BLOB_BYTES, np.uint8)
    out[:3 * NB] = np.concatenate([s[0][0], s[0][1], u[0][0]])
    out[T_OFFSET:] = np.concatenate([s[1][0], s[1][1], u[1][0]]).astype(np.float32).view(np.uint8)
    return out


def lookup(x, codes, T, signed):
    """Host restatement of the kernel's table rule (used by tests)."""
    x = np.asarray(x, np.float32)
    ab = x.view(np.uint32) & np.uint32(0x7FFFFFFF)
    b = np.clip((ab >> BUCKET_SHIFT).astype(np.int64) - BASE, 0, NB - 1)
    neg = (x < 0) if signed else np.zeros(x.shape, bool)
    side = neg.astype(np.int64)
    c = codes[side, b].astype(np.int32)
    ax = ab.view(np.float32)
    hit = ax >= T[side, c]
    return np.where(neg, c - hit, c + hit)
