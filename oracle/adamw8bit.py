"""8-bit blockwise AdamW of the reference, restated in numpy.

Follows ``muon_sr/triton_adamw_8bit.py``: ``create_dynamic_map`` (:14-25), ``_quantize``
(:27-53) and ``_adamw_8bit_kernel`` (:56-99). The codebook construction and quantiser
search are the reference's adaptation of bitsandbytes (dynamic map, quantize_2D pivot
walk); bitsandbytes itself is not installed here and is not needed: parity is anchored on
the reference's own code run under the Triton interpreter.
"""
import numpy as np

from .elementwise import sr_round
from .philox import triton_key
from .sr import bf16_to_f32

f32 = np.float32


def _fma32(a, b, c):
    """fp32 fused multiply-add: the product of two fp32 values is exact in float64, and for
    the magnitudes used here (grid points in [0.1, 1]) so is the sum, so one rounding to fp32
    gives the fused result."""
    return f32(np.float64(a) * np.float64(b) + np.float64(c))


def _linspace_f32(start, end, steps):
    """torch's fp32 ``linspace`` on the CPU: step = (end - start) / (steps - 1) in fp32; the
    first half of the points is start + step * i, the second end - step * (steps - 1 - i),
    each as one fused multiply-add (checked bit-exact against torch for 2..129 points)."""
    s, e = f32(start), f32(end)
    step = f32((e - s) / f32(steps - 1))
    half = steps // 2
    return np.array([_fma32(step, f32(i), s) if i < half else _fma32(-step, f32(steps - 1 - i), e)
                     for i in range(steps)], dtype=f32)


def create_dynamic_map(signed: bool = True) -> np.ndarray:
    """``create_dynamic_map`` -- ``triton_adamw_8bit.py:14-25``, restated in numpy: for decade
    k = 0..6 the fp32 midpoints of a ``linspace(0.1, 1)`` grid of 2^k intervals (2^(k+1) for
    the unsigned map) scaled by fp32(10^(k-6)), mirrored for the signed map, plus 0 and 1,
    sorted. Pinned against the reference's table by the golden codebooks."""
    vals = [f32(0.0), f32(1.0)]
    for k in range(7):
        grid = _linspace_f32(0.1, 1.0, (1 << (k if signed else k + 1)) + 1)
        mids = ((grid[:-1] + grid[1:]) / f32(2)).astype(f32)
        scaled = (f32(10.0 ** (k - 6)) * mids).astype(f32)
        vals.extend(scaled)
        if signed:
            vals.extend(-scaled)
    return np.sort(np.array(vals, dtype=f32))


def quantize(x, Q, signed: bool) -> np.ndarray:
    """``_quantize`` -- ``triton_adamw_8bit.py:27-53``: 7-step pivot walk from 127 with
    deltas 64..1, midpoint tie rules against the bracketing values, and for the signed map
    a +-1 fix when the decoded sign disagrees with the sign of x."""
    x = np.asarray(x, dtype=np.float32)
    Q = np.asarray(Q, dtype=np.float32)
    pivot = np.full(x.shape, 127, np.int32)
    lower_pivot = np.zeros(x.shape, np.int32)
    upper_pivot = np.full(x.shape, 255, np.int32)
    lower = np.full(x.shape, -1.0 if signed else 0.0, np.float32)
    upper = np.full(x.shape, 1.0, np.float32)
    val = Q[pivot]
    for shift in range(7):
        delta = 64 >> shift
        right = x > val
        lower_pivot = np.where(right, pivot, lower_pivot)
        upper_pivot = np.where(right, upper_pivot, pivot)
        lower = np.where(right, val, lower)
        upper = np.where(right, upper, val)
        pivot = pivot + np.where(right, delta, -delta).astype(np.int32)
        val = Q[pivot]
    mid_up = ((upper + val) * f32(0.5)).astype(f32)
    mid_lo = ((lower + val) * f32(0.5)).astype(f32)
    result = np.where(x > val,
                      np.where(x > mid_up, upper_pivot, pivot),
                      np.where(x < mid_lo, lower_pivot, pivot)).astype(np.int32)
    if signed:
        decoded = Q[result]
        mismatch = (decoded < 0) != (x < 0)
        result = result + np.where(mismatch, np.where(x > 0, 1, -1), 0)
    return result.astype(np.uint8)


def adamw8bit_coefficients(lr, beta1, beta2, eps, weight_decay, step):
    """Scalars of ``_adamw_8bit_kernel`` as the interpreter evaluates them: BC1/BC2 come
    from the host in double (:203); ``1 - B1``, ``1 - B2`` and ``1 - LR * WD`` are
    scalar-only (double, then fp32); ``tl.sqrt(BC2)`` and the products with it run in fp32.
    Returns (bc1, bc2, lr, b1, 1-b1, b2, 1-b2, eps, 1-lr*wd) as fp32."""
    return (f32(1.0 - beta1 ** step), f32(1.0 - beta2 ** step), f32(lr), f32(beta1),
            f32(1.0 - beta1), f32(beta2), f32(1.0 - beta2), f32(eps), f32(1.0 - lr * weight_decay))


def adamw8bit(p_bits, g_bits, s1, s2, absmax1, absmax2, Q1, Q2, lr, beta1, beta2, eps,
              weight_decay, step, seed, block, quantized, noise="reference"):
    """``_adamw_8bit_kernel`` -- ``triton_adamw_8bit.py:56-99``, all blocks of one tensor.

    Quantized path: s1/s2 are uint8 codes and absmax1/absmax2 fp32 per block. Otherwise
    s1/s2 are bf16 bits (SR with seed + 1 / seed + 2). BC1 = 1 - b1**step and
    BC2 = 1 - b2**step come from the host in double and are passed as fp32 (:203).
    Returns (p, s1, s2, absmax1, absmax2) with the same dtypes as the inputs. ``noise``
    selects the rounding (``elementwise.sr_round``).
    """
    n = p_bits.size
    bc1, bc2, lr32, b1, omb1, b2, omb2, eps32, decay = adamw8bit_coefficients(
        lr, beta1, beta2, eps, weight_decay, step)
    p = bf16_to_f32(p_bits)
    g = bf16_to_f32(g_bits)
    nblk = (n + block - 1) // block
    if quantized:
        blk = np.arange(n) // block
        m = (Q1[s1.astype(np.int64)] * absmax1[blk]).astype(f32)
        v = (Q2[s2.astype(np.int64)] * absmax2[blk]).astype(f32)
    else:
        m = bf16_to_f32(s1)
        v = bf16_to_f32(s2)
    with np.errstate(invalid="ignore", over="ignore"):
        finite = np.abs(g) < np.inf
        m = np.where(finite, b1 * m + omb1 * g, f32(0.0)).astype(f32)
        v = np.where(finite, b2 * v + omb2 * g * g, f32(0.0)).astype(f32)
        sq_bc2 = np.sqrt(bc2)
        coef = f32(lr32 * sq_bc2 / bc1)
        upd = (p - coef * m / (np.sqrt(v) + sq_bc2 * eps32)).astype(f32)
        updated = (upd * decay).astype(f32)
    rounded = sr_round(updated, triton_key(seed), 0, noise)
    p_out = np.where(finite, rounded, p_bits.astype(np.uint16)).astype(np.uint16)
    if quantized:
        s1o = np.empty(n, np.uint8)
        s2o = np.empty(n, np.uint8)
        a1 = np.empty(nblk, np.float32)
        a2 = np.empty(nblk, np.float32)
        for b in range(nblk):
            sl = slice(b * block, min(n, (b + 1) * block))
            mm = np.abs(m[sl]).max()
            vm = np.abs(v[sl]).max()
            s1o[sl] = quantize(m[sl] / (mm if mm > 0 else f32(1.0)), Q1, True)
            s2o[sl] = quantize(v[sl] / (vm if vm > 0 else f32(1.0)), Q2, False)
            a1[b] = mm
            a2[b] = vm
        return p_out, s1o, s2o, a1, a2
    m_sr = sr_round(m, triton_key(seed, 1), 0, noise)
    v_sr = sr_round(v, triton_key(seed, 2), 0, noise)
    return p_out, m_sr, v_sr, absmax1, absmax2
