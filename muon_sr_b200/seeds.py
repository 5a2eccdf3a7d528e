"""Seeds and Philox keys, with the reference's formulas.

* ``deterministic_seed`` -- ``muon_sr/triton_muon_sr.py:83-85`` (the AdamW and 8-bit
  optimizers use the same formula with salt 0: ``triton_adamw.py:97``,
  ``triton_adamw_8bit.py:197``).
* ``triton_key`` -- the 64-bit Philox key a Triton kernel derives from a Python int seed
  plus an in-kernel constant: Triton types ints in [-2^31, 2^31) as i32 (so ``seed + 1``
  wraps in 32 bits and is sign-extended when widened to the 64-bit key) and larger ones as
  i64 (``triton/language/random.py:47-57``).
"""


def deterministic_seed(step: int, param_idx: int, salt: int = 0) -> int:
    return (step * 2654435761 ^ param_idx * 1234567891 ^ salt) & 0xFFFFFFFF


def triton_key(seed: int, add: int = 0) -> int:
    if -(1 << 31) <= seed < (1 << 31):
        v = (seed + add + (1 << 31)) % (1 << 32) - (1 << 31)
    else:
        v = seed + add
    return v & 0xFFFFFFFFFFFFFFFF
