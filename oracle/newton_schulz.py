"""Newton-Schulz quintic orthogonalisation, restated with torch bf16 ops on the CPU.

Follows ``_newton_schulz`` -- ``muon_sr/muon_sr.py:82-98`` op for op: X = bf16(G); if
rows > cols work on X^T; X /= (||X||_F + 1e-7) per matrix; ``steps`` times
{A = X X^T; B = b A + c (A A); X = a X + B X} with (a, b, c) = (3.4445, -4.7750, 2.0315),
every torch op rounding to bf16; transpose back. The reference runs the same torch ops on
the GPU through cuBLAS; on the CPU torch uses its own bf16 GEMM, so two runs of the
reference itself on different devices agree only to within a few 1e-3 in relative
Frobenius norm. The engine's gate is the north-star tolerance of 1e-2.
"""
import torch

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def newton_schulz(G: torch.Tensor, steps: int = 5, out_dtype=None) -> torch.Tensor:
    assert G.ndim >= 2
    a, b, c = NS_COEFFS
    X = G.bfloat16()
    transposed = X.size(-2) > X.size(-1)
    if transposed:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if transposed:
        X = X.mT
    return X if out_dtype is None else X.to(out_dtype)


def ns_flops(rows: int, cols: int, steps: int = 5) -> int:
    """Algorithmic FLOPs of one matrix: per step 2 m^2 n (X X^T) + 2 m^3 (A A) + 2 m^2 n
    (B X) with m = min(rows, cols), n = max(rows, cols)."""
    m, n = min(rows, cols), max(rows, cols)
    return steps * (4 * m * m * n + 2 * m ** 3)


def rel_frobenius(x: torch.Tensor, ref: torch.Tensor) -> float:
    x = x.float()
    ref = ref.float()
    return float((x - ref).norm() / ref.norm().clamp_min(1e-30))
