"""Coefficients of the software 2^f used by the attention softmax (qik_attn.cu).

2^x is split as x = n + f with n = round(x) and f in [-1/2, 1/2]; 2^f is a degree-3
polynomial c0 + c1 f + c2 f^2 + c3 f^3 fitted here for least relative error by a
Remez-style iteration: weighted least squares on Chebyshev nodes, re-weighted by the
error envelope until the equioscillation settles.  The result is then 2^n added to
the exponent bits.  Run this file to print the coefficients as float32 literals and
the maximum relative error over a dense grid (float32 Horner evaluation).
"""
import numpy as np


def fit(deg: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 60):
    k = np.arange(4000)
    f = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * (k + 0.5) / len(k))
    target = np.exp2(f)
    w = np.ones_like(f)
    V = np.vander(f, deg + 1, increasing=True)
    for _ in range(iters):
        A = V / target[:, None] * w[:, None]
        c, *_ = np.linalg.lstsq(A, w, rcond=None)
        err = np.abs(V @ c / target - 1.0)
        w = w * (err / err.max() + 1e-3) ** 0.5
    return c


def horner32(c, f):
    c = c.astype(np.float32)
    p = np.full_like(f, c[-1], dtype=np.float32)
    for ci in c[-2::-1]:
        p = (p * f + ci).astype(np.float32)
    return p


if __name__ == "__main__":
    c = fit()
    grid = np.linspace(-0.5, 0.5, 2000001, dtype=np.float32)
    rel = np.abs(horner32(c, grid).astype(np.float64) / np.exp2(grid.astype(np.float64)) - 1.0)
    for i, ci in enumerate(np.float32(c)):
        print(f"c{i} = {float(ci).hex()}  ({ci!r})")
    print(f"max relative error {rel.max():.3e} (2^{np.log2(rel.max()):.2f})")
