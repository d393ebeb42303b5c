"""Fit of the degree-3 polynomial behind ``ex2_poly2`` (common.cuh).

2^f on f in [-0.5, 0.5] with minimax *relative* error, by the Remez exchange
algorithm (solve for the equioscillating error on n + 2 reference points, move
the points to the new extrema, repeat).  Prints the float32 coefficients
c0..c3 and the maximum relative error of the float32 Horner evaluation.

    python lastkv_b200/csrc/exp2_poly_fit.py
"""

import numpy as np


def remez_exp2(degree: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 30):
    n = degree
    k = np.arange(n + 2)
    x = (lo + hi) / 2 + (hi - lo) / 2 * np.cos(np.pi * (n + 1 - k) / (n + 1))
    grid = np.linspace(lo, hi, 200001)
    c = None
    for _ in range(iters):
        a = np.zeros((n + 2, n + 2))
        for i in range(n + 1):
            a[:, i] = x ** i
        a[:, n + 1] = -((-1.0) ** k) * np.exp2(x)
        sol = np.linalg.solve(a, np.exp2(x))
        c = sol[:n + 1]
        err = (np.polyval(c[::-1], grid) - np.exp2(grid)) / np.exp2(grid)
        idx = [0]
        sign = np.sign(err)
        for j in range(1, len(grid)):
            if sign[j] != sign[idx[-1]]:
                idx.append(j)
            elif abs(err[j]) > abs(err[idx[-1]]):
                idx[-1] = j
        if len(idx) >= n + 2:
            best = max(range(len(idx) - (n + 1)), key=lambda s: min(abs(err[idx[s:s + n + 2]])))
            x = grid[idx[best:best + n + 2]]
    return c.astype(np.float32)


def horner_f32(c, f):
    p = np.float32(c[-1]) * np.ones_like(f, dtype=np.float32)
    for ci in c[-2::-1]:
        p = (p.astype(np.float64) * f + np.float64(ci)).astype(np.float32)
    return p


if __name__ == "__main__":
    c = remez_exp2()
    f = np.linspace(-0.5, 0.5, 1000001).astype(np.float32)
    rel = np.abs(horner_f32(c, f) - np.exp2(f.astype(np.float64))) / np.exp2(f.astype(np.float64))
    print("c0..c3 =", ", ".join("%.8g" % v for v in c), " max rel error %.3g" % rel.max())
