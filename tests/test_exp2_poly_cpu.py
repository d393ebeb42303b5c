"""The FMA-pipe exponential of the prefill softmax (``ex2_poly2`` in
lastkv_b200/csrc/common.cuh), restated bit for bit in numpy float32 and
checked against 2^x: the committed coefficients are the ones the Remez fit
below produces, and the reconstruction (round-to-nearest split, polynomial,
exponent add) stays within the fit's relative error over the whole range the
softmax feeds it (x <= 8 after the lazy max; clamped at -125)."""

import os
import re

import numpy as np

from conftest import ROOT

CSRC = os.path.join(ROOT, "lastkv_b200", "csrc")


def remez_exp2(degree: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 30):
    """2^f on f in [-0.5, 0.5] with minimax *relative* error, by the Remez exchange
    algorithm (solve for the equioscillating error on n + 2 reference points, move the
    points to the new extrema, repeat); float32 coefficients c0..c3 (the constants
    kExp2C0..kExp2C3 of common.cuh)."""
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


def _coefficients():
    src = open(os.path.join(CSRC, "common.cuh")).read()
    m = re.search(r"kExp2C0 = ([0-9.e+-]+)f, kExp2C1 = ([0-9.e+-]+)f, kExp2C2 = ([0-9.e+-]+)f, kExp2C3 = ([0-9.e+-]+)f", src)
    assert m, "coefficients not found in common.cuh"
    return np.array([float(v) for v in m.groups()], dtype=np.float32)


def _fma_f32(a, b, c):
    # a * b is exact in float64 for float32 inputs; one float64 add, then round to float32
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def ex2_poly_f32(x, c):
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    f = _fma_f32(np.full_like(x, -1.0), j, x)
    p = _fma_f32(np.full_like(x, c[3]), f, np.full_like(x, c[2]))
    p = _fma_f32(p, f, np.full_like(x, c[1]))
    p = _fma_f32(p, f, np.full_like(x, c[0]))
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_coefficients_are_the_remez_fit():
    np.testing.assert_array_equal(remez_exp2(), _coefficients())


def test_relative_error_over_the_softmax_range():
    c = _coefficients()
    rng = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
                        rng.uniform(-30.0, 8.0, 1_000_000).astype(np.float32),
                        np.array([0.0, -0.5, 0.5, -1.0, 1.0, 8.0, -125.0], dtype=np.float32)])
    got = ex2_poly_f32(x, c).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 8e-5, rel.max()
    assert np.all(np.isfinite(got)) and np.all(got > 0)


def test_clamped_inputs_give_a_negligible_weight():
    c = _coefficients()
    x = np.array([-np.inf, -1e30, -126.0, -200.0], dtype=np.float32)
    got = ex2_poly_f32(x, c)
    assert np.all(got > 0) and np.all(got < 2.0 ** -124)
