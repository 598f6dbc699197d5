"""Fit the polynomial used by the FMA-pipe exp2 (exp2_fma_x2 in ptx.cuh).

2^x is split as 2^j * 2^r with j = round(x) (round-to-nearest via the
1.5 * 2^23 addition trick, so r lies in [-0.5, 0.5]) and 2^r approximated by a
degree-3 polynomial whose maximum RELATIVE error on [-0.5, 0.5] is minimised
with the Remez exchange algorithm (equioscillating error at n + 2 points).
The fit is done in float64; the coefficients are then rounded to fp32 and the
error of the rounded polynomial, evaluated with fp32 Horner steps, is reported.

    python benchmark_b200/csrc/fit_exp2_poly.py
"""
from __future__ import annotations

import numpy as np


def remez_relative(deg: int = 3, lo: float = -0.5, hi: float = 0.5, iters: int = 30):
    f = np.exp2
    n = deg + 2
    k = np.arange(n)
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * -np.cos(np.pi * k / (n - 1))  # Chebyshev extrema
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        # p(x_i) - f(x_i) = (-1)^i * E * f(x_i)
        A = np.zeros((n, n))
        for i in range(n):
            A[i, :deg + 1] = x[i] ** np.arange(deg + 1)
            A[i, deg + 1] = -((-1) ** i) * f(x[i])
        c = np.linalg.solve(A, f(x))[:deg + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        # new reference set: the extremum of each sign run of the error
        idx = np.flatnonzero(np.diff(np.sign(err)) != 0)
        bounds = np.concatenate(([0], idx + 1, [len(grid)]))
        ext = [b0 + int(np.argmax(np.abs(err[b0:b1]))) for b0, b1 in zip(bounds[:-1], bounds[1:])]
        if len(ext) < n:
            break
        while len(ext) > n:  # keep n alternating extrema, dropping the smaller end
            ext.pop(0 if abs(err[ext[0]]) < abs(err[ext[-1]]) else len(ext) - 1)
        x = grid[ext]
    return c, float(np.max(np.abs(err)))


def fp32_horner_error(c32: np.ndarray) -> float:
    r = np.linspace(-0.5, 0.5, 1000001).astype(np.float32)
    p = np.float32(c32[3])
    for ci in (c32[2], c32[1], c32[0]):
        p = (p * r + np.float32(ci)).astype(np.float32)
    return float(np.max(np.abs(p.astype(np.float64) / np.exp2(r.astype(np.float64)) - 1.0)))


if __name__ == "__main__":
    c, e = remez_relative()
    c32 = c.astype(np.float32)
    print("coefficients c0..c3 as fp32 literals:", [repr(float(v)) for v in c32])
    print(f"minimax relative error (float64 fit): {e:.3e}")
    print(f"relative error, fp32 coefficients + fp32 Horner: {fp32_horner_error(c32):.3e}")
