"""Derive the coefficients of ``exp2_poly2`` (bsa_common.cuh): the degree-3
polynomial p with minimal maximum *relative* error |p(f) / 2^f - 1| on
f in [-1/2, 1/2], by the Remez exchange algorithm (float64, numpy).

    python dit_sparse_atten_b200/csrc/fit_exp2_poly.py

prints the coefficients (constant term first), the float32 values the kernel
uses, and the achieved maximum relative error (about 7.5e-5).
"""

from __future__ import annotations

import numpy as np

DEGREE = 3
LO, HI = -0.5, 0.5


def remez(degree=DEGREE, iterations=30):
    n = degree + 2
    # Chebyshev extrema as the first reference set
    x = 0.5 * (LO + HI) + 0.5 * (HI - LO) * -np.cos(np.pi * np.arange(n) / (n - 1))
    grid = np.linspace(LO, HI, 200001)
    for _ in range(iterations):
        # p(x_i) - 2^x_i = (-1)^i E 2^x_i  (equioscillating relative error)
        a = np.zeros((n, n))
        for i, xi in enumerate(x):
            a[i, :degree + 1] = xi ** np.arange(degree + 1)
            a[i, degree + 1] = -((-1) ** i) * 2.0 ** xi
        sol = np.linalg.solve(a, 2.0 ** x)
        coef = sol[:degree + 1]
        err = np.polyval(coef[::-1], grid) / 2.0 ** grid - 1
        # new reference: the extremum of each sign-alternating segment
        sign = np.sign(err)
        cuts = np.flatnonzero(np.diff(sign)) + 1
        segments = np.split(np.arange(grid.size), cuts)
        if len(segments) < n:
            break
        extrema = [seg[np.argmax(np.abs(err[seg]))] for seg in segments]
        while len(extrema) > n:   # drop the smallest end extremum
            drop = 0 if abs(err[extrema[0]]) < abs(err[extrema[-1]]) else -1
            extrema.pop(drop)
        x = grid[extrema]
    err = np.polyval(coef[::-1], grid) / 2.0 ** grid - 1
    return coef, float(np.abs(err).max())


if __name__ == "__main__":
    coef, max_rel = remez()
    print("coefficients c0..c3:", ", ".join(f"{c:.10f}" for c in coef))
    print("float32:            ", ", ".join(repr(float(np.float32(c))) for c in coef))
    print(f"max relative error:  {max_rel:.3e}")
