"""Coefficients of the FP32-pipe exponential in ssm.cu (exp2_poly2).

Fits p(f) ~ 2^f on [-1/2, 1/2] with the Remez exchange algorithm for minimum
RELATIVE error, rounds the coefficients to float32, and reports the error of
float32 Horner evaluation on a dense grid.  Run it to reproduce the constants:

    python mamba_tp_lite_b200/csrc/fit_exp2_poly.py [degree]

Degree 5 (the one in ssm.cu) gives 7.5e-8 in exact arithmetic and 2.4e-7 with
float32 coefficients and Horner rounding.
"""
from __future__ import annotations

import sys

import numpy as np


def remez(degree: int, iters: int = 30, lo: float = -0.5, hi: float = 0.5):
    n = degree + 2
    # Chebyshev extrema as the initial reference set
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        f = np.exp2(x)
        # p(x_i) + (-1)^i E f(x_i) = f(x_i): equioscillating relative error E
        a = np.zeros((n, n))
        for i in range(n):
            a[i, :degree + 1] = x[i] ** np.arange(degree + 1)
            a[i, degree + 1] = (-1) ** i * f[i]
        coef = np.linalg.solve(a, f)[:degree + 1]
        err = (np.polyval(coef[::-1], grid) - np.exp2(grid)) / np.exp2(grid)
        # one extremum per run of equal sign becomes the next reference set
        ext, start, sign = [], 0, np.sign(err)
        for i in range(1, len(grid) + 1):
            if i == len(grid) or sign[i] != sign[start]:
                ext.append(start + int(np.argmax(np.abs(err[start:i]))))
                start = i
        while len(ext) > n:
            ext = ext[1:] if abs(err[ext[0]]) < abs(err[ext[-1]]) else ext[:-1]
        x = grid[np.array(ext)]
    return coef, float(np.abs(err).max())


def main():
    degree = int(sys.argv[1]) if len(sys.argv) > 1 else 5
    coef, exact_err = remez(degree)
    c32 = coef.astype(np.float32)
    g = np.linspace(-0.5, 0.5, 2000001).astype(np.float32)
    p = np.full_like(g, c32[-1])
    for k in range(degree - 1, -1, -1):
        p = (p * g + c32[k]).astype(np.float32)
    rel = np.abs(p.astype(np.float64) - np.exp2(g.astype(np.float64))) / np.exp2(g.astype(np.float64))
    print(f"degree {degree}: relative error {exact_err:.3e} exact, {rel.max():.3e} float32 Horner")
    for k, v in enumerate(c32):
        print(f"  P{k} = {float(v)!r}f")


if __name__ == "__main__":
    main()
