"""Derives the coefficients of ``exp2_poly`` in common.cuh.

Method: Remez exchange (E. Ya. Remez, 1934) for the polynomial of degree ``deg``
that minimises the maximum RELATIVE error of 2^f on [-1/2, 1/2].  The kernel
reduces 2^x to 2^n * 2^f with n = round(x) (the Cody-Waite style split of
W. J. Cody and W. Waite, "Software Manual for the Elementary Functions", 1980),
so only the interval [-1/2, 1/2] matters.  The script prints the coefficients
rounded to fp32 and the error of a fp32 Horner evaluation of them.

    python attention_b200/csrc/derive_exp2_poly.py [deg]
"""

from __future__ import annotations

import sys

import numpy as np


def remez(deg: int, a: float = -0.5, b: float = 0.5, iters: int = 30):
    f = lambda x: 2.0 ** x  # noqa: E731
    n = deg + 2
    xs = 0.5 * (a + b) - 0.5 * (b - a) * np.cos(np.pi * np.arange(n) / (n - 1))
    grid = np.linspace(a, b, 200001)
    c = None
    for _ in range(iters):
        # p(x_i) + (-1)^i E f(x_i) = f(x_i): equioscillating relative error on the reference set
        m = np.zeros((n, n))
        for i, x in enumerate(xs):
            m[i, :deg + 1] = [x ** k for k in range(deg + 1)]
            m[i, deg + 1] = (-1) ** i * f(x)
        c = np.linalg.solve(m, f(xs))[:deg + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        # new reference set: the alternating local extrema of the error
        idx = [0] + [k for k in range(1, len(grid) - 1)
                     if (err[k] - err[k - 1]) * (err[k + 1] - err[k]) <= 0] + [len(grid) - 1]
        sel: list[tuple[float, float]] = []
        for x, e in zip(grid[idx], err[idx]):
            if sel and np.sign(e) == np.sign(sel[-1][1]):
                if abs(e) > abs(sel[-1][1]):
                    sel[-1] = (x, e)
            else:
                sel.append((x, e))
        while len(sel) > n:
            sel.pop(0 if abs(sel[0][1]) < abs(sel[-1][1]) else -1)
        if len(sel) < n:
            break
        xs = np.array([s[0] for s in sel])
    return c


def fp32_horner_error(c32: np.ndarray) -> float:
    x = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    p = np.full_like(x, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        p = p * x + c32[k]
    ref = 2.0 ** x.astype(np.float64)
    return float(np.max(np.abs(p.astype(np.float64) - ref) / ref))


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    c32 = remez(deg).astype(np.float32)
    for k, v in enumerate(c32):
        print(f"c{k} = {float(v)!r}f")
    print(f"max relative error (fp32 Horner): {fp32_horner_error(c32):.3e}")
