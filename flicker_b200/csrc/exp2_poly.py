"""Derive the polynomial used for 2^f, f in [-1/2, 1/2], in the attend kernel's FMA-pipe exp.

    python flicker_b200/csrc/exp2_poly.py [degree]

Method: Remez exchange for the minimax RELATIVE error of p(f) ~ 2^f (Remez, 1934;
the form in Muller, "Elementary Functions", ch. 3), started from Chebyshev nodes,
with the constant term pinned to 1 so p(0) = 1 exactly. The kernel evaluates
2^x = p(x - round(x)) * 2^round(x), the scaling done by adding round(x) << 23 to
the float's bits. The printed coefficients are pasted into ptx.cuh (kExp2C*);
the script also prints the max relative error in fp64 and after fp32 Horner.
"""
from __future__ import annotations

import sys

import numpy as np


def remez_rel(degree: int, iters: int = 40):
    lo, hi = -0.5, 0.5
    n = degree  # unknowns c1..cn plus the levelled error E
    k = np.arange(n + 1)
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * (n - k) / n)  # n+1 reference points
    for _ in range(iters):
        # p(x) = 1 + sum c_i x^i ;  (p(x) - 2^x) / 2^x = (-1)^k E
        a = np.zeros((n + 1, n + 1))
        b = np.zeros(n + 1)
        t = np.exp2(x)
        for r in range(n + 1):
            for i in range(1, n + 1):
                a[r, i - 1] = x[r] ** i / t[r]
            a[r, n] = -((-1) ** r)
            b[r] = 1.0 - 1.0 / t[r]
        sol = np.linalg.solve(a, b)
        c = np.concatenate([[1.0], sol[:n]])
        grid = np.linspace(lo, hi, 200001)
        err = np.polyval(c[::-1], grid) / np.exp2(grid) - 1.0
        # new reference set: extrema of err between sign changes
        idx = [0]
        for i in range(1, len(grid) - 1):
            if (err[i] - err[i - 1]) * (err[i + 1] - err[i]) <= 0:
                idx.append(i)
        idx.append(len(grid) - 1)
        idx = np.array(sorted(set(idx)))
        ext = idx[np.argsort(-np.abs(err[idx]))][: n + 1]
        x = np.sort(grid[ext])
    return c, float(np.max(np.abs(err)))


def fp32_error(c):
    f = np.linspace(-0.5, 0.5, 400001).astype(np.float32)
    cc = [np.float32(v) for v in c]
    p = np.full_like(f, cc[-1])
    for v in cc[-2::-1]:
        p = (p * f + v).astype(np.float32)
    return float(np.max(np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)))


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 4
    coeffs, e = remez_rel(deg)
    print(f"degree {deg}: minimax relative error {e:.3e} (fp64), {fp32_error(coeffs):.3e} (fp32 Horner)")
    for i, v in enumerate(coeffs):
        print(f"  c{i} = {np.float32(v).item()!r}f")
