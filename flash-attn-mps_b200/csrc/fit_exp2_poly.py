"""Minimax polynomial for 2^f on [-1/2, 1/2] (relative error), by Remez exchange.

The prefill softmax evaluates part of its exponentials as
2^x = 2^n * p(x - n), n = round(x), on the FMA pipe instead of the MUFU unit.
This script derives p's coefficients (printed as float32 literals, constant
term pinned to 1 so that 2^0 == 1 exactly) and reports the float32 Horner error
measured against float64 exp2 on a dense grid.

    python flash-attn-mps_b200/csrc/fit_exp2_poly.py [degree]
"""

import sys

import numpy as np


def remez(deg, iters=30):
    lo, hi = -0.5, 0.5
    n = deg  # unknowns: c1..c_deg and the levelled error E (c0 = 1)
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * np.arange(n + 1)[::-1] / n)
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        # relative error r(x) = (p(x) - 2^x) / 2^x, with p(x) = 1 + sum c_k x^k
        a = np.zeros((n + 1, n + 1))
        rhs = np.zeros(n + 1)
        for i, xi in enumerate(x):
            t = 2.0 ** xi
            for k in range(1, deg + 1):
                a[i, k - 1] = xi ** k / t
            a[i, n] = (-1) ** i
            rhs[i] = 1.0 - 1.0 / t
        sol = np.linalg.solve(a, rhs)
        c = np.concatenate([[1.0], sol[:deg]])
        err = (np.polyval(c[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
        # new reference: extrema of err between sign changes
        idx = np.where(np.diff(np.sign(err)) != 0)[0]
        bounds = np.concatenate([[0], idx + 1, [len(grid)]])
        ext = [b0 + np.argmax(np.abs(err[b0:b1])) for b0, b1 in zip(bounds[:-1], bounds[1:]) if b1 > b0]
        if len(ext) != n + 1:
            break
        x = grid[ext]
    return c, np.abs(err).max()


def horner32(c, f):
    acc = np.float32(c[-1])
    for ck in c[-2::-1]:
        acc = np.float32(acc * f + np.float32(ck))
    return acc


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    c, e = remez(deg)
    c32 = [np.float32(v) for v in c]
    f = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    got = horner32(c32, f).astype(np.float64)
    rel = np.abs(got / np.exp2(f.astype(np.float64)) - 1).max()
    print(f"degree {deg}: minimax relative error {e:.3e}, float32 Horner {rel:.3e}")
    print("coefficients c0..c%d:" % deg, ", ".join(f"{float(v):.9e}f" for v in c32))
