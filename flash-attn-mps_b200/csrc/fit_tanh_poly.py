"""Minimax polynomial for tanh(y)/y on |y| <= Y0 (relative error), by Remez exchange.

The prefill softcap evaluates cap * tanh(s * scale / cap) for key tiles whose
scores all satisfy |s * scale / cap| <= Y0 = 3/4 as y * Q(y^2) on the FMA pipe,
with Q(v) ~ tanh(sqrt(v)) / sqrt(v) on v in [0, Y0^2] (even in y, so a polynomial in
v = y^2; constant term pinned to 1 so that tanh(y) ~ y exactly near zero).
Larger arguments keep the identity tanh(y) = 1 - 2 / (e^(2y) + 1).
This script derives Q's coefficients (printed as float32 literals) and reports
the float32 Horner error of y * Q(y^2) measured against float64 tanh on a
dense grid.

    python flash-attn-mps_b200/csrc/fit_tanh_poly.py [degree in v] [Y0]
"""

import sys

import numpy as np


def target(v):
    y = np.sqrt(v)
    out = np.ones_like(v)
    nz = y > 0
    out[nz] = np.tanh(y[nz]) / y[nz]
    return out


def remez(deg, vmax=1.0, iters=40):
    n = deg  # unknowns: c1..c_deg and the levelled error E (c0 = 1)
    # The relative error is 0 at v = 0 (c0 pinned), so the n + 1 alternation
    # points lie in (0, vmax].
    v = 0.5 * vmax * (1.0 - np.cos(np.pi * (np.arange(n + 1) + 1) / (n + 1)))
    grid = np.linspace(0.0, vmax, 200001)[1:]
    for _ in range(iters):
        # relative error r(v) = (Q(v) - f(v)) / f(v), with Q(v) = 1 + sum c_k v^k
        a = np.zeros((n + 1, n + 1))
        rhs = np.zeros(n + 1)
        f = target(v)
        for i, vi in enumerate(v):
            for k in range(1, deg + 1):
                a[i, k - 1] = vi ** k / f[i]
            a[i, n] = (-1) ** i
            rhs[i] = 1.0 - 1.0 / f[i]
        sol = np.linalg.solve(a, rhs)
        c = np.concatenate([[1.0], sol[:deg]])
        ft = target(grid)
        err = (np.polyval(c[::-1], grid) - ft) / ft
        idx = np.where(np.diff(np.sign(err)) != 0)[0]
        bounds = np.concatenate([[0], idx + 1, [len(grid)]])
        ext = [b0 + np.argmax(np.abs(err[b0:b1])) for b0, b1 in zip(bounds[:-1], bounds[1:]) if b1 > b0]
        if len(ext) != n + 1:
            break
        v = grid[ext]
    return c, np.abs(err).max()


def tanh32(c, y):
    """y * Q(y^2) in float32 Horner steps (the kernel folds the cap and scale into c)."""
    v = np.float32(y * y)
    acc = np.float32(c[-1])
    for ck in c[-2::-1]:
        acc = np.float32(acc * v + np.float32(ck))
    return np.float32(y * acc)


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 4
    y0 = float(sys.argv[2]) if len(sys.argv) > 2 else 0.75
    c, e = remez(deg, vmax=y0 * y0)
    c32 = [np.float32(x) for x in c]
    y = np.linspace(-y0, y0, 400001).astype(np.float32)
    y = y[y != 0]
    got = tanh32(c32, y).astype(np.float64)
    ref = np.tanh(y.astype(np.float64))
    print(f"|y| <= {y0}, degree {deg} in y^2: minimax relative error {e:.3e}, float32 Horner relative "
          f"{np.abs(got / ref - 1).max():.3e}, absolute {np.abs(got - ref).max():.3e}")
    print("coefficients c0..c%d:" % deg, ", ".join(f"{float(x):.9e}f" for x in c32))
