"""Recompute the 2^f polynomial used by exp2_poly.cuh.

Remez exchange for the minimax RELATIVE error of a degree-n polynomial p
against 2^f on [-1/2, 1/2] (mpmath, 40 digits), then the coefficients
rounded to fp32 and the error of the fp32 Horner evaluation measured on a
dense grid.  Run:  python infercache_b200/csrc/exp2_poly_fit.py [degree]
"""
import sys

import mpmath as mp
import numpy as np

mp.mp.dps = 40
A, B = mp.mpf(-0.5), mp.mpf(0.5)


def rel_err(c, x):
    return sum(ck * x ** k for k, ck in enumerate(c)) / mp.power(2, x) - 1


def extrema(c, n_pts):
    """Points where the error alternates: the endpoints plus the interior
    local extrema, each refined by a ternary search."""
    grid = [A + (B - A) * i / 2000 for i in range(2001)]
    ev = [rel_err(c, x) for x in grid]
    pts = [A]
    for i in range(1, len(grid) - 1):
        if (ev[i] - ev[i - 1]) * (ev[i + 1] - ev[i]) <= 0:
            lo, hi = grid[i - 1], grid[i + 1]
            sgn = 1 if ev[i] > 0 else -1
            for _ in range(60):
                m1, m2 = lo + (hi - lo) / 3, hi - (hi - lo) / 3
                if sgn * rel_err(c, m1) < sgn * rel_err(c, m2):
                    lo = m1
                else:
                    hi = m2
            pts.append((lo + hi) / 2)
    pts.append(B)
    return pts[:n_pts] if len(pts) >= n_pts else None


def remez(deg, iters=12):
    n = deg + 2
    xs = [(A + B) / 2 - (B - A) / 2 * mp.cos(mp.pi * i / (n - 1)) for i in range(n)]
    c = None
    for _ in range(iters):
        M = mp.matrix(n, n)
        rhs = mp.matrix(n, 1)
        for i, x in enumerate(xs):
            for k in range(deg + 1):
                M[i, k] = x ** k
            M[i, deg + 1] = (-1) ** i * mp.power(2, x)
            rhs[i] = mp.power(2, x)
        sol = mp.lu_solve(M, rhs)
        c = [sol[k] for k in range(deg + 1)]
        nxt = extrema(c, n)
        if nxt is None:
            break
        xs = nxt
    return c


def fp32_horner_rel_err(c32, n=2_000_001):
    f = np.linspace(-0.5, 0.5, n).astype(np.float32)
    p = np.full_like(f, c32[-1])
    for ck in c32[-2::-1]:
        p = (p.astype(np.float64) * f.astype(np.float64) + np.float64(ck)).astype(np.float32)
    return float(np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1).max())


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 4
    c = remez(deg)
    c32 = np.array([float(x) for x in c], np.float32)
    print("degree", deg, "minimax relative error", float(max(abs(rel_err(c, x)) for x in extrema(c, deg + 2))))
    for k, v in enumerate(c32):
        print("c%d = 0x%08X  (%.8g)" % (k, v.view(np.uint32), v))
    print("fp32 Horner relative error on the grid:", fp32_horner_rel_err(c32))
