"""Derive the cubic used by the kernels' FMA-pipe exp2 (Remez exchange).

2^x is split as 2^n * 2^f with n = round(x) and f in [-1/2, 1/2]; 2^f is
approximated by c0 + c1 f + c2 f^2 + c3 f^3 whose coefficients minimise the
maximum *relative* error on [-1/2, 1/2] (minimax, found with the classical
Remez exchange algorithm on the weighted error (p(f) - 2^f) / 2^f).  Run this
file to reprint the coefficients and the error bound that ffa_common.cuh
quotes.
"""
import numpy as np


def remez(deg=3, lo=-0.5, hi=0.5, iters=30):
    n = deg + 2
    # Chebyshev extrema as the initial reference
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(lo, hi, 200001)
    for _ in range(iters):
        f = np.exp2(x)
        # p(x_i) + (-1)^i E f(x_i) = f(x_i)
        A = np.zeros((n, n))
        for j in range(deg + 1):
            A[:, j] = x ** j
        A[:, deg + 1] = (-1.0) ** np.arange(n) * f
        sol = np.linalg.solve(A, f)
        c = sol[:deg + 1]
        err = (np.polyval(c[::-1], grid) - np.exp2(grid)) / np.exp2(grid)
        # new reference: extrema of the error between sign changes
        s = np.sign(err)
        idx = np.concatenate(([0], np.nonzero(np.diff(s))[0] + 1, [len(grid)]))
        ext = [seg[np.argmax(np.abs(err[seg]))] for seg in (np.arange(a, b) for a, b in zip(idx[:-1], idx[1:]))]
        if len(ext) != n:
            break
        x = grid[ext]
    return c, np.abs(err).max()


if __name__ == "__main__":
    c, e = remez()
    c32 = c.astype(np.float32)
    print("coefficients (c0..c3):", ", ".join(f"{v:.9e}f" for v in c32))
    print(f"max relative error on [-1/2, 1/2]: {e:.3e}")
