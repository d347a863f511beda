"""Fit the coefficients of the FMA-pipe exp2 used by the attention kernel.

The kernel evaluates 2**x as 2**j * p(f) with j = round(x) and
f = x - j in [-0.5, 0.5]; p is a polynomial of small degree whose maximum
RELATIVE error on [-0.5, 0.5] is minimised with the Remez exchange algorithm
(equioscillation of the weighted error p(f)/2**f - 1 at degree+2 points).
The coefficients are rounded to float32 and the error is re-measured in
float32 Horner arithmetic, which is what the kernel does.

Run:  python llm_fa_b200/csrc/fit_exp2_poly.py [degree]
The printed constants are pasted into softmax_exp2.cuh.
"""
import sys

import numpy as np


def remez_exp2(deg: int, lo: float = -0.5, hi: float = 0.5, iters: int = 60):
    n = deg + 2
    # Chebyshev extrema as the initial reference set.
    k = np.arange(n)
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * k[::-1] / (n - 1))
    grid = np.linspace(lo, hi, 200001)
    f_grid = np.exp2(grid)
    c = None
    for _ in range(iters):
        # Solve p(x_i) - f(x_i) = (-1)^i E f(x_i)  (relative error weight 1/f).
        fx = np.exp2(x)
        A = np.zeros((n, n))
        for j in range(deg + 1):
            A[:, j] = x ** j
        A[:, deg + 1] = -((-1.0) ** k) * fx
        sol = np.linalg.solve(A, fx)
        c = sol[: deg + 1]
        err = np.polyval(c[::-1], grid) / f_grid - 1.0
        # New reference: extrema of err on each sign-alternating segment.
        sign = np.sign(err)
        sign[sign == 0] = 1
        idx = np.flatnonzero(np.diff(sign) != 0)
        bounds = np.concatenate(([0], idx + 1, [len(grid)]))
        ext = []
        for a, b in zip(bounds[:-1], bounds[1:]):
            seg = np.abs(err[a:b])
            ext.append(a + int(np.argmax(seg)))
        ext = np.array(ext)
        if len(ext) > n:  # keep the n largest consecutive alternations
            while len(ext) > n:
                if abs(err[ext[0]]) < abs(err[ext[-1]]):
                    ext = ext[1:]
                else:
                    ext = ext[:-1]
        if len(ext) < n:
            break
        x = grid[ext]
    return c


def f32_horner_rel_err(c, lo=-0.5, hi=0.5):
    f = np.linspace(lo, hi, 400001).astype(np.float32)
    cf = [np.float32(v) for v in c]
    p = np.full_like(f, cf[-1])
    for v in cf[-2::-1]:
        p = (p * f + v).astype(np.float32)
    return float(np.max(np.abs(p.astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0)))


if __name__ == "__main__":
    deg = int(sys.argv[1]) if len(sys.argv) > 1 else 3
    c = remez_exp2(deg)
    print(f"degree {deg}, float32 Horner max relative error = {f32_horner_rel_err(c):.3e}")
    for i, v in enumerate(c):
        print(f"  c{i} = {np.float32(v)!r}  ({float(np.float32(v)).hex()})")
