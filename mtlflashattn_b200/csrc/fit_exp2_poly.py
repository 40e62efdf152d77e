"""Derives the polynomial the attention kernel uses to evaluate part of its exp2 on the FMA
pipe instead of the MUFU unit (exp2_poly2 in ptx.cuh).

Method: Cody-Waite style range reduction x = n + f with n = round(x), f in [-1/2, 1/2], so
2^x = 2^n * 2^f; 2^f is approximated by a degree-3 polynomial whose coefficients come from a
Remez exchange minimising the maximum RELATIVE error on [-1/2, 1/2] (relative, because the
result multiplies probabilities that are then rounded to bf16/fp16 with 2^-9 / 2^-11
relative precision). Run it to print the coefficients and the achieved error bound:

    python mtlflashattn_b200/csrc/fit_exp2_poly.py
"""
import numpy as np


def remez_relative(deg, a=-0.5, b=0.5, iters=30):
    f = np.exp2
    n = deg + 2
    x = (a + b) / 2 + (b - a) / 2 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(a, b, 200001)
    for _ in range(iters):
        # p(x_i) + (-1)^i E f(x_i) = f(x_i): solve for the coefficients and the level E
        A = np.zeros((n, n))
        for i, xi in enumerate(x):
            A[i, :deg + 1] = xi ** np.arange(deg + 1)
            A[i, deg + 1] = (-1) ** i * f(xi)
        c = np.linalg.solve(A, f(x))[:deg + 1]
        err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
        idx = np.where(np.diff(np.sign(err)) != 0)[0]
        bounds = np.concatenate([[0], idx + 1, [len(grid)]])
        ext = [seg[np.argmax(np.abs(err[seg]))] for seg in
               (np.arange(bounds[i], bounds[i + 1]) for i in range(len(bounds) - 1))]
        if len(ext) != n:
            break
        x = grid[ext]
    return c, np.max(np.abs(err))


if __name__ == "__main__":
    c, e = remez_relative(3)
    for i, ci in enumerate(c):
        print(f"c{i} = {np.float32(ci)!r}  ({ci:.10e})")
    print(f"max relative error on [-1/2, 1/2]: {e:.3e} (2^{np.log2(e):.2f})")
    c32 = c.astype(np.float32)
    xs = np.linspace(-0.5, 0.5, 100001, dtype=np.float32)
    p = ((c32[3] * xs + c32[2]) * xs + c32[1]) * xs + c32[0]
    print(f"float32 Horner max relative error: {np.max(np.abs(p / np.exp2(xs.astype(np.float64)) - 1)):.3e}")
