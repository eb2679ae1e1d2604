"""Coefficients of the degree-4 polynomial p(f) ~ 2^f on [-1/2, 1/2] used by the attention kernel's FMA-pipe exp2
(the other half of its softmax exponentials go to the MUFU ex2): a minimax fit in relative error by the Remez
exchange, computed here in float64 from the definition of 2^f; nothing else. Run: python opendecider_b200/csrc/fit_exp2.py"""
import numpy as np

DEG = 4


def remez(deg=DEG, iters=30):
    n = deg + 2
    x = 0.5 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))          # Chebyshev extrema on [-1/2, 1/2]
    grid = np.linspace(-0.5, 0.5, 200001)
    for _ in range(iters):
        # solve p(x_i) - 2^x_i = (-1)^i E 2^x_i  (relative error alternation)
        A = np.zeros((n, n))
        for i, xi in enumerate(x):
            A[i, :deg + 1] = xi ** np.arange(deg + 1)
            A[i, deg + 1] = -((-1) ** i) * 2.0 ** xi
        sol = np.linalg.solve(A, 2.0 ** x)
        c = sol[:deg + 1]
        err = (np.polyval(c[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
        # new alternation points: the extrema of the error between sign changes
        idx = [0]
        for k in range(1, grid.size - 1):
            if (err[k] - err[k - 1]) * (err[k + 1] - err[k]) <= 0:
                idx.append(k)
        idx.append(grid.size - 1)
        idx = np.array(idx)
        if idx.size >= n:
            best = idx[np.argsort(-np.abs(err[idx]))[:n]]
            x = np.sort(grid[best])
    return c, float(np.abs(err).max())


if __name__ == "__main__":
    c, e = remez()
    c32 = c.astype(np.float32)
    grid = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    p = np.zeros_like(grid)
    for ck in c32[::-1]:
        p = p * grid + ck
    e32 = float(np.abs((p.astype(np.float64) - 2.0 ** grid.astype(np.float64)) / 2.0 ** grid.astype(np.float64)).max())
    print("max relative error (float64 coefficients):", e)
    print("max relative error (float32 Horner):", e32)
    for k, ck in enumerate(c32):
        print(f"c{k} = {float(ck)!r}  # {np.float32(ck).view(np.uint32):#010x}")
