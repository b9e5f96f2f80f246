"""Fit of the polynomial 2^f ~ c0 + c1 f + c2 f^2 + c3 f^3 + c4 f^4 on
[-0.5, 0.5] used by the attention kernel's FMA-pipe exponential
(attention_ws.cu, ex2_poly2): weighted least squares on Chebyshev nodes,
reweighted towards the largest relative error (a Remez-style iteration).
Run it to reproduce the coefficients and their float32 error."""
import numpy as np


def fit(deg=4, iters=60):
    f = np.cos(np.linspace(0, np.pi, 4001)) * 0.5
    y = np.exp2(f)
    w = 1 / y
    for _ in range(iters):
        a = np.vander(f, deg + 1, increasing=True) * w[:, None]
        c, *_ = np.linalg.lstsq(a, y * w, rcond=None)
        err = np.polyval(c[::-1], f) / y - 1
        w = w * (1 + 4 * np.abs(err) / np.abs(err).max())
    return c.astype(np.float32)


def max_rel_error(c):
    ff = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = np.zeros_like(ff) + c[-1]
    for k in range(len(c) - 2, -1, -1):
        p = (p * ff + c[k]).astype(np.float32)
    return float(np.abs(p.astype(np.float64) / np.exp2(ff.astype(np.float64)) - 1).max())


if __name__ == "__main__":
    c = fit()
    print("coefficients", [float(x) for x in c], "max relative error", max_rel_error(c))
