"""Coefficients of the polynomial erf used by the GEMM's GELU epilogue.

erf(z) is approximated on [-Z, Z] (Z = 2.9) as z * P(z^2), P of degree 9,
by weighted least squares on Chebyshev nodes (weight z, so the absolute error
of erf is levelled); |z| is clamped to Z, where 1 - erf(Z) = 4.1e-5.  The
script prints the coefficients (lowest degree first) and the maximum
absolute error of a float32 Horner evaluation against scipy's erf.

    python mergenet_b200/csrc/gelu_fit.py
"""
import numpy as np
import scipy.special as sp

Z, DEG = 2.9, 9


def fit():
    z = np.cos(np.linspace(0, np.pi, 6000)) * Z / 2 + Z / 2
    y = np.where(z == 0, 2 / np.sqrt(np.pi), sp.erf(z) / np.where(z == 0, 1, z))
    v = np.vander(z * z, DEG + 1, increasing=True)
    w = np.maximum(z, 1e-3)
    c, *_ = np.linalg.lstsq(v * w[:, None], y * w, rcond=None)
    return c.astype(np.float32)


def max_error(c):
    zz = np.linspace(-6, 6, 1200001)
    zc = np.clip(zz, -Z, Z).astype(np.float32)
    u = (zc * zc).astype(np.float32)
    acc = np.full_like(u, c[-1])
    for k in range(DEG - 1, -1, -1):
        acc = (acc * u + c[k]).astype(np.float32)
    return float(np.abs((zc * acc).astype(np.float64) - sp.erf(zz)).max())


if __name__ == "__main__":
    c = fit()
    print("coefficients:", ", ".join(f"{float(v):.9e}f" for v in c))
    print(f"max |erf error| on [-6, 6] (float32, clamped): {max_error(c):.2e}")
