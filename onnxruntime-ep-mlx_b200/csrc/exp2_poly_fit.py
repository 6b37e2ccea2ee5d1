"""Coefficients of the degree-4 polynomial for 2^f, f in [-1/2, 1/2], used by tc::exp2_poly2.

Minimax in relative error, found with Lawson's algorithm (iteratively reweighted least squares on
Chebyshev-spaced points).  Prints the fp32 coefficients and the maximum relative error of their
fp32 Horner evaluation (about 2.7e-6).  Run: python exp2_poly_fit.py
"""
import numpy as np


def fit(degree=4, points=4001, iterations=2000):
    f = np.cos(np.linspace(0.0, np.pi, points)) * 0.5
    y = 2.0 ** f
    basis = np.vander(f, degree + 1, increasing=True) / y[:, None]
    w = np.full_like(f, 1.0 / points)
    for _ in range(iterations):
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(basis * sw[:, None], sw, rcond=None)
        err = np.abs(basis @ c - 1.0)
        w = w * err
        w /= w.sum()
    return c.astype(np.float32)


def fp32_horner_error(c):
    x = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = np.full_like(x, c[-1])
    for k in range(len(c) - 2, -1, -1):
        p = (p * x + c[k]).astype(np.float32)
    return float(np.max(np.abs(p.astype(np.float64) / 2.0 ** x.astype(np.float64) - 1.0)))


if __name__ == "__main__":
    c = fit()
    print("coefficients c0..c4:", ", ".join(f"{float(v):.9g}f" for v in c))
    print("max relative error (fp32 Horner):", fp32_horner_error(c))
