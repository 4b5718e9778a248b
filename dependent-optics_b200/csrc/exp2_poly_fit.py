"""Coefficients of exp2_poly2 (tc_ptx.cuh): a degree-3 polynomial for 2^f on
[-1/2, 1/2] that minimises the maximum relative error, by Lawson's
iteratively reweighted least squares on a dense grid.  Prints the
coefficients (highest degree first) and the maximum relative error of their
fp32 Horner evaluation.

    python dependent-optics_b200/csrc/exp2_poly_fit.py
"""
import numpy as np


def fit(deg: int = 3, iters: int = 60):
    f = np.linspace(-0.5, 0.5, 20001)
    y = 2.0 ** f
    w = 1.0 / y
    c = np.polyfit(f, y, deg, w=w)
    for _ in range(iters):
        err = (np.polyval(c, f) - y) / y
        w = w * np.sqrt(np.abs(err) + 1e-18)
        w /= w.max()
        c = np.polyfit(f, y, deg, w=w / y)
    c32 = c.astype(np.float32)
    p = np.full_like(f, c32[0], dtype=np.float32)
    for k in c32[1:]:
        p = (p * f.astype(np.float32) + k).astype(np.float32)
    return c32, float(np.abs((p.astype(np.float64) - y) / y).max())


if __name__ == "__main__":
    c, e = fit()
    print("coefficients (c3, c2, c1, c0):", [repr(float(x)) for x in c])
    print("max relative error (fp32 Horner):", e)
