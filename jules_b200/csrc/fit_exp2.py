"""Coefficients of the degree-3 polynomial p(f) ~= 2^f on [-0.5, 0.5] used by
exp2_fma() in attn_tc.cuh (the FMA-pipe half of the softmax exponentials).

Method: Cody-Waite style split x = n + f with n = rint(x), so 2^x = 2^n * 2^f;
2^f is approximated by the polynomial minimising the maximum relative error
on [-0.5, 0.5] (iteratively reweighted least squares, a discrete Lawson
variant of the Remez exchange), then rounded to fp32.
Run: python jules_b200/csrc/fit_exp2.py
"""
import numpy as np


def fit(degree=3, iters=200):
    f = np.linspace(-0.5, 0.5, 4001)
    y = np.exp2(f)
    V = np.vander(f, degree + 1, increasing=True)
    w = np.ones_like(f)
    for _ in range(iters):
        sw = np.sqrt(w) / y  # relative error weighting
        c, *_ = np.linalg.lstsq(V * sw[:, None], y * sw, rcond=None)
        err = np.abs(V @ c - y) / y
        w = w * (err + 1e-30)
        w /= w.sum()
    c32 = c.astype(np.float32)
    err32 = np.max(np.abs((V @ c32.astype(np.float64)) - y) / y)
    return c32, err32


if __name__ == "__main__":
    c, e = fit()
    for i, v in enumerate(c):
        print(f"C{i} = {float(v)!r}f  ({np.float32(v).view(np.uint32):#010x})")
    print(f"max relative error {e:.3e}")
