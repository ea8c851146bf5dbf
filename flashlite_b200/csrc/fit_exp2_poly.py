"""Fit the cubic used by the FMA-pipe exp2 in fl_ptx.cuh (exp2_poly2).

2^x = 2^floor(x) * 2^f with f = x - floor(x) in [0, 1) (Cody-Waite style
split by an integer). 2^f is approximated by

    p(f) = 1 + f * (c1 + f * (c2 + f * c3)),   c3 = 1 - c1 - c2,

so that p(0) = 1 and p(1) = 2 hold exactly (no jump where floor(x) changes).
(c1, c2) minimise the maximum relative error max |p(f) / 2^f - 1| on a dense
grid of [0, 1] (Nelder-Mead on the minimax objective, started from the
least-squares solution). Coefficients are rounded to fp32 and the error is
re-evaluated in fp32 Horner arithmetic.

Run: python flashlite_b200/csrc/fit_exp2_poly.py
"""
import numpy as np
from scipy.optimize import minimize


def rel_err(c, f):
    c1, c2 = c
    c3 = 1.0 - c1 - c2
    p = 1.0 + f * (c1 + f * (c2 + f * c3))
    return np.abs(p / np.exp2(f) - 1.0)


def main():
    f = np.linspace(0.0, 1.0, 200001)
    # least-squares start on the constrained form
    A = np.stack([f - f ** 3, f ** 2 - f ** 3], axis=1)
    b = (np.exp2(f) - 1.0 - f ** 3) / np.exp2(f)
    x0, *_ = np.linalg.lstsq(A / np.exp2(f)[:, None], b, rcond=None)
    res = minimize(lambda c: rel_err(c, f).max(), x0, method="Nelder-Mead",
                   options={"xatol": 1e-12, "fatol": 1e-14, "maxiter": 20000})
    c1, c2 = res.x
    c3 = 1.0 - c1 - c2
    c32 = np.float32([c1, c2, c3])
    ff = f.astype(np.float32)
    p32 = np.float32(1.0) + ff * (c32[0] + ff * (c32[1] + ff * c32[2]))
    err32 = np.abs(p32.astype(np.float64) / np.exp2(f) - 1.0).max()
    print(f"c1 = {c32[0]!r}f\nc2 = {c32[1]!r}f\nc3 = {c32[2]!r}f")
    print(f"max relative error: {rel_err(res.x, f).max():.3e} (float64), {err32:.3e} (fp32 Horner)")


if __name__ == "__main__":
    main()
