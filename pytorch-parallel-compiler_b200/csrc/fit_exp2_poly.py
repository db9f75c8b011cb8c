"""Fits the polynomial p(f) ~ 2^f on [-1/2, 1/2] used by the attention
kernel's FMA-pipe exp2 (attention_sm100.cu, exp2_poly2).

Method: 2^x = 2^n * 2^f with n = rint(x), f = x - n (Cody-Waite range
reduction); 2^f by a degree-3 polynomial fitted here by iteratively
reweighted least squares on Chebyshev nodes (Lawson's algorithm), which
converges to the minimax fit of the relative error. Prints the float32
coefficients c0..c3 and the maximum relative error of the float32
polynomial on a dense grid.

    python fit_exp2_poly.py
"""
import numpy as np


def fit(deg=3, nodes=2000, iters=200):
    k = np.arange(nodes)
    x = 0.5 * np.cos((2 * k + 1) * np.pi / (2 * nodes))
    y = 2.0 ** x
    a = np.vstack([x ** i for i in range(deg + 1)]).T / y[:, None]
    b = np.ones_like(y)
    w = np.ones(nodes)
    for _ in range(iters):
        c, *_ = np.linalg.lstsq(a * np.sqrt(w)[:, None], b * np.sqrt(w), rcond=None)
        e = np.abs(a @ c - b)
        w = w * e
        w /= w.sum()
    c32 = c.astype(np.float32)
    xs = np.linspace(-0.5, 0.5, 200001)
    p = np.zeros_like(xs)
    for ci in c32[::-1]:
        p = p * xs + float(ci)
    return c32, float(np.max(np.abs(p - 2.0 ** xs) / 2.0 ** xs))


if __name__ == "__main__":
    coef, err = fit()
    print("coefficients c0..c3:", ", ".join(f"{float(v):.9g}f" for v in coef))
    print(f"max relative error on [-1/2, 1/2]: {err:.3g}")
