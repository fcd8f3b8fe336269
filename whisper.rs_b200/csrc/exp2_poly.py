"""Fits the cubic used by exp2_fma2 (wattn_common.cuh), the FMA-pipe exp2.

2^x = 2^j * 2^f with j = rint(x) and f = x - j in [-1/2, 1/2]. 2^f is
approximated by p(f) = c0 + c1 f + c2 f^2 + c3 f^3 whose coefficients minimise
the maximum *relative* error on [-1/2, 1/2]: a discretised Chebyshev (minimax)
approximation solved as a linear programme (minimise t subject to
|p(f_i) - 2^f_i| <= t * 2^f_i on a dense grid). The coefficients are rounded to
f32 and the error of the f32 Horner evaluation is reported; P is stored as
bf16 (2^-9 relative) or f16 (2^-12), so an error near 1e-4 is below either.

Run: python whisper.rs_b200/csrc/exp2_poly.py
"""
import numpy as np
from scipy.optimize import linprog


def fit(degree: int = 3, n: int = 4001):
    f = np.linspace(-0.5, 0.5, n)
    y = np.exp2(f)
    V = np.vander(f, degree + 1, increasing=True)
    c = np.zeros(degree + 2)
    c[-1] = 1.0  # minimise t
    A = np.vstack([np.hstack([V, -y[:, None]]), np.hstack([-V, -y[:, None]])])
    b = np.concatenate([y, -y])
    res = linprog(c, A_ub=A, b_ub=b, bounds=[(None, None)] * (degree + 1) + [(0, None)],
                  method="highs")
    assert res.success, res.message
    return res.x[:-1].astype(np.float32), res.x[-1]


def horner_f32(coef, f):
    f = f.astype(np.float32)
    acc = np.full_like(f, coef[-1])
    for c in coef[-2::-1]:
        acc = (acc * f + np.float32(c)).astype(np.float32)
    return acc


if __name__ == "__main__":
    coef, t = fit()
    f = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    rel = np.abs(horner_f32(coef, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1)
    print("coefficients (f32):", ", ".join(f"{c:.9e}f" for c in coef))
    print(f"LP minimax relative error {t:.3e}; f32 Horner max relative error {rel.max():.3e}")
