"""Derives the exp polynomial of vs_math.h (vs_expf_core).

e^r is approximated on |r| <= ln2/2 (slightly widened) by
1 + r + c2 r^2 + c3 r^3 + c4 r^4 + c5 r^5, keeping the constant and linear
terms exact (e^0 = 1) and choosing c2..c5 to minimise the largest RELATIVE
error over a dense grid.  Relative error is linear in the coefficients, so the
minimax problem is a linear program: minimise t subject to
|(1 + r + sum c_k r^k - e^r) / e^r| <= t at every grid point.  The f32
roundings of the printed coefficients are the constants in vs_math.h.

    python vauss_b200/csrc/exp_minimax.py
"""
import numpy as np
from scipy.optimize import linprog


def fit(degree: int = 5, points: int = 4001):
    h = np.log(2.0) / 2 * 1.0005
    r = np.linspace(-h, h, points)
    e = np.exp(r)
    a = np.stack([r ** k / e for k in range(2, degree + 1)], axis=1)
    b = (e - 1 - r) / e
    nv = a.shape[1]
    a_ub = np.vstack([np.hstack([a, -np.ones((points, 1))]), np.hstack([-a, -np.ones((points, 1))])])
    b_ub = np.concatenate([b, -b])
    cost = np.zeros(nv + 1)
    cost[-1] = 1.0
    res = linprog(cost, A_ub=a_ub, b_ub=b_ub, bounds=[(None, None)] * nv + [(0, None)], method="highs")
    assert res.success, res.message
    return res.x[:nv], res.x[-1]


if __name__ == "__main__":
    coef, err = fit()
    print(f"largest relative error before f32 rounding: {err:.3g}")
    for k, c in zip(range(2, 6), coef):
        print(f"c{k} = {np.float32(c).item()!r}")
