"""Derive the polynomial used for the FMA-pipe exp2 in h3_ptx.cuh (ex2_poly2).

2^x = 2^n * 2^f with n = floor(x) (taken with the 1.5*2^23 shifter under round-toward-minus-
infinity) and f = x - n in [0, 1). 2^f is approximated by p(f) = 1 + c1 f + c2 f^2 + c3 f^3:
the constant term is exactly 1 so that p(0) = 1 (x = -127 after the clamp, i.e. a masked key,
then gives exactly +0 once n is added into the exponent field). c1..c3 minimise the maximum
RELATIVE error |p(f) / 2^f - 1| over [0, 1], found as a linear programme on a dense grid
(minimise E subject to -E <= p(f_i)/2^f_i - 1 <= E), then rounded to fp32. The result only
feeds bf16 probabilities (relative step 2^-8), so ~1e-4 is ample. Run:
    python minimaxh3-on-a100-x4_b200/csrc/gen_exp2_poly.py
"""
import numpy as np
from scipy.optimize import linprog

DEG = 3


def fit(deg: int = DEG, points: int = 4001):
    f = np.linspace(0.0, 1.0, points)
    w = 2.0 ** -f                                   # relative error weight
    powers = np.stack([f ** k for k in range(1, deg + 1)], axis=1) * w[:, None]
    base = w - 1.0                                  # p(f)/2^f - 1 = base + sum c_k f^k / 2^f
    # variables: c1..c_deg, E ; minimise E
    n = deg + 1
    cost = np.zeros(n)
    cost[-1] = 1.0
    a_ub = np.vstack([np.hstack([powers, -np.ones((points, 1))]),
                      np.hstack([-powers, -np.ones((points, 1))])])
    b_ub = np.concatenate([-base, base])
    res = linprog(cost, A_ub=a_ub, b_ub=b_ub, bounds=[(None, None)] * n, method="highs")
    if not res.success:
        raise RuntimeError(res.message)
    return res.x[:deg], res.x[deg]


def max_rel_error_f32(c):
    """Maximum relative error with fp32 Horner evaluation (each FMA rounded once)."""
    f = np.linspace(0.0, 1.0, 200001, dtype=np.float32)[:-1]
    c1, c2, c3 = (np.float32(v) for v in c)
    q = (c3.astype(np.float64) * f + c2).astype(np.float32)
    q = (q.astype(np.float64) * f + c1).astype(np.float32)
    q = (q.astype(np.float64) * f + 1.0).astype(np.float32)
    return float(np.max(np.abs(q / np.exp2(f.astype(np.float64)) - 1.0)))


if __name__ == "__main__":
    c, e = fit()
    c32 = c.astype(np.float32)
    print("coefficients c1..c3 (f32):", ", ".join(f"{v:.9e}f" for v in c32))
    print(f"max relative error: {e:.3e} (exact arithmetic), {max_rel_error_f32(c32):.3e} (fp32 Horner)")
