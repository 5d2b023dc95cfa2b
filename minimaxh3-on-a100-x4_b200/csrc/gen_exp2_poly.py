"""Derive the polynomial used for the FMA-pipe exp2 in h3_attn_fwd.cu.

2^x = 2^n * 2^f with n = round(x) (Cody-Waite style split, done with the 1.5*2^23 shifter)
and f = x - n in [-1/2, 1/2]. 2^f is approximated by a degree-3 polynomial whose maximum
RELATIVE error on [-1/2, 1/2] is minimised by a Remez exchange on the equioscillation
conditions. The result only feeds bf16 probabilities (relative step 2^-8), so ~1e-4 is
ample. Run:  python minimaxh3-on-a100-x4_b200/csrc/gen_exp2_poly.py
"""
import numpy as np

DEG = 3


def remez(deg=DEG, iters=30):
    n = deg + 2
    # initial reference: Chebyshev extrema on [-1/2, 1/2]
    x = 0.5 * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    for _ in range(iters):
        # solve sum c_k x^k - 2^x = (-1)^i E 2^x  (relative error equioscillation)
        A = np.zeros((n, n))
        for i, xi in enumerate(x):
            A[i, :deg + 1] = xi ** np.arange(deg + 1)
            A[i, deg + 1] = -((-1) ** i) * 2.0 ** xi
        sol = np.linalg.solve(A, 2.0 ** x)
        c = sol[:deg + 1]
        grid = np.linspace(-0.5, 0.5, 200001)
        err = (np.polyval(c[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
        # new reference: local extrema of the error (including the end points)
        idx = [0] + [i for i in range(1, len(grid) - 1)
                     if (err[i] - err[i - 1]) * (err[i + 1] - err[i]) <= 0] + [len(grid) - 1]
        if len(idx) >= n:
            # keep the n extrema with alternating signs and largest magnitude
            cand = sorted(idx, key=lambda i: grid[i])
            sel = [cand[0]]
            for i in cand[1:]:
                if np.sign(err[i]) == np.sign(err[sel[-1]]):
                    if abs(err[i]) > abs(err[sel[-1]]):
                        sel[-1] = i
                else:
                    sel.append(i)
            if len(sel) >= n:
                x = grid[sel[:n]] if len(sel) == n else grid[sorted(sel, key=lambda i: -abs(err[i]))[:n]]
                x = np.sort(x)
    return c, np.abs(err).max()


if __name__ == "__main__":
    c, e = remez()
    c32 = c.astype(np.float32)
    print("coefficients (f32):", ", ".join(f"{v:.9e}f" for v in c32))
    print(f"max relative error (exact arithmetic): {e:.3e}")
