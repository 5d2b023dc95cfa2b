"""The FMA-pipe exp2 of the attention kernel (ex2_poly in h3_ptx.cuh), emulated
operation by operation in fp32: relative error well under bf16's rounding step, exact
zero below the clamp, and the coefficient derivation reproduces the constants used."""
import os
import re
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "minimaxh3-on-a100-x4_b200", "csrc")
f32 = np.float32


def _coeffs():
    src = open(os.path.join(CSRC, "h3_ptx.cuh")).read()
    start = src.index("float ex2_poly(")
    body = src[start:src.index("\n}\n", start)]
    return [f32(x) for x in re.findall(r"(-?\d\.\d+e[-+]\d+)f", body)]


def ex2_poly(x):
    c3, c2, c1, c0 = _coeffs()
    x = np.asarray(x, f32)
    xc = np.maximum(x, f32(-125.0))
    sh = f32(12582912.0)
    t = (xc + sh).astype(f32)
    n = (t - sh).astype(f32)
    f = (xc - n).astype(f32)
    # fmaf: single rounding of a*b+c -- emulate in float64 then round (exact for these sizes)
    fma = lambda a, b, c: (a.astype(np.float64) * b + c).astype(f32)
    q = fma(np.full_like(f, c3), f, c2)
    q = fma(q, f, c1)
    q = fma(q, f, c0)
    ni = t.view(np.int32) - np.int32(0x4B400000)
    r = (q.view(np.int32) + (ni << 23)).view(f32)
    return np.where(x < -125.0, f32(0), r)


def test_relative_error_bound():
    x = np.linspace(-125, 8, 2_000_001, dtype=f32)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(ex2_poly(x) - ref) / ref
    assert rel.max() < 1.0e-4


def test_masked_and_extremes():
    assert ex2_poly(np.array([-np.inf, -1e30, -125.5], f32)).tolist() == [0.0, 0.0, 0.0]
    assert ex2_poly(np.array([0.0], f32))[0] == np.float32(0.9999280572)  # c0 exactly
    assert np.isfinite(ex2_poly(np.array([8.0], f32))).all()


def test_coefficients_match_derivation():
    out = subprocess.run([sys.executable, os.path.join(CSRC, "gen_exp2_poly.py")], capture_output=True,
                         text=True, check=True).stdout
    derived = [f32(float(v.rstrip("f,"))) for v in re.search(r"\(f32\): (.*)", out).group(1).split(", ")]
    c3, c2, c1, c0 = _coeffs()
    assert derived == [c0, c1, c2, c3]
