"""The FMA-pipe exp2 of the attention kernel (ex2_poly2 in h3_ptx.cuh), emulated operation by
operation in fp32: relative error well under bf16's rounding step, exact zero for masked keys,
valid numbers down to the clamp, and the coefficient derivation reproduces the constants used."""
import os
import re
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "minimaxh3-on-a100-x4_b200", "csrc")
f32 = np.float32


def _coeffs():
    """c3, c2, c1 from the kernel source (their float comments beside the bit patterns)."""
    src = open(os.path.join(CSRC, "h3_ptx.cuh")).read()
    start = src.index("void ex2_poly2(")
    body = src[start:src.index("\n}\n", start)]
    consts = {}
    for name, hexbits, comment in re.findall(r"const uint64_t (k\d) = 0x([0-9A-F]{8})\2ull;\s*// (\S+)f", body):
        val = np.array([int(hexbits, 16)], np.uint32).view(f32)[0]
        assert val == f32(float(comment)), (name, val, comment)
        consts[name] = val
    return consts["k3"], consts["k2"], consts["k1"]


def _fma(a, b, c):
    # one rounding of a*b+c: float64 holds the exact product of two fp32 values
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(f32)


def ex2_poly2(x):
    c3, c2, c1 = _coeffs()
    x = np.asarray(x, f32)
    xc = np.maximum(x, f32(-127.0))
    sh = f32(12582912.0)
    t = np.floor(xc.astype(np.float64) + np.float64(sh)).astype(f32)  # add.rm: exact sum rounded down
    n = (t - sh).astype(f32)
    f = (xc - n).astype(f32)
    q = _fma(np.full_like(f, c3), f, c2)
    q = _fma(q, f, c1)
    q = _fma(q, f, f32(1.0))
    r = (q.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << np.uint64(23)))
    return (r & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(f32)


def test_relative_error_bound():
    x = np.linspace(-120, 8, 2_000_001, dtype=f32)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(ex2_poly2(x).astype(np.float64) - ref) / ref
    assert rel.max() < 1.0e-4


def test_masked_keys_and_underflow():
    got = ex2_poly2(np.array([-np.inf, -1e30, -127.0], f32))
    assert got.tolist() == [0.0, 0.0, 0.0]
    tiny = ex2_poly2(np.array([-126.5, -126.0], f32))  # subnormal / smallest normal, never wrapped
    assert np.all(tiny >= 0) and np.all(tiny < 2.0 ** -125)
    assert ex2_poly2(np.array([0.0], f32))[0] == f32(1.0)
    assert np.isfinite(ex2_poly2(np.array([8.0], f32))).all()


def test_coefficients_match_derivation():
    out = subprocess.run([sys.executable, os.path.join(CSRC, "gen_exp2_poly.py")], capture_output=True,
                         text=True, check=True).stdout
    derived = [f32(float(v.rstrip("f,"))) for v in re.search(r"\(f32\): (.*)", out).group(1).split(", ")]
    c3, c2, c1 = _coeffs()
    assert derived == [c1, c2, c3]
