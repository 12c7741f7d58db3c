"""Error bound of the prefill softmax's FMA-pipe 2^x (`ex2_poly2` in brimkern_b200/csrc/common.cuh).

The prefill kernel computes a quarter of its probabilities p = 2^(s - m) without the MUFU unit:
x = n + f with n = round(x) (add and subtract 1.5 * 2^23), 2^f from a cubic in f on [-0.5, 0.5],
and n added to the float's exponent field; x is clamped at -127, where the result is 0.  The
probabilities are rounded to fp16 (11-bit significand) before the PV product, so the cubic only
needs a relative error below half an fp16 ulp (2.4e-4).

This test reads the coefficients from the source, replays the device's float32 operation
sequence in numpy, and checks the bound over the range the kernel feeds it (scores at most 8 above
the running maximum, since the maximum is only raised when a tile exceeds it by 2^8), plus the
edge values (masked scores = -inf -> 0, exact powers of two at integers).
"""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _coefficients():
    src = open(os.path.join(ROOT, "brimkern_b200", "csrc", "common.cuh")).read()
    body = src[src.index("float2 ex2_poly2(float2 x)"):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"make_float2\(([0-9.]+)f, \1f\)", body)]
    # Horner order in the source: c3, c2, then c1, then the constant 1.
    assert len(vals) == 4 and vals[3] == 1.0, vals
    c3, c2, c1 = (np.float32(v) for v in vals[:3])
    assert "12582912.f" in body and "-127.f" in body and "<< 23" in body
    return c3, c2, c1


def ex2_poly(x):
    """The device sequence in float32 (each packed f32x2 lane rounds like the scalar op)."""
    c3, c2, c1 = _coefficients()
    f32 = np.float32
    x = np.maximum(np.asarray(x, np.float32), f32(-127.0))
    j = (x + f32(12582912.0)).astype(np.float32)
    n = (j - f32(12582912.0)).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = (c3 * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + f32(1.0)).astype(np.float32)
    bits = (p.view(np.int32).astype(np.int64) + (j.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_bound():
    x = np.linspace(-100.0, 8.0, 2_000_001).astype(np.float32)
    got = ex2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 1.05e-4, rel.max()
    # Below half an fp16 ulp, so p rounds to the same fp16 as 2^x in almost every case.
    assert rel.max() < 2.0 ** -12


def test_reduced_argument_range():
    x = np.linspace(-60.0, 8.0, 400_001).astype(np.float32)
    j = (np.maximum(x, np.float32(-127)) + np.float32(12582912.0)).astype(np.float32)
    f = x - (j - np.float32(12582912.0))
    assert f.min() >= -0.5 and f.max() <= 0.5


def test_edge_values():
    vals = ex2_poly(np.array([-np.inf, -1e30, -127.0, -126.9, 0.0, 1.0, 8.0, -3.0], np.float32))
    assert vals[0] == 0.0 and vals[1] == 0.0 and vals[2] == 0.0
    assert 0.0 <= vals[3] < 2.0 ** -120
    assert vals[4] == 1.0 and vals[5] == 2.0 and vals[6] == 256.0 and vals[7] == 0.125


def test_monotone_over_a_tile_range():
    # Probabilities of larger scores never come out smaller (row sums and maxima stay consistent).
    x = np.linspace(-30.0, 8.0, 1_000_001).astype(np.float32)
    y = ex2_poly(x)
    assert np.all(np.diff(y.astype(np.float64)) >= 0.0)
