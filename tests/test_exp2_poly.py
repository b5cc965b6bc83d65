"""
The polynomial 2^x used for part of the attention softmax (csrc/fa_fwd.cuh,
ex2_poly) emulated step by step in fp32 NumPy: round-to-nearest range
reduction with the 1.5·2^23 constant, degree-3 polynomial for 2^f on
[-1/2, 1/2], exponent insertion. Its relative error must stay below 2e-4 over
the range the kernel feeds it ([-125, 8]), far inside bf16's 2^-8 spacing.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parent.parent / "cd-cuda-course-project_b200" / "csrc" / "fa_fwd.cuh"


def coefficients():
    body = SRC.read_text().split("float ex2_poly(float x)", 1)[1].split("}", 1)[0]
    vals = [float(v) for v in re.findall(r"(-?\d+\.\d+)f", body) if abs(float(v)) < 2.0]
    c3, c2, c1, c0 = vals[0], vals[1], vals[2], vals[3]
    return np.float32(c0), np.float32(c1), np.float32(c2), np.float32(c3)


def ex2_poly(x):
    c0, c1, c2, c3 = coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    y = (x + magic).astype(np.float32)
    n = (y - magic).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = (c3 * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    ni = y.view(np.int32) - np.int32(0x4B400000)
    return (p.view(np.int32) + (ni << 23)).view(np.float32)


def test_ex2_poly_relative_error():
    x = np.linspace(-125.0, 8.0, 4_000_001, dtype=np.float64).astype(np.float32)
    r = ex2_poly(x)
    rel = np.abs(r.astype(np.float64) / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 2e-4
    assert np.all(r > 0) and np.all(np.isfinite(r))


def test_ex2_poly_clamps_large_negative():
    r = ex2_poly(np.array([-1000.0, -200.0, -126.0], np.float32))
    assert np.all(r > 0) and np.all(r < 1e-37)
