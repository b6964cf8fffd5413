"""The attention kernel's own 2^x for the exponentials it moves off the SFU
(poly_ex2x2 in attention.cu), restated in numpy with the kernel's float32 steps and
coefficients (read from the source): relative error within the bound the kernel's comment
states, over the whole input range the softmax gives it."""

from __future__ import annotations

import re

import numpy as np

from helpers import ROOT

SRC = (ROOT / "crumpet_b200" / "csrc" / "attention.cu").read_text()


def _coefficients():
    body = SRC[SRC.index("float2 poly_ex2x2(float2 x)"):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"make_float2\(([0-9.]+)f, \1f\)", body)]
    # Horner order in the source: c3 (times f) + c2, then c1, then c0
    c3, c2, c1, c0 = vals[:4]
    return np.float32(c0), np.float32(c1), np.float32(c2), np.float32(c3)


def _fma32(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)


def poly_ex2(x):
    c0, c1, c2, c3 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-125))
    r = np.float32(12582912.0)
    t = (x + r).astype(np.float32)
    n = (t - r).astype(np.float32)
    f = _fma32(n, np.float32(-1), x)
    p = _fma32(np.full_like(f, c3), f, np.full_like(f, c2))
    p = _fma32(p, f, np.full_like(f, c1))
    p = _fma32(p, f, np.full_like(f, c0))
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_within_the_stated_bound():
    x = np.linspace(-124.0, 15.0, 2_000_001, dtype=np.float64).astype(np.float32)
    got = poly_ex2(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / want - 1)) < 7.5e-5


def test_far_below_the_range_gives_a_tiny_normal():
    got = poly_ex2(np.array([-125.0, -1000.0, -30000.0], dtype=np.float32))
    assert np.all(got > 0) and np.all(got < 2.0 ** -124)
