"""The codec snake's sin^2 (csrc/conv.cu `sin2_reduced2`): period-pi Cody-Waite reduction and a degree-5 polynomial in
r^2. The constants are read from the CUDA source itself and the kernel's fp32 fused multiply-add sequence is emulated
with numpy (a product of two fp32 values is exact in float64; one rounding to fp32 after the add), against a float64
sin^2, over |t| < 2^21 (SIN2_RANGE: beyond it the epilogue falls back to sinf). CPU only."""
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "..", "audio8-turbo-engine_b200", "csrc", "conv.cu")
f32 = np.float32


def _constants():
    src = open(SRC).read()
    body = src[src.index("float2 sin2_reduced2(float2 t) {"):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"f2\(([-+0-9.eE]+)f\)", body)]
    rng = float(re.search(r"constexpr float SIN2_RANGE = ([0-9.]+)f;", src).group(1))
    return vals, rng


def _fma(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(f32)


def _sin2(t, c):
    inv_pi, magic, _magic2, neg_pi_hi, neg_pi_lo = (f32(v) for v in c[:5])
    poly = [f32(v) for v in c[5:]]
    one = np.ones_like(t)
    big = _fma(t, one * inv_pi, one * magic)
    k = (big - magic).astype(f32)
    r = _fma(k, one * neg_pi_hi, t)
    r = _fma(k, one * neg_pi_lo, r)
    u = (r * r).astype(f32)
    p = _fma(one * poly[0], u, one * poly[1])
    for q in poly[2:]:
        p = _fma(p, u, one * q)
    return (u * p).astype(f32)


def test_sin2_constants_parsed():
    c, rng = _constants()
    assert len(c) == 11 and rng == 2.0 ** 21
    assert abs(c[0] - 1 / np.pi) < 1e-7 and abs(-(c[3] + c[4]) - np.pi) < 1e-12


def test_sin2_error_bound():
    c, rng = _constants()
    gen = np.random.default_rng(7)
    worst = 0.0
    e = -6
    while 2.0 ** e <= rng:
        t = (gen.uniform(-1, 1, 200_000) * 2.0 ** e).astype(f32)
        t = t[np.abs(t) < rng]
        err = np.abs(_sin2(t, c).astype(np.float64) - np.sin(t.astype(np.float64)) ** 2)
        worst = max(worst, float(err.max()))
        e += 1
    assert worst < 2.5e-7, worst


def test_sin2_small_arguments_relative():
    # near 0 sin^2(t) ~ t^2: the polynomial keeps the relative error small, not only the absolute one
    c, _ = _constants()
    t = np.geomspace(1e-6, 1e-1, 20001).astype(f32)
    got = _sin2(t, c).astype(np.float64)
    ref = np.sin(t.astype(np.float64)) ** 2
    assert np.max(np.abs(got - ref) / ref) < 2e-6
