"""Error bound of the FMA-pipe 2^x used by the attention softmax
(exp2_poly2 in dllm-serve_b200/csrc/common.cuh), emulated step by step in
fp32 on the CPU with the coefficients read from the header."""
import os
import re

import numpy as np

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "dllm-serve_b200", "csrc", "common.cuh")


def _coef(name):
    m = re.search(rf"{name}\s*=\s*([0-9.eE+-]+)f;", open(HDR).read())
    return np.float32(float(m.group(1)))


def _fma(a, b, c):
    # a*b is exact in float64 for fp32 inputs; one rounding to fp32 afterwards
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x):
    c0, c1, c2, c3 = (_coef(f"kExp2C{i}") for i in range(4))
    magic = _coef("kRoundMagic")
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    f = _fma(n, np.float32(-1.0) * np.ones_like(n), x)
    p = _fma(np.full_like(f, c3), f, np.full_like(f, c2))
    p = _fma(p, f, np.full_like(f, c1))
    p = _fma(p, f, np.full_like(f, c0))
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.view(np.float32)


def test_relative_error_bound():
    x = np.linspace(-124.0, 8.0, 2_000_003, dtype=np.float64).astype(np.float32)
    y = exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() < 1e-4  # bf16 rounding of P is 2^-9 ~ 2e-3


def test_clamped_inputs_stay_tiny_and_positive():
    y = exp2_poly(np.array([-125.0, -200.0, -1e30], np.float32))
    assert np.all(y > 0) and np.all(y < 1e-37)
