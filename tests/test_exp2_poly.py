"""The attention kernel's FMA-pipe exp2 (ex2_poly2 in opendecider_b200/csrc/prefix_attn.cu): its coefficients are the
Remez fit of opendecider_b200/csrc/fit_exp2.py, and its range reduction + polynomial + exponent insertion, emulated
here in float32, stays within 5e-6 relative error of 2^x over the softmax's input range (x <= 8, clamped at -125)."""
import os
import re
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "opendecider_b200", "csrc"))

import fit_exp2  # noqa: E402

F32 = np.float32


def kernel_constants():
    src = open(os.path.join(ROOT, "opendecider_b200", "csrc", "prefix_attn.cu")).read()
    body = src[src.index("ex2_poly2"):]
    return [F32(float(re.search(rf"kC{k} = ([0-9.e-]+)f", body).group(1))) for k in range(5)]


def ex2_poly_emulated(x):
    c = kernel_constants()
    x = np.maximum(x.astype(F32), F32(-125.0))
    t = (x + F32(12582912.0)).astype(F32)
    r = (t - F32(12582912.0)).astype(F32)
    f = (x - r).astype(F32)
    p = np.full_like(f, c[4])
    for ck in (c[3], c[2], c[1], c[0]):
        p = (p.astype(np.float64) * f + ck).astype(F32)        # one rounding per FMA
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(F32)


def test_constants_are_the_fit():
    c, _ = fit_exp2.remez()
    assert [F32(v) for v in c] == kernel_constants()


def test_relative_error_bound():
    x = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001), np.linspace(-1.0, 1.0, 200_001)]).astype(F32)
    got = ex2_poly_emulated(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.all(np.isfinite(got)) and np.all(got > 0)
    assert float(np.max(np.abs(got - want) / want)) < 5e-6


def test_masked_keys_weigh_nothing():
    """-inf (a masked key) becomes 2^-125: a normal number far below one bf16 ulp of any visible weight."""
    y = ex2_poly_emulated(np.array([-np.inf, -1000.0], dtype=F32)).astype(np.float64)
    assert np.all(np.abs(y / 2.0 ** -125 - 1.0) < 5e-6)
    assert np.all(y >= np.finfo(F32).tiny)
