"""The prefill softmax's FMA-pipe exponential (prefill::ex2_fma in csrc/attn_prefill.cuh) restated in float32 on the
CPU from the constants in that file, and held to its stated bound against exp2: relative error at most 2.7e-6 over the
range the softmax feeds it (scores minus a running max: at most +8, down to where the result underflows), exactly 0
below -125 and for -inf (masked scores)."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(__file__), "..", "larder_b200", "csrc", "attn_prefill.cuh")


def _body():
    text = open(SRC).read()
    start = text.index("__device__ __forceinline__ float ex2_fma(float x)")
    return text[start:text.index("\n}\n", start)]


def _coefficients():
    """(c4, c3, c2, c1, c0) in the order the Horner chain uses them."""
    body = _body()
    first = re.search(r"fmaf\(([0-9.e+-]+)f, f, ([0-9.e+-]+)f\)", body)
    rest = re.findall(r"fmaf\(p, f, ([0-9.e+-]+)f\)", body)
    assert first and len(rest) == 3, "ex2_fma's polynomial changed shape"
    return [np.float32(first.group(1)), np.float32(first.group(2))] + [np.float32(c) for c in rest]


def _fma(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)


def ex2_fma(x):
    x = np.asarray(x, np.float32)
    c4, c3, c2, c1, c0 = _coefficients()
    xc = np.maximum(x, np.float32(-125.0))
    t = (xc + np.float32(12582912.0)).astype(np.float32)
    f = (xc - (t - np.float32(12582912.0)).astype(np.float32)).astype(np.float32)
    p = _fma(np.full_like(f, c4), f, c3)
    for c in (c2, c1, c0):
        p = _fma(p, f, c)
    bits = (p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    r = bits.astype(np.uint32).view(np.float32)
    return np.where(x < np.float32(-125.0), np.float32(0.0), r)


def test_relative_error_within_the_stated_bound():
    x = np.concatenate([np.linspace(-125, 8, 2_000_001, dtype=np.float32),
                        np.random.default_rng(5).uniform(-30, 8, 1_000_000).astype(np.float32)])
    got = ex2_fma(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1)
    assert rel.max() <= 2.7e-6 * 1.05, rel.max()


def test_integer_points_exact_and_underflow_zero():
    j = np.arange(-125, 9, dtype=np.float32)
    assert np.all(np.abs(ex2_fma(j).astype(np.float64) / np.exp2(j.astype(np.float64)) - 1) <= 1e-6)
    low = np.array([-125.5, -126.0, -200.0, -1e30, -np.inf], np.float32)
    assert np.all(ex2_fma(low) == 0)
