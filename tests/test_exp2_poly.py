"""The FMA-pipe exponential of the prefill softmax (prefill_attn.cu, exp2_poly2), on the CPU.

A share of the softmax's 2^x evaluations runs on the FMA pipe instead of MUFU: Cody-Waite
range reduction (n = round(x), f = x - n) and a degree-3 polynomial for 2^f, scaled by 2^n
through the exponent field.  This restates those steps in float32 numpy with the
coefficients read from the kernel source, and checks the relative error against exp2
over the input range the softmax produces (x in [-125, 8]; the running maximum moves
before a score exceeds it by 8): at most 1e-4, below the 2^-11 rounding of the fp16
probabilities it feeds.  Inputs below -126 must give values that round to 0 in fp16.
"""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "smol-genius_b200", "csrc",
                   "prefill_attn.cu")


def _coefficients():
    body = open(SRC).read().split("void exp2_poly2(", 1)[1].split("\n}\n", 1)[0]
    c = [float(x) for x in re.findall(r"fma2\(p0, p1, (?:p0, p1|[-0-9.ef]+, [-0-9.ef]+), f0, f1, ([-0-9.e]+)f", body)]
    lead = float(re.search(r"fma2\(p0, p1, ([-0-9.e]+)f, ", body).group(1))
    assert len(c) == 3, body
    return lead, c


def exp2_poly(x):
    lead, (c2, c1, c0) = _coefficients()
    f32 = np.float32
    x = np.maximum(x.astype(f32), f32(-126.0))
    magic = f32(12582912.0)
    j = (x + magic).astype(f32)
    r = (j - magic).astype(f32)
    f = (x - r).astype(f32)
    f64 = f.astype(np.float64)   # fused multiply-adds: one rounding each, as fma.rn.f32x2
    p = (lead * f64 + c2).astype(f32)
    p = (p.astype(np.float64) * f64 + c1).astype(f32)
    p = (p.astype(np.float64) * f64 + c0).astype(f32)
    n = (j.view(np.uint32) << np.uint32(23)).astype(np.uint32)
    return (p.view(np.uint32) + n).view(np.float32)


def test_relative_error_over_the_softmax_range():
    # results for x near -126 fall below 2^-126 (float32 subnormals): far below fp16's
    # smallest value, so only normal results are checked
    x = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
                        np.float32(-8.0) + np.arange(-4096, 4096, dtype=np.float32) * np.float32(2.0 ** -12)])
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 1e-4, float(rel.max())


def test_underflow_rounds_to_zero_in_fp16():
    got = exp2_poly(np.array([-126.0, -127.5, -300.0, -np.inf], np.float32))
    assert np.all(got.astype(np.float16) == 0)
