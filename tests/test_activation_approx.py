"""The bf16-output epilogues of the tcgen05 GEMM use erf by Abramowitz & Stegun
formula 7.1.26 (|error| <= 1.5e-7).  This checks the formula with the constants
exactly as written in the CUDA header, evaluated in fp32, against math.erf; the
GPU side is covered by the GEMM tests against a torch fp32 GELU."""
import math
import os
import re

import numpy as np

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "spider_web_moe_b200", "csrc", "sb_common.cuh")


def header_constants():
    text = open(HDR).read()
    body = text[text.index("SB_DEVINL float erf_as7126"):]
    body = body[:body.index("}")]
    p = float(re.search(r"fmaf\(([-0-9.]+)f, ax, 1\.0f\)", body).group(1))
    # Horner order in the header: a5, a4, a3, a2, a1
    horner = [float(v) for v in re.findall(r"([-0-9]+\.[0-9]+)f", body.split("const float poly")[1])]
    a5, a4, a3, a2, a1 = horner[:5]
    return p, (a1, a2, a3, a4, a5)


def erf_as7126_f32(x):
    p, (a1, a2, a3, a4, a5) = header_constants()
    f = np.float32
    x = x.astype(np.float32)
    ax = np.abs(x)
    t = f(1) / (f(p) * ax + f(1))
    poly = ((((f(a5) * t + f(a4)) * t + f(a3)) * t + f(a2)) * t + f(a1)) * t
    return np.copysign(f(1) - poly * np.exp(-ax * ax), x)


def test_published_constants():
    p, a = header_constants()
    assert p == 0.3275911
    assert a == (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def test_error_bound_over_the_line():
    x = np.linspace(-8, 8, 400001)
    want = np.array([math.erf(v) for v in x.astype(np.float32).astype(np.float64)])
    got = erf_as7126_f32(x).astype(np.float64)
    # 1.5e-7 of the method; near 0, 1 - poly*exp(-x^2) cancels in fp32 (a few ulp of 1)
    assert np.max(np.abs(got - want)) <= 6e-7


def test_gelu_error_is_below_bf16_resolution():
    x = np.linspace(-10, 10, 200001).astype(np.float32)
    exact = np.array([0.5 * v * (1 + math.erf(v / math.sqrt(2))) for v in x.astype(np.float64)])
    approx = 0.5 * x.astype(np.float64) * (1 + erf_as7126_f32(x * np.float32(0.70710678118654752)))
    # absolute error <= 0.5 |x| 6e-7: far below one bf16 step (2^-8 relative) of
    # any activation of order one, the scale the down projection sums
    assert np.all(np.abs(approx - exact) <= 0.5 * np.abs(x) * 6e-7 + 1e-12)
