"""The attention kernel's FMA-pipe 2^x (exp2_fma_h2 in
textsift_b200/csrc/k_attn_umma.cu), replayed on the CPU with the
coefficients read out of the source: clamp at -125, round-to-nearest
integer by the 1.5 * 2^23 addition, the fitted cubic on [-1/2, 1/2], 2^n
added to the exponent field, then f32 -> fp16 round to nearest.  Every fp16
result must be within one ulp of 2^x rounded from the exact value, and
-inf and very negative inputs must give 0 (masked keys).  CPU only.
"""
import os
import re

import numpy as np

from conftest import ROOT

SRC = os.path.join(ROOT, "textsift_b200", "csrc", "k_attn_umma.cu")


def _coefficients():
    body = open(SRC).read()
    body = body[body.index("uint32_t exp2_fma_h2("):]
    body = body[:body.index("return f32x2_to_h2")]
    vals = [float(v) for v in re.findall(r"f2pack\(([0-9.eE+-]+)f, \1f\)", body)]
    # magic, -magic, -1, then c3, c2 (first fma), c1, c0
    assert vals[:3] == [12582912.0, -12582912.0, -1.0], vals
    return [np.float32(v) for v in vals[3:7]]


def _exp2_fma(x):
    c3, c2, c1, c0 = _coefficients()
    f32 = np.float32
    xx = np.maximum(x.astype(np.float32), f32(-125.0))
    t = (xx + f32(12582912.0)).astype(np.float32)
    n = (t + f32(-12582912.0)).astype(np.float32)
    f = (xx - n).astype(np.float32)
    # fused multiply-adds: evaluate in f64 and round once to f32
    p = (f.astype(np.float64) * c3 + c2).astype(np.float32)
    p = (p.astype(np.float64) * f + c1).astype(np.float32)
    p = (p.astype(np.float64) * f + c0).astype(np.float32)
    y = (p.view(np.int32) + (t.view(np.int32) << 23)).astype(np.int32).view(np.float32)
    return y.astype(np.float16)


def test_within_one_ulp_of_exact():
    x = np.linspace(-30.0, 0.25, 1_000_001).astype(np.float32)
    got = _exp2_fma(x)
    ref = np.exp2(x.astype(np.float64)).astype(np.float16)
    ulp = np.abs(got.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    assert ulp.max() <= 1
    assert (ulp > 0).mean() < 0.05


def test_masked_and_tiny_inputs_give_zero():
    x = np.array([-np.inf, -1e30, -200.0, -125.0, -30.0], np.float32)
    assert np.all(_exp2_fma(x) == 0)
