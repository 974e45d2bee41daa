"""Known-answer tests of the oracle's numeric helpers.

The cases are the reference's own zig tests (packages/textsift/src/zig/
math.zig:120-199) plus the documented quirks of its fp16 conversions
(math.zig:45-82) that the CUDA kernels must reproduce.
"""
import math
import struct

import numpy as np


def f32_from_bits(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


def test_bf16_roundtrip_clean(oracle):                        # math.zig:124-132
    for f in (0.0, 1.0, -1.0, 2.5, -3.25, 1024.0):
        assert oracle.bf16_to_f32(oracle.f32_to_bf16(f)) == f


def test_bf16_ties_to_even(oracle):                           # math.zig:134-147
    assert oracle.f32_to_bf16(f32_from_bits(0x3F808000)) == 0x3F80
    assert oracle.f32_to_bf16(f32_from_bits(0x3F818000)) == 0x3F82


def test_bf16_above_halfway(oracle):                          # math.zig:149-153
    assert oracle.f32_to_bf16(f32_from_bits(0x3F808001)) == 0x3F81


def test_bf16_nan_preserved(oracle):                          # math.zig:155-165
    b = oracle.f32_to_bf16(f32_from_bits(0x7F800001))
    assert b != 0x7F80 and (b & 0x7F80) == 0x7F80 and (b & 0x007F) != 0


def test_bf16_infinity(oracle):                               # math.zig:167-172
    assert oracle.f32_to_bf16(f32_from_bits(0x7F800000)) == 0x7F80
    assert oracle.f32_to_bf16(f32_from_bits(0xFF800000)) == 0xFF80


def test_fp16_roundtrip_clean(oracle):                        # math.zig:183-188
    for f in (0.0, 1.0, -1.0, 2.5, -3.25, 1024.0):
        assert oracle.f16_to_f32(oracle.f32_to_f16(f)) == f


def test_fp16x4_matches_scalar(oracle):                       # math.zig:190-197
    s = np.array([0x0000, 0x3C00, 0xBC00, 0x5000], dtype=np.uint16)
    assert list(oracle.f16_to_f32_array(s)) == [oracle.f16_to_f32(int(x)) for x in s] == [0.0, 1.0, -1.0, 32.0]


def test_fp16_decode_quirks(oracle):
    # math.zig:45-52: subnormals are decoded with the normal-number formula
    assert oracle.f16_to_f32(0x0001) == f32_from_bits((1 << 13) + (112 << 23))
    assert oracle.f16_to_f32(0x8000) == 0.0 and math.copysign(1, oracle.f16_to_f32(0x8000)) == -1
    # inf is not special-cased: 0x7C00 decodes to 2^16
    assert oracle.f16_to_f32(0x7C00) == 65536.0


def test_fp16_encode_rounding(oracle):
    # RNE for normals (math.zig:73-81)
    one = 1.0
    ulp = 2.0 ** -10
    assert oracle.f32_to_f16(one + ulp / 2) == 0x3C00            # tie -> even
    assert oracle.f32_to_f16(one + 3 * ulp / 2) == 0x3C02        # tie -> even (up)
    assert oracle.f32_to_f16(65520.0) == 0x7C00                  # overflow
    # subnormal branch rounds half UP (math.zig:67-69), unlike RNE
    half_sub = 2.0 ** -25                                        # exactly half of the smallest subnormal
    assert oracle.f32_to_f16(half_sub) == 0x0001
    assert oracle.f32_to_f16(3 * 2.0 ** -25) == 0x0002           # 1.5 ulp -> 2 (RNE would also give 2)
    assert oracle.f32_to_f16(5 * 2.0 ** -25) == 0x0003           # 2.5 ulp -> 3 (RNE would give 2)
    assert oracle.f32_to_f16(float("nan")) & 0x7E00 == 0x7E00
    assert oracle.f32_to_f16(2.0 ** -26) == 0x0000               # below half the smallest subnormal


def test_exp_approx_accuracy(oracle):
    # wasm_exports.zig:812-838.  Its comment claims ~3e-7 relative error, but
    # the coefficients it ships (822-827) give 2.76e-4 at worst on 2^f, f in
    # [0,1): the oracle must reproduce that polynomial, not exp.
    xs = np.linspace(-40, 0, 2001)
    rel = max(abs(oracle.exp_approx(x) - math.exp(x)) / math.exp(x) for x in xs)
    assert 1e-4 < rel < 3e-4
    f = np.linspace(0, 1, 10001)
    c = [1.000000012, 0.693154774, 0.240226522, 0.055053319, 0.009679494, 0.001333355]
    p = ((((c[5] * f + c[4]) * f + c[3]) * f + c[2]) * f + c[1]) * f + c[0]
    assert abs(np.max(np.abs(p / 2 ** f - 1)) - 2.7626e-4) < 1e-7
    assert oracle.exp_approx(-1000.0) == 0.0 and oracle.exp_approx(float("-inf")) == 0.0
    assert oracle.exp_approx(0.0) == np.float32(1.000000012)


def test_rope_tables_reference_constants(oracle):
    # rope.ts:117-135 with the PF_CONFIG YaRN parameters (wasm.ts:474-482):
    # position 0 is (cos, sin) = (mscale, 0) with mscale = 0.1 ln 32 + 1.
    c, s = oracle.rope_tables(4)
    msc = 0.1 * math.log(32.0) + 1.0
    assert np.all(c[0] == oracle.f32_to_f16(msc))
    assert np.all(s[0] == 0)
    # the first pair rotates at inv_freq[0] = 1 (extrapolation side of the ramp)
    assert c[1, 0] == oracle.f32_to_f16(math.cos(1.0) * msc)
    assert s[1, 0] == oracle.f32_to_f16(math.sin(1.0) * msc)


def test_simd_matmul_matches_scalar_restatement(oracle):
    """The SIMD oracle matmul equals the lane-by-lane scalar restatement bit
    for bit, on both the 8-row tile path and the tail path."""
    r = np.random.Generator(np.random.PCG64(5))
    for T in (1, 7, 8, 19, 64):
        N, K = 37, 96
        int4 = r.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
        sc = r.uniform(1e-3, 1e-2, size=(N, K // 32)).astype(np.float16).view(np.uint16)
        zp = r.integers(0, 256, size=(N, 2), dtype=np.uint8)
        b = r.normal(0, 0.1, size=N).astype(np.float16).view(np.uint16)
        x = r.normal(0, 1, size=(T, K)).astype(np.float32)
        for out_f32 in (True, False):
            a = oracle.matmul_int4(x, int4, sc, zp, b, out_f32)
            s = oracle.matmul_int4(x, int4, sc, zp, b, out_f32, scalar=True)
            assert np.array_equal(a.view(np.uint32 if out_f32 else np.uint16),
                                  s.view(np.uint32 if out_f32 else np.uint16))
