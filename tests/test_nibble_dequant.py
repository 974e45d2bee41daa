"""The int4 weight decode of the exact matmul (k_simt.cu
matmul_w4_exact_kernel) and the router candidate pass (k_router.cu):
nib_raw (ts_common.cuh) puts a nibble q in the mantissa of 2^23 (bits
0x4B000000 | q) and one packed add of -(2^23 + zp) gives q - zp.  The
embedding gather (k_simt.cu embed_block_ref) uses the same byte permute and
subtracts 2^23 + zp, the same value.  Replayed in numpy for every nibble
and zero point: the result must be the f32 value of the integer q - zp, bit
for bit (+0.0 where equal, as the integer conversion gives), which is what
the reference's (q - zp) * scale starts from.  The byte-permute selector is
checked against the byte it must pick.  CPU only.
"""
import os
import re

import numpy as np

from conftest import ROOT

COMMON = os.path.join(ROOT, "textsift_b200", "csrc", "ts_common.cuh")


def _byte_perm(x: int, y: int, s: int) -> int:
    """__byte_perm(x, y, s): result byte i = byte (s >> 4i) & 7 of the
    eight bytes y:x (x bytes 0-3, y bytes 4-7)."""
    src = x | (y << 32)
    out = 0
    for i in range(4):
        sel = (s >> (4 * i)) & 7
        out |= ((src >> (8 * sel)) & 0xFF) << (8 * i)
    return out


def _nib_raw_selector():
    body = open(COMMON).read()
    body = body[body.index("float nib_raw("):]
    body = body[:body.index("}")]
    m = re.search(r"__byte_perm\(lohi, (0x[0-9A-Fa-f]+)u, (0x[0-9A-Fa-f]+)u \| j\)", body)
    assert m, "nib_raw's byte permute not found"
    return int(m.group(1), 16), int(m.group(2), 16)


def test_nib_raw_places_each_nibble_in_the_mantissa_of_two_to_23():
    hi_word, sel = _nib_raw_selector()
    rng = np.random.default_rng(7)
    for w in rng.integers(0, 2**32, size=2000, dtype=np.uint64):
        w = int(w)
        lo, hi = w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F
        for j in range(4):
            for lohi, shift in ((lo, 0), (hi, 4)):
                bits = _byte_perm(lohi, hi_word, sel | j)
                q = (w >> (8 * j + shift)) & 15
                assert bits == 0x4B000000 | q
                assert np.uint32(bits).view(np.float32) == np.float32(2.0**23 + q)


def test_two_to_23_offset_gives_q_minus_zp_exactly():
    q = np.arange(16, dtype=np.uint32)
    raw = (np.uint32(0x4B000000) | q).view(np.float32)
    for zp in range(16):
        nz = -(np.float32(8388608.0) + np.float32(zp))  # the kernels' -(2^23 + zp)
        got = raw + nz  # f32 round-to-nearest add, as add.rn.f32x2 per half
        want = (q.astype(np.int64) - zp).astype(np.float32)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
