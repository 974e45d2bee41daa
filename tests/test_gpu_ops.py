"""Per-op parity of the CUDA kernels against the CPU oracle, called through
the C ABI (the analogue of textsift's kernel-conformance suite,
tests/native/vulkan/conformance-all.js).

Bars: embeddings, dequantised operand tiles and
router top-k indices bit-exact; the exact-order kernels bit-exact; tensor-core
kernels within the tolerances stated per test.
"""
import ctypes

import numpy as np
import pytest

from gpu_util import dev, empty, f16, host, ptr, rand_w4, stream, ulp_diff, w4_handle

pytestmark = pytest.mark.gpu

F16 = np.uint16


@pytest.fixture(scope="module")
def L(cuda_lib):
    import torch
    assert torch.cuda.is_available()
    return cuda_lib


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


# ----------------------------------------------------------------- embedding
@pytest.mark.parametrize("scale_range", [(1e-3, 1e-2), (1e-7, 1e-4), (2e3, 6e4)])
def test_gather_bq_bit_exact(L, oracle, scale_range):
    # small scales give fp16-subnormal products and subnormal scales (the
    # reference's decode and half-up rounding), large ones overflow to inf
    r = rng(1)
    V, D, T = 1000, 640, 777
    w = r.integers(0, 256, size=(V, D // 2), dtype=np.uint8)
    sc = r.uniform(*scale_range, size=(V, D // 32)).astype(np.float16).view(F16)
    zp = r.integers(0, 256, size=(V, D // 64), dtype=np.uint8)
    ids = r.integers(0, V, size=T).astype(np.int32)
    ids[:5] = [-1, V, V + 7, -2 ** 31, 0]  # out of range -> zero rows (wasm_exports.zig:1545-1549)
    out = empty((T, D), np.uint16)
    assert L.ts_cuda_op_gather_bq(ptr(dev(w)), ptr(dev(sc)), ptr(dev(zp)), ptr(dev(ids)), ptr(out), T, V, D,
                                  stream()) == 0
    ref = oracle.embed_lookup_int4(w, sc, zp, ids, V, D)
    assert np.array_equal(host(out, F16), ref)
    assert not host(out, F16)[:4].any()


# ----------------------------------------------------------------- dequant tile
@pytest.mark.parametrize("E,N,K", [(2, 256, 640), (1, 200, 96), (3, 1280, 640), (1, 640, 896)])
def test_dequant_tile_bit_exact(L, oracle, E, N, K):
    r = rng(2)
    int4, sc, zp, bias = rand_w4(r, E, N, K)
    h = w4_handle(L, int4, sc, zp, bias)
    try:
        for e in range(E):
            out = empty((N, K), np.uint16)
            assert L.ts_cuda_op_dequant(h, e, ptr(out), stream()) == 0
            ref = oracle.dequant_int4(int4[e], sc[e], zp[e], N, K)
            assert np.array_equal(host(out, F16), ref), f"expert {e}"
    finally:
        L.ts_cuda_w4_destroy(h)


def test_subnormal_scales_rejected(L):
    r = rng(3)
    int4, sc, zp, bias = rand_w4(r, 1, 128, 64)
    sc[0, 5, 1] = 0x0003  # subnormal fp16: the reference decodes it with its own quirk
    err = ctypes.create_string_buffer(512)
    h = L.ts_cuda_w4_create(0, int4.ctypes.data, sc.ctypes.data, zp.ctypes.data, bias.ctypes.data, 1, 128, 64, err, 512)
    assert not h and b"scale" in err.value


# ----------------------------------------------------------------- MatMulNBits
@pytest.mark.parametrize("M", [1, 7, 8, 13, 128, 301])
@pytest.mark.parametrize("x_f32,out_f32", [(True, True), (True, False), (False, False), (False, True)])
def test_matmul_exact_bit_exact(L, oracle, M, x_f32, out_f32):
    r = rng(4 + M)
    N, K = 160, 640
    int4, sc, zp, bias = rand_w4(r, 1, N, K)
    x = r.normal(0, 1, size=(M, K)).astype(np.float32)
    if not x_f32:
        x = x.astype(np.float16).view(F16)
    h = w4_handle(L, int4, sc, zp, bias)
    try:
        out = empty((M, N), np.float32 if out_f32 else np.uint16)
        assert L.ts_cuda_op_matmul_nbits(h, 0, ptr(dev(x)), 2 if x_f32 else 1, ptr(out), 2 if out_f32 else 1, M, 1,
                                         stream()) == 0
        ref = oracle.matmul_int4(x, int4[0], sc[0], zp[0], bias[0], out_f32)
        got = host(out, np.float32 if out_f32 else F16)
        assert np.array_equal(got.view(np.uint32 if out_f32 else F16), ref.view(np.uint32 if out_f32 else F16))
    finally:
        L.ts_cuda_w4_destroy(h)


@pytest.mark.parametrize("M,N", [(1, 640), (100, 640), (128, 1280), (1000, 640), (4096, 640), (4096, 1280),
                                 (333, 1152)])
def test_matmul_tensor_core(L, oracle, M, N):
    """fp16 activations x fp16((q-zp)*s) on tcgen05, f32 accumulate, vs the
    reference's f32 block-sum order.  Tolerance: |err| <= 2e-3 * max|y| + 1e-3,
    and relative RMS error < 1e-3 (fp16 operand rounding is ~2^-12)."""
    r = rng(10 + M + N)
    K = 640
    int4, sc, zp, bias = rand_w4(r, 1, N, K, zp_random=False)
    x = r.normal(0, 1, size=(M, K)).astype(np.float16).view(F16)
    h = w4_handle(L, int4, sc, zp, bias)
    try:
        out = empty((M, N), np.float32)
        assert L.ts_cuda_op_matmul_nbits(h, 0, ptr(dev(x)), 1, ptr(out), 2, M, 0, stream()) == 0
        got = host(out, np.float32)
        ref = oracle.matmul_int4(x, int4[0], sc[0], zp[0], bias[0], True)
        err = np.abs(got - ref)
        assert err.max() <= 2e-3 * np.abs(ref).max() + 1e-3, err.max()
        assert np.sqrt((err ** 2).mean() / (ref ** 2).mean()) < 1e-3
        # fp16 output path: rounding of the same accumulator
        out16 = empty((M, N), np.uint16)
        assert L.ts_cuda_op_matmul_nbits(h, 0, ptr(dev(x)), 1, ptr(out16), 1, M, 0, stream()) == 0
        g16 = f16(host(out16, F16))
        assert np.abs(g16 - got).max() <= np.abs(got).max() * 2.0 ** -10
    finally:
        L.ts_cuda_w4_destroy(h)


# ----------------------------------------------------------------- RMSNorm
def test_rmsnorm_bit_exact(L, oracle):
    r = rng(5)
    T, D = 300, 640
    a = r.normal(0, 1, size=(T, D)).astype(np.float16).view(F16)
    b = r.normal(0, 1, size=(T, D)).astype(np.float16).view(F16)
    a[0, :7] = [0x0001, 0x8003, 0x7BFF, 0x0000, 0x8000, 0x03FF, 0x0400]  # quirky decodes
    g = r.uniform(0.5, 1.5, size=D).astype(np.float16).view(F16)
    out = empty((T, D), np.float32)
    assert L.ts_cuda_op_rmsnorm(ptr(dev(a)), None, ptr(dev(g)), None, ptr(out), T, D, 1e-5, stream()) == 0
    assert np.array_equal(host(out, np.float32).view(np.uint32), oracle.rms_norm_fp16_to_f32(a, g, 1e-5).view(np.uint32))
    s = empty((T, D), np.uint16)
    assert L.ts_cuda_op_rmsnorm(ptr(dev(a)), ptr(dev(b)), ptr(dev(g)), ptr(s), ptr(out), T, D, 1e-5, stream()) == 0
    rs, rn = oracle.add_rmsnorm_fp16_to_f32(a, b, g, 1e-5)
    assert np.array_equal(host(s, F16), rs)
    assert np.array_equal(host(out, np.float32).view(np.uint32), rn.view(np.uint32))


# ----------------------------------------------------------------- attention
def _attn_inputs(seed, T, Hq=14, Hkv=2, hd=64, mask_tail=0.1):
    r = rng(seed)
    q = r.normal(0, 1, size=(T, Hq * hd)).astype(np.float16).view(F16)
    k = r.normal(0, 1, size=(T, Hkv * hd)).astype(np.float16).view(F16)
    v = r.normal(0, 1, size=(T, Hkv * hd)).astype(np.float16).view(F16)
    sinks = r.uniform(-2, 2, size=Hq).astype(np.float32)
    mask = np.ones(T, np.uint8)
    mask[int(T * (1 - mask_tail)):] = 0
    return q, k, v, sinks, mask


@pytest.mark.parametrize("T,mode", [(300, 1), (300, 0), (9, 0), (9, 1), (1000, 0)])
def test_banded_attention(L, oracle, T, mode):
    q, k, v, sinks, mask = _attn_inputs(6 + T, T)
    out = empty((T, 14 * 64), np.uint16)
    assert L.ts_cuda_op_banded_attention(ptr(dev(q)), ptr(dev(k)), ptr(dev(v)), ptr(dev(sinks)), ptr(dev(mask)),
                                         ptr(out), T, 14, 2, 64, 128, None, 0, mode, stream()) == 0
    got = host(out, F16)
    ref = oracle.banded_attention(q, k, v, sinks, mask, T, 14, 2, 64, 128)
    if mode == 1:
        # reference order on CUDA cores; only the 0-3 exact-exp tail entries
        # may differ by an ulp of expf -> at most 1 fp16 ULP of output
        assert ulp_diff(got, ref).max() <= 1
        assert (got == ref).mean() > 0.99
    else:
        # tensor cores: fp16 probabilities into P.V -> |err| <= 4e-3, mean < 3e-4
        d = np.abs(f16(got) - f16(ref))
        assert d.max() <= 4e-3 and d.mean() < 3e-4, (d.max(), d.mean())


@pytest.mark.parametrize("Hq,Hkv,W", [(12, 2, 128), (4, 2, 16), (7, 7, 64), (14, 2, 0), (14, 2, 200)])
def test_banded_attention_shapes(L, oracle, Hq, Hkv, W):
    """Tensor-core path over GQA groups 1..7 and windows 0..128 (tcgen05
    kernel) and a window past 128 (the mma.sync kernel), packed sequences."""
    lens = [100, 3, 157, 40]
    T = sum(lens)
    q, k, v, sinks, mask = _attn_inputs(8 + Hq + W, T, Hq=Hq, Hkv=Hkv, mask_tail=0.0)
    mask[np.random.Generator(np.random.PCG64(1)).integers(0, T, size=20)] = 0
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    out = empty((T, Hq * 64), np.uint16)
    assert L.ts_cuda_op_banded_attention(ptr(dev(q)), ptr(dev(k)), ptr(dev(v)), ptr(dev(sinks)), ptr(dev(mask)),
                                         ptr(out), T, Hq, Hkv, 64, W, offs.ctypes.data, len(lens), 0,
                                         stream()) == 0, L.ts_cuda_last_error()
    got = host(out, F16)
    for s in range(len(lens)):
        a, b = offs[s], offs[s + 1]
        ref = oracle.banded_attention(q[a:b], k[a:b], v[a:b], sinks, mask[a:b], b - a, Hq, Hkv, 64, W)
        d = np.abs(f16(got[a:b]) - f16(ref))
        assert d.max() <= 4e-3 and d.mean() < 3e-4, (s, d.max(), d.mean())


@pytest.mark.parametrize("mode", [0, 1])
def test_banded_attention_packed(L, oracle, mode):
    lens = [5, 130, 257, 64, 400, 1]
    T = sum(lens)
    q, k, v, sinks, mask = _attn_inputs(7, T, mask_tail=0.0)
    mask[np.random.Generator(np.random.PCG64(0)).integers(0, T, size=40)] = 0
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    out = empty((T, 14 * 64), np.uint16)
    assert L.ts_cuda_op_banded_attention(ptr(dev(q)), ptr(dev(k)), ptr(dev(v)), ptr(dev(sinks)), ptr(dev(mask)),
                                         ptr(out), T, 14, 2, 64, 128, offs.ctypes.data, len(lens), mode,
                                         stream()) == 0
    got = host(out, F16)
    for s in range(len(lens)):
        a, b = offs[s], offs[s + 1]
        ref = oracle.banded_attention(q[a:b], k[a:b], v[a:b], sinks, mask[a:b], b - a, 14, 2, 64, 128)
        if mode == 1:
            assert ulp_diff(got[a:b], ref).max() <= 1
        else:
            assert np.abs(f16(got[a:b]) - f16(ref)).max() <= 4e-3
