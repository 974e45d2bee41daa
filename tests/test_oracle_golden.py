"""The oracle against textsift's own kernel-conformance fixtures.

Fixtures: tests/native/conformance/fixtures/<op>/ of teamchong/textsift,
packed into tests/golden/conformance.npz by tests/golden/make_golden.py.
They were produced by browser WebGPU, so -- exactly as the reference's own
harness (tests/native/vulkan/conformance-all.js:33-44, 120-160) -- fp16
outputs must agree within 1 ULP (rope_apply 32 ULP) and f32 outputs within 1%
relative.  They pin layouts and semantics: nibble order, zero-point packing,
block size, bias, masks, the sink column, GQA grouping.
"""
import numpy as np
import pytest

F16 = np.uint16


def f16_ulp_diff(actual_bits, expected_bits):
    a = actual_bits.view(np.float16).astype(np.float64)
    e = expected_bits.view(np.float16).astype(np.float64)
    mag = np.maximum(np.abs(e), 2.0 ** -14)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - 10)
    return np.abs(a - e) / ulp


def assert_f16(actual, expected, ulps=1.0, atol=0.0):
    """Within `ulps` fp16 ULP of the fixture, or within `atol` absolute (for
    outputs near zero after cancellation, where an ULP is tiny)."""
    a = np.asarray(actual, F16).ravel()
    e = np.asarray(expected, F16).ravel()
    d = f16_ulp_diff(a, e)
    ad = np.abs(a.view(np.float16).astype(np.float64) - e.view(np.float16).astype(np.float64))
    bad = (d > ulps + 1e-3) & (ad > atol)
    assert not bad.any(), f"{bad.sum()} outputs beyond {ulps} ULP and {atol} abs (worst {d.max():.1f} ULP)"


def assert_f32(actual, expected, rel=1e-2):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    r = np.abs(a - e) / np.maximum(1e-6, np.abs(e))
    assert r.max() <= rel, f"max rel {r.max():.3g} (limit {rel})"


def test_golden_has_every_op(golden):
    assert sorted(golden.meta) == sorted([
        "add_fp16", "add_rmsnorm_fp16_to_f32", "banded_attention", "cast_f32_to_fp16_scaled",
        "cast_fp16_to_f32", "embed_lookup_int4", "matmul_int4_f32_f32", "matmul_int4_fp16_f16",
        "qmoe_down_scatter", "qmoe_gate_up", "rms_norm", "rope_apply", "router_topk", "swiglu_clamp",
        "zero_f32"])


def test_add_fp16(oracle, golden):
    n = golden.uniform("add_fp16")[0]
    out = oracle.add_fp16(golden.arr("add_fp16", "a", F16)[:n], golden.arr("add_fp16", "b", F16)[:n])
    assert_f16(out, golden.arr("add_fp16", "expected", F16))


def test_cast_fp16_to_f32(oracle, golden):
    out = oracle.convert_fp16_to_f32(golden.arr("cast_fp16_to_f32", "src", F16))
    assert_f32(out, golden.arr("cast_fp16_to_f32", "expected", np.float32), rel=0.0)


def test_cast_f32_to_fp16_scaled(oracle, golden):
    op = "cast_f32_to_fp16_scaled"
    scale = golden.arr(op, "_uniform_scale", np.float32)[0]
    out = oracle.cast_f32_to_fp16_scaled(golden.arr(op, "src", np.float32), scale)
    assert_f16(out, golden.arr(op, "expected", F16))


def test_zero_f32(golden):
    assert not np.any(golden.raw("zero_f32", "expected"))


def test_rms_norm(oracle, golden):
    op = "rms_norm"
    T, D, eps_bits = golden.uniform(op)[:3]
    eps = np.array([eps_bits], np.uint32).view(np.float32)[0]
    out = oracle.rms_norm(golden.arr(op, "x", F16).reshape(T, D), golden.arr(op, "gamma", F16), eps)
    assert_f16(out, golden.arr(op, "expected", F16))


def test_add_rmsnorm(oracle, golden):
    op = "add_rmsnorm_fp16_to_f32"
    T, D, eps_bits = golden.uniform(op)[:3]
    eps = np.array([eps_bits], np.uint32).view(np.float32)[0]
    _, n = oracle.add_rmsnorm_fp16_to_f32(golden.arr(op, "a", F16).reshape(T, D),
                                          golden.arr(op, "b", F16).reshape(T, D), golden.arr(op, "gamma", F16), eps)
    assert_f32(n, golden.arr(op, "expected", np.float32))


def test_swiglu_clamp(oracle, golden):
    op = "swiglu_clamp"
    T, D = golden.uniform(op)[:2]
    out = oracle.swiglu_clamp(golden.arr(op, "gate_up", np.float32).reshape(T, 2 * D))
    assert_f32(out, golden.arr(op, "expected", np.float32))


def test_rope_apply(oracle, golden):
    op = "rope_apply"
    T, H, hd = golden.uniform(op)[:3]
    qk = golden.arr(op, "_output_initial", F16)
    out = oracle.rope_apply(qk, golden.arr(op, "cos_tab", F16), golden.arr(op, "sin_tab", F16), T, H, hd)
    # The fixture's shader (native/shaders/rope_apply.wgsl:40-49) rounds in
    # fp16 like the WASM, but the browser GPU fused the pairs: in the
    # cancellation region a*c - b*s the two differ by up to one ULP of the
    # operands (|x| < 2 here: 2^-10) although that is many ULPs of a
    # near-zero result.  The reference's harness allows 32 ULP for the same
    # effect (tests/native/vulkan/conformance-all.js:33-44).
    assert_f16(out, golden.arr(op, "expected", F16), ulps=32, atol=2.0 ** -10)


def test_embed_lookup_int4(oracle, golden):
    op = "embed_lookup_int4"
    T, V, D = golden.uniform(op)[:3]
    out = oracle.embed_lookup_int4(golden.raw(op, "embed_int4"), golden.arr(op, "embed_scales", F16),
                                   golden.raw(op, "embed_zp"), golden.arr(op, "ids", np.int32), V, D)
    assert_f16(out, golden.arr(op, "expected", F16))


@pytest.mark.parametrize("op,x_f32,out_f32", [("matmul_int4_f32_f32", True, True),
                                              ("matmul_int4_fp16_f16", False, False)])
def test_matmul_int4(oracle, golden, op, x_f32, out_f32):
    T, N, K = golden.uniform(op)[:3]
    x = golden.arr(op, "x", np.float32 if x_f32 else F16).reshape(T, K)
    out = oracle.matmul_int4(x, golden.raw(op, "w_int4").reshape(N, K // 2),
                             golden.arr(op, "w_scales", F16).reshape(N, K // 32),
                             golden.raw(op, "w_zp").reshape(N, -1), golden.arr(op, "bias", F16), out_f32)
    if out_f32:
        # The fixture dispatched one 64-thread workgroup for a one-thread-per-
        # output shader (meta.json "dispatch": [1,1,1]), so only outputs
        # 0..63 (row 0) were computed; the rest of expected.bin is zero.
        exp = golden.arr(op, "expected", np.float32).reshape(T, N)
        assert np.all(exp[1:] == 0)
        assert_f32(out[0], exp[0])
    else:
        assert_f16(out, golden.arr(op, "expected", F16))


def test_banded_attention(oracle, golden):
    op = "banded_attention"
    T, Hq, Hkv, hd, W, use_mask = golden.uniform(op)[:6]
    mask = golden.raw(op, "mask")[:T] if use_mask else None
    out = oracle.banded_attention(golden.arr(op, "q", F16), golden.arr(op, "k", F16), golden.arr(op, "v", F16),
                                  golden.arr(op, "sinks", np.float32), mask, T, Hq, Hkv, hd, W)
    # WGSL sums each score with one fma chain over d (banded_attention.wgsl)
    # and uses exact exp; the WASM uses 4x4 partial sums and the polynomial
    # exp.  Outputs agree to 1 ULP except near zero, where the difference is
    # below one ULP of the largest output (|out| < 0.25 here: 2^-13).
    assert_f16(out, golden.arr(op, "expected", F16), ulps=1, atol=2.0 ** -13)


def test_router_topk(oracle, golden):
    # The WGSL kernel emits its k slots in replacement order; the WASM path
    # sorts descending (wasm_exports.zig:367-426).  Compare per-row sets.
    op = "router_topk"
    T, E, K = golden.uniform(op)[:3]
    logits = golden.arr(op, "logits", np.float32).reshape(T, E)
    idx, val = oracle.topk(logits, K)
    w = oracle.softmax(val) * np.float32(1.0 / K)
    exp = golden.arr(op, "expected", np.float32).reshape(T, K)
    assert_f32(np.sort(w, axis=1), np.sort(exp, axis=1))
    # indices: the k largest logits, descending, ties to the lower index
    ref = np.argsort(-logits, axis=1, kind="stable")[:, :K]
    assert np.array_equal(idx, ref)


def _expert_matmul(oracle, golden, op, x, e, N, D):
    w4 = golden.raw(op, "w_int4").reshape(-1, N, D // 2)
    sc = golden.arr(op, "w_scales", F16).reshape(-1, N, D // 32)
    zp = golden.raw(op, "w_zp").reshape(-1, N, (D // 32 + 1) // 2)
    b = golden.arr(op, "bias", F16).reshape(-1, N)
    return oracle.matmul_int4(x[None, :].astype(np.float32), w4[e], sc[e], zp[e], b[e], True)[0]


def test_qmoe_gate_up(oracle, golden):
    op = "qmoe_gate_up"
    T, K, N, D = golden.uniform(op)[:4]
    x = golden.arr(op, "x", np.float32).reshape(T, D)
    ridx = golden.arr(op, "routing_idx", np.int32)
    out = np.stack([_expert_matmul(oracle, golden, op, x[tk // K], ridx[tk], N, D) for tk in range(T * K)])
    assert_f32(out, golden.arr(op, "expected", np.float32).reshape(T * K, N))


def test_qmoe_down_scatter(oracle, golden):
    op = "qmoe_down_scatter"
    T, K, N, D = golden.uniform(op)[:4]
    glu = golden.arr(op, "glu", np.float32).reshape(T * K, D)
    ridx = golden.arr(op, "routing_idx", np.int32)
    rsc = golden.arr(op, "routing_scores", np.float32)
    acc = golden.arr(op, "_output_initial", np.float32).reshape(T, N).copy()
    for tk in range(T * K):
        acc[tk // K] = np.float32(acc[tk // K] + rsc[tk] * _expert_matmul(oracle, golden, op, glu[tk], ridx[tk], N, D))
    assert_f32(acc, golden.arr(op, "expected", np.float32).reshape(T, N))
