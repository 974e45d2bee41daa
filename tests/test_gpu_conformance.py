"""The CUDA kernels on textsift's own kernel-conformance fixtures.

The same 15 fixtures that pin the oracle (tests/native/conformance/fixtures/
of the reference, packed into tests/golden/conformance.npz) are run through
the library's per-op C ABI on the GPU, with the reference harness's own
tolerances (tests/native/vulkan/conformance-all.js:33-44, 120-160: 1 fp16
ULP, rope 32 ULP, f32 1% relative) and the deviations of the fixtures
themselves that tests/test_oracle_golden.py documents.  Fast-mode
(tensor-core) kernels take their documented tolerances instead, named per
test.  Ops with no device entry point of their own (add_fp16, the two casts,
zero_f32, swiglu_clamp, router_topk on given logits) run inside the fused
kernels of the forward and are covered by the model tests.
"""
import numpy as np
import pytest

from gpu_util import dev, empty, f16, host, ptr, stream, w4_handle
from test_oracle_golden import assert_f16, assert_f32

pytestmark = pytest.mark.gpu

F16 = np.uint16


@pytest.fixture(scope="module")
def L(cuda_lib):
    import torch
    assert torch.cuda.is_available()
    return cuda_lib


def _eps(golden, op):
    return np.array([golden.uniform(op)[2]], np.uint32).view(np.float32)[0]


def test_embed_lookup_int4(L, golden):
    op = "embed_lookup_int4"
    T, V, D = (int(x) for x in golden.uniform(op)[:3])
    ids = golden.arr(op, "ids", np.int32)[:T]
    out = empty((T, D), np.uint16)
    assert L.ts_cuda_op_gather_bq(ptr(dev(golden.raw(op, "embed_int4"))), ptr(dev(golden.arr(op, "embed_scales", F16))),
                                  ptr(dev(golden.raw(op, "embed_zp"))), ptr(dev(ids)), ptr(out), T, V, D,
                                  stream()) == 0, L.ts_cuda_last_error()
    assert_f16(host(out, F16), golden.arr(op, "expected", F16))


def test_rms_norm(L, golden):
    # the fixture's shader writes fp16; the library's op is the WASM's
    # rms_norm_fp16_to_f32, whose f32 output is rounded to fp16 here
    op = "rms_norm"
    T, D = (int(x) for x in golden.uniform(op)[:2])
    out = empty((T, D), np.float32)
    assert L.ts_cuda_op_rmsnorm(ptr(dev(golden.arr(op, "x", F16))), None, ptr(dev(golden.arr(op, "gamma", F16))),
                                None, ptr(out), T, D, float(_eps(golden, op)), stream()) == 0
    got = host(out, np.float32).astype(np.float16).view(F16)
    assert_f16(got, golden.arr(op, "expected", F16))


def test_add_rmsnorm(L, golden):
    op = "add_rmsnorm_fp16_to_f32"
    T, D = (int(x) for x in golden.uniform(op)[:2])
    s = empty((T, D), np.uint16)
    out = empty((T, D), np.float32)
    assert L.ts_cuda_op_rmsnorm(ptr(dev(golden.arr(op, "a", F16))), ptr(dev(golden.arr(op, "b", F16))),
                                ptr(dev(golden.arr(op, "gamma", F16))), ptr(s), ptr(out), T, D,
                                float(_eps(golden, op)), stream()) == 0
    assert_f32(host(out, np.float32), golden.arr(op, "expected", np.float32))


def _w4(L, golden, op, N, K):
    w = golden.raw(op, "w_int4").reshape(-1, N, K // 2)
    E = w.shape[0]
    sc = golden.arr(op, "w_scales", F16).reshape(E, N, K // 32)
    zp = golden.raw(op, "w_zp").reshape(E, N, (K // 32 + 1) // 2)
    b = golden.arr(op, "bias", F16).reshape(E, N)
    return w4_handle(L, np.ascontiguousarray(w), np.ascontiguousarray(sc), np.ascontiguousarray(zp),
                     np.ascontiguousarray(b))


@pytest.mark.parametrize("mode", [1, 0])
def test_matmul_int4_fp16_f16(L, golden, mode):
    op = "matmul_int4_fp16_f16"
    T, N, K = (int(x) for x in golden.uniform(op)[:3])
    h = _w4(L, golden, op, N, K)
    try:
        out = empty((T, N), np.uint16)
        assert L.ts_cuda_op_matmul_nbits(h, 0, ptr(dev(golden.arr(op, "x", F16))), 1, ptr(out), 1, T, mode,
                                         stream()) == 0, L.ts_cuda_last_error()
        got, exp = host(out, F16), golden.arr(op, "expected", F16)
        if mode == 1:
            assert_f16(got, exp)
        else:
            # tensor cores (fp16 dequantised operand, f32 accumulation):
            # |err| <= 2e-3 max|y| + 1e-3, as in test_gpu_ops.py
            e = f16(exp).reshape(T, N)
            assert np.abs(f16(got) - e).max() <= 2e-3 * np.abs(e).max() + 1e-3
    finally:
        L.ts_cuda_w4_destroy(h)


def test_matmul_int4_f32_f32(L, golden):
    op = "matmul_int4_f32_f32"
    T, N, K = (int(x) for x in golden.uniform(op)[:3])
    h = _w4(L, golden, op, N, K)
    try:
        out = empty((T, N), np.float32)
        assert L.ts_cuda_op_matmul_nbits(h, 0, ptr(dev(golden.arr(op, "x", np.float32))), 2, ptr(out), 2, T, 1,
                                         stream()) == 0
        # only row 0 of the fixture was computed (one workgroup dispatched)
        assert_f32(host(out, np.float32)[0], golden.arr(op, "expected", np.float32).reshape(T, N)[0])
    finally:
        L.ts_cuda_w4_destroy(h)


def test_rope_apply(L, golden):
    op = "rope_apply"
    T, H, hd = (int(x) for x in golden.uniform(op)[:3])
    out = empty((T, H * hd), np.uint16)
    pos = np.arange(T, dtype=np.int32)
    assert L.ts_cuda_op_rope(ptr(dev(golden.arr(op, "_output_initial", F16))), ptr(out),
                             ptr(dev(golden.arr(op, "cos_tab", F16))), ptr(dev(golden.arr(op, "sin_tab", F16))),
                             ptr(dev(pos)), T, H, hd, stream()) == 0, L.ts_cuda_last_error()
    # the harness's 32 ULP, plus the cancellation-region allowance of
    # test_oracle_golden.py (the fixture's GPU fused the pair products)
    assert_f16(host(out, F16), golden.arr(op, "expected", F16), ulps=32, atol=2.0 ** -10)


def test_banded_attention(L, golden):
    # head_dim 32: the exact-order kernel (the tensor-core kernels need 64)
    op = "banded_attention"
    T, Hq, Hkv, hd, W, use_mask = (int(x) for x in golden.uniform(op)[:6])
    mask = dev(golden.raw(op, "mask")[:T]) if use_mask else None
    out = empty((T, Hq * hd), np.uint16)
    assert L.ts_cuda_op_banded_attention(ptr(dev(golden.arr(op, "q", F16))), ptr(dev(golden.arr(op, "k", F16))),
                                         ptr(dev(golden.arr(op, "v", F16))),
                                         ptr(dev(golden.arr(op, "sinks", np.float32))),
                                         ptr(mask) if mask is not None else None, ptr(out), T, Hq, Hkv, hd, W, None,
                                         0, 1, stream()) == 0, L.ts_cuda_last_error()
    assert_f16(host(out, F16), golden.arr(op, "expected", F16), ulps=1, atol=2.0 ** -13)


def _expert_rows(L, golden, op, x_rows, ridx, N, D, mode):
    """Per routed row r: expert ridx[r] applied to x_rows[r] (f32 in, f32 out
    in exact mode; fp16 in, f32 out on the tensor cores)."""
    h = _w4(L, golden, op, N, D)
    try:
        out = np.empty((len(ridx), N), np.float32)
        for r, e in enumerate(ridx):
            o = empty((1, N), np.float32)
            if mode == 1:
                x = dev(np.ascontiguousarray(x_rows[r:r + 1], np.float32))
                xd = 2
            else:
                x = dev(np.ascontiguousarray(x_rows[r:r + 1]).astype(np.float16).view(F16))
                xd = 1
            assert L.ts_cuda_op_matmul_nbits(h, int(e), ptr(x), xd, ptr(o), 2, 1, mode, stream()) == 0, \
                L.ts_cuda_last_error()
            out[r] = host(o, np.float32)[0]
        return out
    finally:
        L.ts_cuda_w4_destroy(h)


@pytest.mark.parametrize("mode", [1, 0])
def test_qmoe_gate_up(L, golden, mode):
    op = "qmoe_gate_up"
    T, K, N, D = (int(x) for x in golden.uniform(op)[:4])
    x = golden.arr(op, "x", np.float32).reshape(T, D)
    ridx = golden.arr(op, "routing_idx", np.int32)[:T * K]
    got = _expert_rows(L, golden, op, x[np.arange(T * K) // K], ridx, N, D, mode)
    exp = golden.arr(op, "expected", np.float32).reshape(T * K, N)
    if mode == 1:
        assert_f32(got, exp)
    else:
        assert np.abs(got - exp).max() <= 2e-3 * np.abs(exp).max() + 1e-3


def test_qmoe_down_scatter(L, golden):
    op = "qmoe_down_scatter"
    T, K, N, D = (int(x) for x in golden.uniform(op)[:4])
    glu = golden.arr(op, "glu", np.float32).reshape(T * K, D)
    ridx = golden.arr(op, "routing_idx", np.int32)[:T * K]
    rsc = golden.arr(op, "routing_scores", np.float32)[:T * K]
    rows = _expert_rows(L, golden, op, glu, ridx, N, D, 1)
    acc = golden.arr(op, "_output_initial", np.float32).reshape(T, N).copy()
    for tk in range(T * K):  # the shader's scatter-add of the weighted rows
        acc[tk // K] = np.float32(acc[tk // K] + rsc[tk] * rows[tk])
    assert_f32(acc, golden.arr(op, "expected", np.float32).reshape(T, N))
