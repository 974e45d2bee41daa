"""The allocation-free banded attention (ts_cuda_op_banded_attention_noalloc)
against the allocating entry point (ts_cuda_op_banded_attention), through the
C ABI.  Both run the same kernels on the same inputs, so the outputs must be
bit-identical; two calls in a row with different shapes check that nothing
left in the shared scratch array by one call leaks into the next.  The
sequence offsets reach the GPU as a kernel parameter and the tile list is
built there, so these comparisons also check that device-side tile list
against the host-built one of the allocating entry point.  This file is
collected last so it also runs after every other GPU test."""
import ctypes

import numpy as np
import pytest

from gpu_util import dev, empty, host, ptr, stream

pytestmark = pytest.mark.gpu

F16 = np.uint16
HQ, HKV, HD, WIN = 14, 2, 64, 128
TS_ERR_UNSUPPORTED = -4


@pytest.fixture(scope="module")
def L(cuda_lib):
    import torch
    assert torch.cuda.is_available()
    return cuda_lib


def _inputs(seed, lens):
    r = np.random.Generator(np.random.PCG64(seed))
    T = int(sum(lens))
    q = r.normal(0, 1, size=(T, HQ * HD)).astype(np.float16).view(F16)
    k = r.normal(0, 1, size=(T, HKV * HD)).astype(np.float16).view(F16)
    v = r.normal(0, 1, size=(T, HKV * HD)).astype(np.float16).view(F16)
    sinks = r.uniform(-2, 2, size=HQ).astype(np.float32)
    mask = (r.random(T) > 0.05).astype(np.uint8)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    return T, [dev(q), dev(k), dev(v), dev(sinks), dev(mask)], offs


def _call(fn, T, bufs, offs, out, mode):
    q, k, v, sinks, mask = bufs
    return fn(ptr(q), ptr(k), ptr(v), ptr(sinks), ptr(mask), ptr(out), T, HQ, HKV, HD, WIN,
              offs.ctypes.data, len(offs) - 1, mode, stream())


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_allocating_op_twice(L, mode):
    # a long packed batch, then a shorter one with more, smaller sequences:
    # the second call reuses scratch entries the first one wrote
    cases = [_inputs(11 + mode, [700, 5, 1024, 300, 1]), _inputs(12 + mode, [17, 1, 64, 129, 33, 2, 90])]
    outs = [empty((T, HQ * HD), np.uint16) for T, _, _ in cases]
    for (T, bufs, offs), out in zip(cases, outs):  # back to back on one stream, no sync between
        assert _call(L.ts_cuda_op_banded_attention_noalloc, T, bufs, offs, out, mode) == 0, L.ts_cuda_last_error()
    for (T, bufs, offs), out in zip(cases, outs):
        ref = empty((T, HQ * HD), np.uint16)
        assert _call(L.ts_cuda_op_banded_attention, T, bufs, offs, ref, mode) == 0, L.ts_cuda_last_error()
        assert np.array_equal(host(out, F16), host(ref, F16))


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_max_size(L, mode):
    # 16384 tokens in 1024 sequences whose lengths are not multiples of the
    # 16-query tile: 1023 x 15 tokens + one of 1039, so the tensor-core tile
    # list built on the GPU has 1023 + 65 = 1088 entries, near T/16 + n_seqs
    lens = [15] * 1023 + [16384 - 15 * 1023]
    T, bufs, offs = _inputs(13 + mode, lens)
    assert T == 16384 and len(offs) == 1025
    out = empty((T, HQ * HD), np.uint16)
    ref = empty((T, HQ * HD), np.uint16)
    assert _call(L.ts_cuda_op_banded_attention_noalloc, T, bufs, offs, out, mode) == 0, L.ts_cuda_last_error()
    assert _call(L.ts_cuda_op_banded_attention, T, bufs, offs, ref, mode) == 0, L.ts_cuda_last_error()
    assert np.array_equal(host(out, F16), host(ref, F16))


def test_noalloc_rejects_oversize(L):
    T, bufs, offs = _inputs(14, [64])
    out = empty((T, HQ * HD), np.uint16)
    q, k, v, sinks, mask = bufs
    too_long = np.array([0, 16385], np.uint32)
    rc = L.ts_cuda_op_banded_attention_noalloc(ptr(q), ptr(k), ptr(v), ptr(sinks), ptr(mask), ptr(out), 16385, HQ,
                                               HKV, HD, WIN, too_long.ctypes.data, 1, 0, stream())
    assert rc == TS_ERR_UNSUPPORTED and b"16384" in L.ts_cuda_last_error()
    many = np.arange(1026, dtype=np.uint32)  # 1025 one-token sequences
    rc = L.ts_cuda_op_banded_attention_noalloc(ptr(q), ptr(k), ptr(v), ptr(sinks), ptr(mask), ptr(out), 1025, HQ,
                                               HKV, HD, WIN, many.ctypes.data, 1025, 0, stream())
    assert rc == TS_ERR_UNSUPPORTED and b"1024" in L.ts_cuda_last_error()
