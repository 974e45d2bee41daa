"""The bounded device waits, made to run out without faulting the GPU.

Every spin-wait in this library's kernels (mbarrier waits of the tensor-core
GEMMs and of the attention kernel) ends after a %globaltimer limit, records
the timeout in the handle's device error flag, raises its CTA's abort flag so
the other roles stop too, and frees its TMEM before the CTA exits.  The
self-test entry runs that path with a short limit on a barrier nothing ever
arrives at; the handle must report TS_ERR_DEVICE once, clear the flag, and
then run a normal forward that still matches the reference.
"""
import numpy as np
import pytest

from gpu_util import empty, host, ptr

pytestmark = pytest.mark.gpu

TS_ERR_DEVICE = -5


@pytest.fixture(scope="module")
def model(cuda_lib):
    from textsift_b200 import CudaBackend, make_weights, small_config
    cfg = small_config(n_layers=1, vocab=2048)
    w = make_weights(cfg, seed=5, bias_std=0.02, sink_range=1.0)
    b = CudaBackend(w, cfg, max_tokens=1024, max_seq_len=1024)
    b.warmup()
    yield cfg, w, b
    b.dispose()


def test_wait_timeout_reports_and_handle_recovers(cuda_lib, oracle, model):
    import time

    import torch
    cfg, w, b = model
    L = cuda_lib
    ids = np.random.Generator(np.random.PCG64(21)).integers(0, cfg["vocab"], size=200).astype(np.int32)
    before = b.forward(ids, np.ones(ids.size, np.uint8)).as_2d()

    res = empty((2,), np.int32)
    res.fill_(7)
    t0 = time.perf_counter()
    assert L.ts_cuda_selftest_wait_timeout(b.handle, 2000, ptr(res), None) == 0, L.ts_cuda_last_error()
    rc = L.ts_cuda_check(b.handle, None)
    dt = time.perf_counter() - t0
    assert rc == TS_ERR_DEVICE and b"bounded wait timed out" in L.ts_cuda_last_error()
    # both roles gave up: the timed wait by its own 2 ms limit, the other one
    # by the abort flag well before its 4 s limit
    assert host(res, np.int32).tolist() == [0, 0]
    assert dt < 2.0, f"self-test took {dt:.2f} s"
    # the flag was cleared by the check that reported it
    assert L.ts_cuda_check(b.handle, None) == 0
    torch.cuda.synchronize()

    # the same handle (and the TMEM the self-test held) still serves forwards
    after = b.forward(ids, np.ones(ids.size, np.uint8)).as_2d()
    assert np.array_equal(before, after)
    ref = oracle.OracleModel(cfg, w).forward(ids)
    assert float(np.abs(after - ref).max()) <= 2e-2


def test_wait_selftest_rejects_bad_limits(cuda_lib, model):
    _, _, b = model
    assert cuda_lib.ts_cuda_selftest_wait_timeout(b.handle, 0, None, None) == -1
    assert cuda_lib.ts_cuda_selftest_wait_timeout(b.handle, 1000001, None, None) == -1
    assert cuda_lib.ts_cuda_selftest_wait_timeout(None, 10, None, None) == -1
