"""BIOES Viterbi decoding on the GPU (k_viterbi.cu) against the oracle's
restatement of textsift's ViterbiDecoder (browser/inference/viterbi.ts), and
the spans it yields (spans.ts).  Bar: tags bit-identical for identical logits;
spans byte-identical wherever the logits are (exact mode)."""
import numpy as np
import pytest

from gpu_util import dev, empty, host, ptr, stream

pytestmark = pytest.mark.gpu

CALS = [(0.0, 0.0, 0.0, 0.0, 0.0, 0.0), (0.8, -1.5, 2.0, -0.5, 1.0, -2.5), (-3.0, 3.0, -1.0, 1.0, -2.0, 2.0)]


@pytest.fixture(scope="module")
def L(cuda_lib):
    import torch
    assert torch.cuda.is_available()
    return cuda_lib


def _decode_gpu(L, logits, lens, cal):
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    T = int(offs[-1])
    d_tags = empty((T,), np.uint8)
    cal32 = np.asarray(cal, np.float32)
    rc = L.ts_cuda_op_viterbi(ptr(dev(np.ascontiguousarray(logits, np.float32).reshape(-1))), offs.ctypes.data,
                              len(lens), cal32.ctypes.data, ptr(d_tags), stream())
    assert rc == 0, L.ts_cuda_last_error()
    return host(d_tags, np.uint8), offs


@pytest.mark.parametrize("ci", range(len(CALS)))
@pytest.mark.parametrize("kind", ["normal", "ties"])
def test_viterbi_matches_reference_decoder(L, oracle, ci, kind):
    r = np.random.Generator(np.random.PCG64(31 + ci))
    lens = [1, 2, 17, 500, 2048, 3000, 64]
    T = sum(lens)
    if kind == "normal":
        lg = r.normal(0, 3, size=(T, 33)).astype(np.float32)
    else:  # small integers: many exact ties between candidate scores
        lg = r.integers(-2, 3, size=(T, 33)).astype(np.float32)
    got, offs = _decode_gpu(L, lg, lens, CALS[ci])
    for s in range(len(lens)):
        a, b = int(offs[s]), int(offs[s + 1])
        ref = oracle.viterbi(lg[a:b], CALS[ci])
        assert np.array_equal(got[a:b], ref), (s, np.flatnonzero(got[a:b] != ref)[:10])


def test_viterbi_rejects_bad_arguments(L):
    lg = dev(np.zeros(33 * 4, np.float32))
    tags = empty((4,), np.uint8)
    good = np.zeros(6, np.float32)
    offs = np.array([0, 4], np.uint32)
    for bad in (np.array([np.nan, 0, 0, 0, 0, 0], np.float32), np.array([0, 0, 1e25, 0, 0, 0], np.float32)):
        assert L.ts_cuda_op_viterbi(ptr(lg), offs.ctypes.data, 1, bad.ctypes.data, ptr(tags), stream()) == -1
    empty_seq = np.array([0, 0, 4], np.uint32)
    assert L.ts_cuda_op_viterbi(ptr(lg), empty_seq.ctypes.data, 2, good.ctypes.data, ptr(tags), stream()) == -1
    long_seq = np.array([0, 8000], np.uint32)
    assert L.ts_cuda_op_viterbi(ptr(lg), long_seq.ctypes.data, 1, good.ctypes.data, ptr(tags), stream()) == -4


@pytest.mark.parametrize("mode", [1, 0])
def test_forward_tags_equal_host_decoding(oracle, cuda_lib, mode):
    """forward_packed_tags = the reference decoder applied to the same
    backend's logits; in exact mode the logits, tags and spans also equal the
    reference forward's."""
    from textsift_b200 import CudaBackend, make_weights, small_config
    cfg = small_config(n_layers=2, vocab=4096)
    w = make_weights(cfg, seed=5, bias_std=0.05, sink_range=1.0)
    b = CudaBackend(w, cfg, max_tokens=4096, max_seq_len=2048)
    b.warmup()
    b.set_mode(mode)
    try:
        r = np.random.Generator(np.random.PCG64(9))
        chunks = [r.integers(0, cfg["vocab"], size=n).astype(np.int32) for n in (300, 1, 77, 1024)]
        cal = CALS[1]
        tags = b.forward_packed_tags(chunks, cal)
        logits = b.forward_packed(chunks)
        om = oracle.OracleModel(cfg, w) if mode == 1 else None
        for c, tg, lo in zip(chunks, tags, logits):
            host_tags = oracle.viterbi(lo.data.reshape(-1, 33), cal)
            assert np.array_equal(tg, host_tags)
            if om is not None:
                ref_logits = om.forward(c, None, n_threads=8)
                ref_tags = oracle.viterbi(ref_logits.reshape(-1, 33), cal)
                assert np.array_equal(tg, ref_tags)
                assert oracle.bioes_spans(tg) == oracle.bioes_spans(ref_tags)
    finally:
        b.dispose()
