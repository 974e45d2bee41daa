"""Fast mode (the benchmarked path) against the free-running reference at the
level the north-star gate names last: argmax labels and emitted spans.

The fast forward's router is exact on its f32 input (test_gpu_model.py), but
the rest of the forward runs on fp16 tensor-core operands, so each block's
hidden state drifts by ~1e-3 relative from the reference's; a router input
that sits at a near-tie of the reference's 4th/5th logits can then land on
the other side, and the flipped expert moves that token's logits by O(0.1).
An argmax flip therefore needs a reference margin (top-1 minus top-2 logit)
of that order.  These tests list every flip with its reference margin and
every span that differs, and assert:
  * with the GPU's routing imposed on the reference (teacher forcing) the
    argmax agrees except where the forced logits' own margin is below twice
    the observed logit difference of that token (floating-point near-ties);
  * free running, every argmax flip has a reference margin below 0.25, and
    flips and span differences stay rare (<= 1% of tokens / spans).
Workloads: BASELINE.json config[0] (1 x 512 tokens, full model) and a
16-document sample of config[4] (lengths U[256, 4096], chunked like
chunkInput), the reference run in its own multi-threaded mode for the
sample (the partition is the reference's MtPool one)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FLIP_MARGIN = 0.25


def _margins(logits):
    s = -np.sort(-logits, axis=1)
    return s[:, 0] - s[:, 1]


def _flip_report(got, ref):
    flips = np.flatnonzero(np.argmax(got, 1) != np.argmax(ref, 1))
    m = _margins(ref)
    d = np.abs(got - ref).max(1)
    return [(int(t), float(m[t]), float(d[t])) for t in flips]


def _span_diff(oracle, got, ref):
    sg = set(oracle.bioes_spans(oracle.viterbi(got)))
    sr = set(oracle.bioes_spans(oracle.viterbi(ref)))
    return sorted(sg ^ sr), max(len(sr), 1)


@pytest.fixture(scope="module")
def full_model(cuda_lib):
    from textsift_b200 import PF_CONFIG, CudaBackend, make_weights
    w = make_weights(PF_CONFIG, seed=0)
    b = CudaBackend(w, PF_CONFIG, max_tokens=65536, max_seq_len=2048)
    b.warmup()
    yield PF_CONFIG, w, b
    b.dispose()


def test_config0_fast_argmax_and_spans(full_model, oracle):
    cfg, w, b = full_model
    ids = np.random.Generator(np.random.PCG64(7)).integers(0, cfg["vocab"], size=512).astype(np.int32)
    lg, topk = b.forward_trace(ids)
    got = lg.as_2d()
    om = oracle.OracleModel(cfg, w)
    forced = om.forward(ids, forced_topk=topk)
    ref = om.forward(ids)
    # teacher-forced: argmax equal unless the forced margin is a float near-tie
    fd = np.abs(got - forced).max(1)
    tf = [(t, m, d) for t, m, d in _flip_report(got, forced) if m >= 2 * fd[t]]
    assert not tf, f"teacher-forced argmax flips beyond near-ties: {tf}"
    flips = _flip_report(got, ref)
    spans, n_spans = _span_diff(oracle, got, ref)
    print(f"\nconfig[0] fast vs reference: {len(flips)} argmax flips of {ids.size} tokens "
          f"(token, reference margin, max |dlogit|): {flips}; {len(spans)} differing spans of {n_spans}: {spans}")
    assert all(m < FLIP_MARGIN for _, m, _ in flips), flips
    assert len(flips) <= 0.01 * ids.size
    assert len(spans) <= max(2, 0.01 * n_spans), spans


def test_config4_sample_fast_argmax_and_spans(full_model, oracle):
    """16 config[4] documents (all their chunks) through one packed fast
    forward, each chunk through the reference in its multi-threaded mode."""
    from textsift_b200.shard import chunk_spans, config4_lengths
    cfg, w, b = full_model
    r = np.random.Generator(np.random.PCG64(41))
    lengths = config4_lengths(16, seed=3)
    chunks = []
    for n in lengths:
        doc = r.integers(0, cfg["vocab"], size=int(n)).astype(np.int32)
        chunks += [doc[s:e] for s, e in chunk_spans(int(n))]
    outs = b.forward_packed(chunks)
    om = oracle.OracleModel(cfg, w)
    flips, spans, n_tok, n_spans = [], [], 0, 0
    for ci, (c, o) in enumerate(zip(chunks, outs)):
        got = o.as_2d()
        ref = om.forward(c, n_threads=6)
        flips += [(ci, t, m, d) for t, m, d in _flip_report(got, ref)]
        sd, ns = _span_diff(oracle, got, ref)
        spans += [(ci,) + s for s in sd]
        n_tok += c.size
        n_spans += ns
    print(f"\nconfig[4] sample ({len(chunks)} chunks, {n_tok} tokens): {len(flips)} argmax flips "
          f"(chunk, token, reference margin, max |dlogit|): {flips}; {len(spans)} differing spans of "
          f"{n_spans}: {spans}")
    assert all(m < FLIP_MARGIN for _, _, m, _ in flips), flips
    assert len(flips) <= 0.01 * n_tok
    assert len(spans) <= max(2, 0.01 * n_spans), spans
