"""The span-decoding oracle (oracle/ts_oracle_decode.c) — a restatement of
packages/textsift/src/browser/inference/viterbi.ts and spans.ts.

The reference ships no fixtures for this stage without the real model, so
the Viterbi restatement is pinned here by brute force: for short sequences
every tag path is scored with the same rounding points (f32 stores, double
sums) and the best legal path must equal the decoder's output.  The span
cases are derived from the run rules of spans.ts:29-104.
"""
import itertools

import numpy as np
import pytest

NEG = -1e30


def test_transition_structure(oracle):
    cal = (0.5, -0.25, 1.5, -2.0, 0.75, -1.0)
    trans, start = oracle.viterbi_tables(cal)
    legal = trans > -1e29
    # O->O, O->{B,S} (16), B->{I,E} (16), I->{I,E} (16), {E,S}->O (16), {E,S}->{B,S} (256)
    assert legal.sum() == 1 + 16 + 16 + 16 + 16 + 256
    assert (start > -1e29).sum() == 17
    assert trans[0, 0] == np.float32(0.5)
    assert trans[1, 0] == np.float32(-0.25) and trans[4, 0] == np.float32(-0.25)  # O -> B0, S0
    assert trans[2, 1] == np.float32(1.5) and trans[3, 2] == np.float32(-2.0)     # B0 -> I0, I0 -> E0
    assert trans[0, 3] == np.float32(0.75) and trans[5, 4] == np.float32(-1.0)    # E0 -> O, S0 -> B1
    assert trans[np.ix_([2, 3], [5])].max() < -1e29                                # B1 cannot enter I0/E0


def _brute_force(lg, cal, trans, start):
    T = lg.shape[0]
    best, best_path = None, None
    for path in itertools.product(range(33), repeat=T):
        s = np.float32(np.float64(start[path[0]]) + np.float64(lg[0, path[0]]))
        ok = start[path[0]] > -1e29
        for t in range(1, T):
            tr = trans[path[t], path[t - 1]]
            ok = ok and tr > -1e29
            if not ok:
                break
            s = np.float32(np.float64(s) + np.float64(tr) + np.float64(lg[t, path[t]]))
        if ok and (best is None or s > best):
            best, best_path = s, path
    return np.array(best_path, np.uint8)


@pytest.mark.parametrize("T,seed", [(1, 0), (2, 1), (3, 2), (3, 3)])
def test_viterbi_matches_brute_force(oracle, T, seed):
    r = np.random.Generator(np.random.PCG64(seed))
    cal = tuple(r.uniform(-2, 2, 6))
    lg = r.normal(0, 2, size=(T, 33)).astype(np.float32)
    trans, start = oracle.viterbi_tables(cal)
    assert np.array_equal(oracle.viterbi(lg, cal), _brute_force(lg, cal, trans, start))


def test_viterbi_paths_are_legal(oracle):
    r = np.random.Generator(np.random.PCG64(7))
    for trial in range(20):
        T = int(r.integers(1, 300))
        cal = tuple(r.uniform(-3, 3, 6)) if trial % 2 else oracle.ZERO_CALIBRATION
        lg = r.normal(0, 4, size=(T, 33)).astype(np.float32)
        tags = oracle.viterbi(lg, cal)
        trans, start = oracle.viterbi_tables(cal)
        assert start[tags[0]] > -1e29
        assert all(trans[tags[t], tags[t - 1]] > -1e29 for t in range(1, T))


def test_viterbi_ties_prefer_lower_index(oracle):
    # all emissions equal: every legal path ties; the decoder keeps the first
    # maximum at each step (strict '>'), so the answer is all background
    lg = np.zeros((5, 33), np.float32)
    assert np.array_equal(oracle.viterbi(lg), np.zeros(5, np.uint8))
    assert oracle.viterbi(np.zeros((0, 33), np.float32)).size == 0


def tag(label, boundary):
    return 1 + 4 * label + "BIES".index(boundary)


@pytest.mark.parametrize("tags,spans", [
    ([0, 0, 0], []),
    ([0, tag(0, "B"), tag(0, "I"), tag(0, "E"), 0], [(1, 3, 0)]),
    ([tag(2, "S")], [(0, 0, 2)]),
    ([tag(1, "I"), tag(1, "I"), 0], [(0, 1, 1)]),                      # I without B: implicit B
    ([tag(0, "B"), tag(1, "I")], [(0, 0, 0), (1, 1, 1)]),              # label change closes the run
    ([tag(3, "E")], [(0, 0, 3)]),                                      # E without B: single token
    ([tag(0, "B"), tag(1, "E")], [(0, 0, 0), (1, 1, 1)]),
    ([tag(0, "B"), tag(0, "B"), tag(0, "E")], [(0, 0, 0), (1, 2, 0)]),
    ([tag(5, "B"), tag(5, "I")], [(0, 1, 5)]),                         # open run closed at the end
    ([tag(4, "B"), tag(4, "S"), tag(4, "E")], [(0, 0, 4), (1, 1, 4), (2, 2, 4)]),
    ([tag(7, "B"), 0, tag(7, "E")], [(0, 0, 7), (2, 2, 7)]),
])
def test_bioes_spans(oracle, tags, spans):
    assert oracle.bioes_spans(np.array(tags, np.uint8)) == spans
