"""Host-side logic of the whole-box benchmark: chunking (chunkInput,
packages/textsift/src/browser/inference/chunking.ts:58-115), packing, and the
document-parallel split, including a 2-rank gloo run on CPU."""
import os

import numpy as np
import pytest

from textsift_b200.shard import (chunk_spans, config4_lengths, lpt_assign, pack_documents,
                                 rank_batches)


def test_chunk_spans_match_chunk_input():
    assert chunk_spans(1) == [(0, 1)]
    assert chunk_spans(2048) == [(0, 2048)]
    assert chunk_spans(2049) == [(0, 2048), (1920, 2049)]
    assert chunk_spans(3000) == [(0, 2048), (1920, 3000)]
    assert chunk_spans(4096) == [(0, 2048), (1920, 3968), (3840, 4096)]
    for n in range(2049, 9000, 97):
        sp = chunk_spans(n)
        assert sp[0][0] == 0 and sp[-1][1] == n
        assert all(e - s <= 2048 for s, e in sp)
        assert all(b[0] == a[0] + 1920 for a, b in zip(sp, sp[1:]))


def test_pack_documents_limits_and_counts():
    lengths = config4_lengths(200, seed=3)
    batches = pack_documents(lengths, list(range(200)), vocab=1000, max_tokens=16384, seed=1)
    assert sum(b.n_docs for b in batches) == 200
    assert sum(b.unique_tokens for b in batches) == int(lengths.sum())
    for b in batches:
        assert b.tokens <= 16384 and b.offsets[0] == 0
        assert np.all(np.diff(b.offsets.astype(np.int64)) > 0)
        assert np.all(np.diff(b.offsets.astype(np.int64)) <= 2048)
        assert b.ids.min() >= 0 and b.ids.max() < 1000


def test_lpt_balance():
    lengths = config4_lengths(8192, seed=0)
    for world in (2, 4, 8):
        parts = lpt_assign(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(8192))
        cost = [sum(e - s for n in lengths[p] for s, e in chunk_spans(int(n))) for p in parts]
        assert max(cost) - min(cost) <= 4096


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bs = rank_batches(rank, world, 256, vocab=5000, max_tokens=32768, seed=7)
        mine = sorted(d for b in bs for d in b.doc_ids)
        toks = sum(b.unique_tokens for b in bs)
        out = [None] * world
        dist.all_gather_object(out, (mine, toks))
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_two_rank_document_split_gloo():
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    docs0, docs1 = res[0][0], res[1][0]
    assert not set(docs0) & set(docs1)
    assert sorted(docs0 + docs1) == list(range(256))
    lengths = config4_lengths(256, seed=7)
    assert res[0][1] + res[1][1] == int(lengths.sum())
