"""Document workload for the whole-box benchmark: generation, chunking,
packing and document-parallel sharding.

* Chunking restates chunkInput (packages/textsift/src/browser/inference/
  chunking.ts:58-115): a document of n tokens is one chunk if n <= 2048,
  otherwise chunks [s, min(s + 2048, n)) for s = 0, 1920, 3840, ... (overlap
  128), ending with the chunk that reaches n.  Every chunk is its own forward
  with positions starting at 0; "classified tokens" counts each document
  token once.
* Packing puts whole documents' chunks back to back into launches of at most
  max_tokens tokens (the C ABI's seq_offsets).
* Sharding assigns documents to ranks longest-processing-time first by
  chunked token count (no collective on the data path).
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field

import numpy as np

MAX_CHUNK_TOKENS = 2048   # browser/privacy-filter.ts:559
OVERLAP_TOKENS = 128      # browser/inference/chunking.ts:154


def chunk_spans(n: int, max_chunk: int = MAX_CHUNK_TOKENS, overlap: int = OVERLAP_TOKENS):
    """[(start, end)] token spans of the chunks chunkInput makes for n tokens."""
    if n <= max_chunk:
        return [(0, n)]
    step = max_chunk - overlap
    spans = []
    s = 0
    while s < n:
        e = min(s + max_chunk, n)
        spans.append((s, e))
        if e >= n:
            break
        s += step
    return spans


def config4_lengths(n_docs: int, seed: int, lo: int = 256, hi: int = 4096) -> np.ndarray:
    """document lengths uniform in [lo, hi]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(lo, hi + 1, size=n_docs).astype(np.int64)


@dataclass
class Batch:
    ids: np.ndarray            # int32 [T] packed chunk tokens
    offsets: np.ndarray        # uint32 [n_chunks + 1]
    unique_tokens: int         # document tokens classified by this batch (overlap counted once)
    n_docs: int = 0
    doc_ids: list = field(default_factory=list)

    @property
    def tokens(self) -> int:
        return int(self.offsets[-1])


def pack_documents(lengths, doc_ids, vocab: int, max_tokens: int, seed: int) -> list[Batch]:
    """Greedy in-order packing of whole documents (all their chunks) into
    batches of at most max_tokens tokens.  Token ids are uniform in [0, vocab)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    batches: list[Batch] = []
    cur_ids, cur_offs, cur_unique, cur_docs = [], [0], 0, []

    def flush():
        nonlocal cur_ids, cur_offs, cur_unique, cur_docs
        if cur_docs:
            batches.append(Batch(np.concatenate(cur_ids).astype(np.int32), np.asarray(cur_offs, np.uint32),
                                 cur_unique, len(cur_docs), cur_docs))
        cur_ids, cur_offs, cur_unique, cur_docs = [], [0], 0, []

    for n, d in zip(lengths, doc_ids):
        n = int(n)
        spans = chunk_spans(n)
        need = sum(e - s for s, e in spans)
        if need > max_tokens:
            raise ValueError(f"document of {n} tokens needs {need} > max_tokens {max_tokens}")
        if cur_offs[-1] + need > max_tokens:
            flush()
        doc = rng.integers(0, vocab, size=n).astype(np.int32)
        for s, e in spans:
            cur_ids.append(doc[s:e])
            cur_offs.append(cur_offs[-1] + (e - s))
        cur_unique += n
        cur_docs.append(int(d))
    flush()
    return batches


def lpt_assign(lengths, n_ranks: int) -> list[list[int]]:
    """Longest-processing-time assignment of documents to ranks by chunked
    token count; returns the document indices of each rank (ascending)."""
    cost = [sum(e - s for s, e in chunk_spans(int(n))) for n in lengths]
    order = sorted(range(len(cost)), key=lambda i: (-cost[i], i))
    heap = [(0, r) for r in range(n_ranks)]
    out: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + cost[i], r))
    return [sorted(x) for x in out]


def rank_batches(rank: int, world: int, n_docs: int, vocab: int, max_tokens: int, seed: int) -> list[Batch]:
    """The batches rank `rank` processes for a config[4]-style job of n_docs
    documents split across `world` ranks."""
    lengths = config4_lengths(n_docs, seed)
    mine = lpt_assign(lengths, world)[rank]
    return pack_documents(lengths[mine], mine, vocab, max_tokens, seed * 1000003 + rank)
