"""CPU checks of CudaBackend.forward_packed_stream's host logic: two pinned
slots used alternately, batch i + 1 begun before batch i is collected, every
batch's logits yielded in order, and the slot in flight collected when the
caller stops early or a call fails.  The C ABI is replaced by a fake that
keeps the library's slot rules (ts_cuda_forward_packed_begin on a slot that
holds an uncollected forward and ts_cuda_forward_packed_end on an empty slot
are TS_ERR_STATE) and writes logits that identify each token."""
import ctypes

import numpy as np
import pytest

from textsift_b200 import abi
from textsift_b200 import backend as backend_mod

C = 3  # classes in the fake's logits


class FakeLib:
    def __init__(self, fail_on_begin: int | None = None):
        self.slots = [None, None]  # ids of the forward each slot holds
        self.calls = []
        self.fail_on_begin = fail_on_begin
        self.n_begin = 0

    def ts_cuda_forward_packed_begin(self, h, ids_p, mask_p, offs_p, n_seqs, slot):
        offs = np.ctypeslib.as_array((ctypes.c_uint32 * (n_seqs + 1)).from_address(offs_p.value))
        T = int(offs[-1])
        ids = np.ctypeslib.as_array((ctypes.c_int32 * T).from_address(ids_p.value)).copy()
        self.calls.append(("begin", slot))
        self.n_begin += 1
        if self.fail_on_begin is not None and self.n_begin == self.fail_on_begin:
            return abi.TS_ERR_ARG
        if slot not in (0, 1):
            return abi.TS_ERR_ARG
        if self.slots[slot] is not None:
            return abi.TS_ERR_STATE
        self.slots[slot] = ids
        return abi.TS_OK

    def ts_cuda_forward_packed_end(self, h, slot, out_p):
        self.calls.append(("end", slot))
        ids = self.slots[slot]
        if ids is None:
            return abi.TS_ERR_STATE
        self.slots[slot] = None
        out = np.ctypeslib.as_array((ctypes.c_float * (ids.size * C)).from_address(out_p.value))
        out[:] = (ids[:, None].astype(np.float32) * 10 + np.arange(C, dtype=np.float32)[None, :]).reshape(-1)
        return abi.TS_OK

    def ts_cuda_last_error(self):
        return b"fake failure"


@pytest.fixture
def fake(monkeypatch):
    lib = FakeLib()
    monkeypatch.setattr(abi, "lib", lambda: lib)
    return lib


def ready_backend():
    b = backend_mod.CudaBackend.__new__(backend_mod.CudaBackend)
    b._h = ctypes.c_void_p(1)
    b._ready = True
    b.num_classes = C
    return b


def batches(n, seed=0):
    rng = np.random.default_rng(seed)
    return [[rng.integers(0, 1000, size=int(rng.integers(1, 40)), dtype=np.int32)
             for _ in range(int(rng.integers(1, 5)))] for _ in range(n)]


def expected(chunk):
    return (chunk[:, None].astype(np.float32) * 10 + np.arange(C, dtype=np.float32)[None, :]).reshape(-1)


def test_stream_yields_every_batch_in_order(fake):
    bs = batches(7)
    got = list(ready_backend().forward_packed_stream(bs))
    assert len(got) == len(bs)
    for out, chunks in zip(got, bs):
        assert [lg.sequence_length for lg in out] == [c.size for c in chunks]
        for lg, c in zip(out, chunks):
            assert lg.num_classes == C
            np.testing.assert_array_equal(lg.data, expected(c))
    # begin 0, begin 1, end 0, begin 0, end 1, ..., and the last end
    want = [("begin", 0)]
    for i in range(1, len(bs)):
        want += [("begin", i % 2), ("end", (i - 1) % 2)]
    want.append(("end", (len(bs) - 1) % 2))
    assert fake.calls == want
    assert fake.slots == [None, None]


def test_stream_of_no_batches_calls_nothing(fake):
    assert list(ready_backend().forward_packed_stream([])) == []
    assert fake.calls == []


def test_stream_closed_early_collects_the_slot_in_flight(fake):
    bs = batches(5, seed=1)
    gen = ready_backend().forward_packed_stream(bs)
    first = next(gen)
    np.testing.assert_array_equal(first[0].data, expected(bs[0][0]))
    gen.close()
    assert fake.slots == [None, None]
    assert fake.calls == [("begin", 0), ("begin", 1), ("end", 0), ("end", 1)]


def test_stream_failed_begin_raises_and_frees_the_other_slot(monkeypatch):
    lib = FakeLib(fail_on_begin=3)
    monkeypatch.setattr(abi, "lib", lambda: lib)
    gen = ready_backend().forward_packed_stream(batches(6, seed=2))
    assert len(next(gen)) >= 1  # batch 0, collected after batch 1 was begun
    with pytest.raises(abi.TextsiftCudaError):
        next(gen)
    assert lib.slots == [None, None]


def test_stream_needs_warmup(fake):
    b = ready_backend()
    b._ready = False
    with pytest.raises(RuntimeError):
        next(b.forward_packed_stream(batches(1)))
