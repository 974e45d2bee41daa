"""Expert-parallel forward on two GPUs (ts_cuda_ep_init): each GPU holds 64 of
the 128 experts of every layer and the routed rows cross NVLink to the GPU
that holds their expert and back (NCCL grouped send/recv, ep.cu).

The logits of every rank must equal, bit for bit, those of a single-GPU
handle with all experts forwarding the same chunks on the same device: the
router, the permutation and the combine are the single-GPU kernels, each
row's expert MLP does not depend on the other rows of its tile, and the
combine adds a token's experts in ascending id order as before
(expert.ts:137-145).  Steps cover uneven loads: a rank with a single token,
and a rank whose tokens all route to the same four experts.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2


def _chunks(rank, step, vocab):
    r = np.random.default_rng(1000 * step + rank)
    if step == 1 and rank == 1:
        return [np.array([17], np.int32)]  # one token: at most 4 routed rows leave this rank
    if step == 2 and rank == 0:
        return [np.full(700, 5, np.int32), np.full(300, 5, np.int32)]  # every token routes alike
    return [r.integers(0, vocab, size=int(n)).astype(np.int32) for n in r.integers(1, 2049, size=3)]


def _worker(rank, id_q, res_q):
    try:
        import torch
        torch.cuda.set_device(rank)
        from textsift_b200 import CudaBackend, make_weights, small_config
        cfg = small_config(n_layers=2, vocab=4096)
        w = make_weights(cfg, seed=23, bias_std=0.02, sink_range=1.0)
        ep = CudaBackend(w, cfg, device=rank, max_tokens=8192, max_seq_len=2048)
        if rank == 0:
            ident = CudaBackend.ep_unique_id()
            for _ in range(WORLD - 1):
                id_q.put(ident)
        else:
            ident = id_q.get(timeout=120)
        ep.ep_init(rank, WORLD, ident)
        ep.warmup()
        ref = CudaBackend(w, cfg, device=rank, max_tokens=8192, max_seq_len=2048)
        ref.warmup()
        bad = []
        for step in range(4):
            chunks = _chunks(rank, step, cfg["vocab"])
            got = ep.forward_packed(chunks)  # every rank runs the same steps: each layer exchanges
            want = ref.forward_packed(chunks)
            for i, (g, e) in enumerate(zip(got, want)):
                if not np.array_equal(g.data.view(np.uint32), e.data.view(np.uint32)):
                    d = np.abs(g.data - e.data)
                    bad.append((step, i, int((d > 0).sum()), float(d.max())))
        # the exact mode is refused on an expert-parallel handle (before any
        # exchange, so neither rank waits for the other)
        from textsift_b200 import abi
        refused = False
        try:
            ep.set_mode(abi.TS_MODE_EXACT)
            ep.forward_packed(_chunks(rank, 0, cfg["vocab"]))
        except Exception:  # noqa: BLE001
            refused = True
        ep.dispose()
        ref.dispose()
        res_q.put((rank, "ok", bad, refused))
    except Exception as e:  # noqa: BLE001
        import traceback
        res_q.put((rank, "error", traceback.format_exc()[-3000:], str(e)))


def test_expert_parallel_equals_single_gpu():
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    id_q, res_q = ctx.Queue(), ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, id_q, res_q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, status, a, b = res_q.get(timeout=600)
            res[rank] = (status, a, b)
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(WORLD):
        status, a, b = res[rank]
        assert status == "ok", a
        assert a == [], f"rank {rank}: (step, chunk, differing logits, max |diff|) {a}"
        assert b, f"rank {rank}: the exact mode ran on an expert-parallel handle"
