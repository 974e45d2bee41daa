"""Host side of the expert-parallel forward (ts_cuda_ep_plan, ep.cu) on CPU:

  * the plan of every rank against the route-count matrix: rows sent to and
    received from each peer, and grouped-GEMM tiles that cover every received
    row once, inside one (source, expert) segment each;
  * the whole exchange emulated with numpy for 2 and 8 ranks: routed rows out,
    a per-expert function applied on the receiving rank, results back to the
    positions the rows had in the source's expert-major permutation;
  * the same exchange between two gloo ranks (all_to_all_single with the
    plan's split sizes), and a rank that fails before the exchange: the
    survivor's collective ends with an error inside the group's short
    timeout instead of waiting for ever.

The reference runs one process on one device (native/backend.ts:361-759), so
there is no reference counterpart; the parity of the GPU path with the
single-GPU forward is checked on two GPUs by test_gpu_ep.py.
"""
import ctypes
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from textsift_b200 import abi

E = 128
TILE = 128


def plan(counts, recv_counts, world, e_local, tile_rows=TILE):
    """ts_cuda_ep_plan through the C-ABI: send_n, recv_n [world] and tiles [n][4]."""
    L = abi.lib()
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    recv_counts = np.ascontiguousarray(recv_counts, dtype=np.int32)
    send_n = np.zeros(world, np.uint64)
    recv_n = np.zeros(world, np.uint64)
    n = ctypes.c_uint32(0)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    abi.check(L.ts_cuda_ep_plan(p(counts), p(recv_counts), world, e_local, tile_rows, None, None, None, 0,
                                ctypes.byref(n)))
    tiles = np.zeros((max(n.value, 1), 4), np.int32)
    abi.check(L.ts_cuda_ep_plan(p(counts), p(recv_counts), world, e_local, tile_rows, p(send_n), p(recv_n),
                                p(tiles), n.value, ctypes.byref(n)))
    return send_n.astype(np.int64), recv_n.astype(np.int64), tiles[:n.value]


def route_counts(world, tokens, seed, skew=0.0):
    """[world][E] routes per (source rank, global expert): top-4 of each
    token, optionally skewed toward low expert ids, with empty experts."""
    rng = np.random.default_rng(seed)
    C = np.zeros((world, E), np.int32)
    for r in range(world):
        pr = np.exp(-skew * np.arange(E) / E)
        pr[rng.choice(E, 5, replace=False)] = 0.0  # experts no token picks
        pr /= pr.sum()
        for _ in range(tokens):
            C[r, rng.choice(E, 4, replace=False, p=pr)] += 1
    return C


def check_plan(C, r, world):
    el = E // world
    recv_counts = C[:, r * el:(r + 1) * el]  # [source][local expert]
    send_n, recv_n, tiles = plan(C[r], recv_counts, world, el)
    assert np.array_equal(send_n, C[r].reshape(world, el).sum(1))
    assert np.array_equal(recv_n, recv_counts.sum(1))
    total = int(recv_n.sum())
    covered = np.zeros(total, np.int32)
    # segment start of (source p, local expert j) in the received rows
    seg = np.zeros((world, el), np.int64)
    for p in range(world):
        seg[p] = int(recv_n[:p].sum()) + np.concatenate([[0], np.cumsum(recv_counts[p])[:-1]])
    for j, r0, r1, s in tiles:
        assert 0 <= j < el and r0 < r1 and r1 - r0 <= TILE
        p = int(np.searchsorted(np.cumsum(recv_n), r0, side="right"))
        assert s == seg[p, j] and s <= r0 and r1 <= s + recv_counts[p, j]
        assert (r0 - s) % TILE == 0
        covered[r0:r1] += 1
    assert np.all(covered == 1)
    # tiles run expert-major (every tile of local expert j before j + 1)
    assert np.all(np.diff(tiles[:, 0]) >= 0)
    return send_n, recv_n, tiles


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_matches_route_counts(world):
    C = route_counts(world, 300, seed=world, skew=3.0)
    for r in range(world):
        check_plan(C, r, world)


def test_plan_empty_and_full_segments():
    world, el = 2, E // 2
    C = np.zeros((world, E), np.int32)
    C[0, 0] = TILE  # exactly one tile
    C[1, 0] = TILE + 1  # one row over
    C[0, el] = 1
    send_n, recv_n, tiles = check_plan(C, 0, world)
    assert send_n.tolist() == [TILE, 1] and recv_n.tolist() == [TILE, TILE + 1]
    assert tiles.tolist() == [[0, 0, TILE, 0], [0, TILE, 2 * TILE, TILE], [0, 2 * TILE, 2 * TILE + 1, TILE]]
    _, recv_n, tiles = check_plan(np.zeros((world, E), np.int32), 1, world)
    assert recv_n.sum() == 0 and len(tiles) == 0


def test_plan_rejects_bad_arguments():
    L = abi.lib()
    c = np.zeros(E, np.int32)
    n = ctypes.c_uint32(0)
    p = c.ctypes.data_as(ctypes.c_void_p)
    assert L.ts_cuda_ep_plan(p, p, 0, 64, TILE, None, None, None, 0, ctypes.byref(n)) == abi.TS_ERR_ARG
    assert L.ts_cuda_ep_plan(p, p, 2, 64, 0, None, None, None, 0, ctypes.byref(n)) == abi.TS_ERR_ARG
    C = np.zeros((2, E), np.int32)
    C[:, 0] = 300
    rc = np.ascontiguousarray(C[:, :64])
    t = np.zeros((1, 4), np.int32)
    assert L.ts_cuda_ep_plan(C[0].ctypes.data_as(ctypes.c_void_p), rc.ctypes.data_as(ctypes.c_void_p), 2, 64, TILE,
                             None, None, t.ctypes.data_as(ctypes.c_void_p), 1, ctypes.byref(n)) == abi.TS_ERR_ARG
    assert n.value == 6


def expert_fn(rows, e):
    """The stand-in for expert e's MLP: any function of (row, expert)."""
    return rows * 1000 + e


def permuted_rows(C, r):
    """Rank r's expert-major permuted operand: row ids and each row's expert."""
    n = int(C[r].sum())
    ids = r * 10**6 + np.arange(n, dtype=np.int64)
    experts = np.repeat(np.arange(E), C[r])
    return ids, experts


def local_experts(recv, tiles, r, el):
    out = np.full_like(recv, -1)
    for j, r0, r1, _ in tiles:
        out[r0:r1] = expert_fn(recv[r0:r1], r * el + j)
    return out


@pytest.mark.parametrize("world", [2, 8])
def test_exchange_emulated(world):
    el = E // world
    C = route_counts(world, 200, seed=10 + world, skew=2.0)
    plans = [check_plan(C, r, world) for r in range(world)]
    rows = [permuted_rows(C, r) for r in range(world)]
    offs = lambda n: np.concatenate([[0], np.cumsum(n)[:-1]])
    # rows out: rank p receives from r the slice r sends to p
    recv = []
    for p in range(world):
        parts = []
        for r in range(world):
            s_n = plans[r][0]
            o = offs(s_n)
            parts.append(rows[r][0][o[p]:o[p] + s_n[p]])
        recv.append(np.concatenate(parts))
        assert len(recv[p]) == plans[p][1].sum()
    outs = [local_experts(recv[p], plans[p][2], p, el) for p in range(world)]
    # results back to the source's permuted positions
    for r in range(world):
        back = np.full(len(rows[r][0]), -1, np.int64)
        so = offs(plans[r][0])
        for p in range(world):
            ro = offs(plans[p][1])
            back[so[p]:so[p] + plans[r][0][p]] = outs[p][ro[r]:ro[r] + plans[p][1][r]]
        assert np.array_equal(back, expert_fn(rows[r][0], rows[r][1]))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gloo_worker(rank, world, port, fail_rank, q):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        el = E // world
        C = route_counts(world, 150, seed=5, skew=1.0)  # every rank derives the same matrix
        mine = torch.from_numpy(C[rank].copy())
        # 1. route counts per peer expert block, as the device exchange sends them
        got = torch.empty(world * el, dtype=torch.int32)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the count exchange")
        dist.all_to_all_single(got, mine)
        recv_counts = got.numpy().reshape(world, el)
        assert np.array_equal(recv_counts, C[:, rank * el:(rank + 1) * el])
        send_n, recv_n, tiles = plan(C[rank], recv_counts, world, el)
        # 2. rows out, local experts, rows back
        ids, experts = permuted_rows(C, rank)
        recv = torch.empty(int(recv_n.sum()), dtype=torch.int64)
        dist.all_to_all_single(recv, torch.from_numpy(ids), recv_n.tolist(), send_n.tolist())
        out = local_experts(recv.numpy(), tiles, rank, el)
        back = torch.empty(len(ids), dtype=torch.int64)
        dist.all_to_all_single(back, torch.from_numpy(out), send_n.tolist(), recv_n.tolist())
        q.put((rank, "ok", bool(np.array_equal(back.numpy(), expert_fn(ids, experts)))))
    except Exception as e:  # noqa: BLE001 - the test reads what each rank saw
        q.put((rank, "error", f"{type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run_ranks(world, fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gloo_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        rank, status, info = q.get(timeout=120)
        res[rank] = (status, info)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_two_rank_exchange_gloo():
    res = _run_ranks(2, fail_rank=-1)
    assert res == {0: ("ok", True), 1: ("ok", True)}


def test_two_rank_exchange_peer_failure():
    res = _run_ranks(2, fail_rank=1)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    # the survivor's count exchange ends with an error (peer closed or the
    # group's 10 s timeout), not a hang
    assert res[0][0] == "error", res[0]
