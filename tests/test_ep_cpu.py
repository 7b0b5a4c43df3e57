"""The expert-parallel exchange on CPU ranks (gloo, world size 2 and 4): every rank dispatches its own tokens' pairs
by expert, the ranks exchange counts, the library's host planner (``artlite_moe_ep_plan``) places each rank's rows in
expert-grouped order on the owner, the owners apply their experts, the outputs return into each rank's dispatch
order and every rank combines its own tokens. The result must equal the single-process block on the same tokens.
The data moves by gloo collectives here; on GPUs the block moves the same blocks by NCCL send / recv and keeps the
received rows source-major, each (source rank, local expert) group run in place (artlite_b200/csrc/ep.cu).

Also: a rank that never joins the exchange ends the others' collective with an error after a short process-group
timeout (the host side of the failure detection; no GPU involved)."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, K, D = 16, 2, 8


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _expert(e: int) -> np.ndarray:
    return np.random.default_rng(1000 + e).standard_normal((D, D))


def _tokens(rank: int):
    rng = np.random.default_rng(rank)
    T = 5 + 3 * rank
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K))
    x = rng.standard_normal((T, D))
    return ids, w, x


def _reference(ids, w, x):
    return np.stack([sum(w[t, i] * (_expert(ids[t, i]) @ x[t]) for i in range(K)) for t in range(len(x))])


def _all_gather(obj, world):
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def _rank_main(rank: int, world: int, port: int, q) -> None:
    from artlite_b200.moe.block import ep_plan

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        El = E // world
        ids, w, x = _tokens(rank)
        flat = ids.reshape(-1)
        order = np.argsort(flat, kind="stable")  # the dispatch: pairs by expert, stable in pair order
        slot = np.empty_like(order)
        slot[order] = np.arange(order.size)
        rows = x[order // K]  # this rank's rows in expert order
        counts = np.bincount(flat, minlength=E).astype(np.int32)
        all_counts = _all_gather(counts, world)
        recv_counts = np.stack([all_counts[s][rank * El:(rank + 1) * El] for s in range(world)])
        send_off, recv_pos, local_off, local_counts = ep_plan(counts, recv_counts, world, rank, E)
        assert np.array_equal(send_off, np.concatenate([[0], np.cumsum(counts)[:-1]]))
        # rows to their owners, placed by the plan
        all_rows = _all_gather(rows, world)
        xl = np.zeros((local_off[-1], D))
        for s in range(world):
            s_off = np.concatenate([[0], np.cumsum(all_counts[s])[:-1]])
            for e in range(El):
                n = all_counts[s][rank * El + e]
                g = s_off[rank * El + e]
                xl[recv_pos[s, e]:recv_pos[s, e] + n] = all_rows[s][g:g + n]
        yl = np.zeros_like(xl)
        for e in range(El):
            a, b = local_off[e], local_off[e + 1]
            assert b - a == local_counts[e]
            yl[a:b] = xl[a:b] @ _expert(rank * El + e).T
        # outputs back into each source's dispatch order
        all_yl = _all_gather(yl, world)
        all_pos = _all_gather(recv_pos, world)
        ys = np.zeros_like(rows)
        for owner in range(world):
            for e in range(El):
                g = owner * El + e
                n = counts[g]
                ys[send_off[g]:send_off[g] + n] = all_yl[owner][all_pos[owner][rank, e]:all_pos[owner][rank, e] + n]
        y = np.stack([sum(w[t, i] * ys[slot[t * K + i]] for i in range(K)) for t in range(len(x))])
        q.put((rank, float(np.abs(y - _reference(ids, w, x)).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=10) for _ in range(world))
    assert max(errs.values()) < 1e-12, errs


def _absent_peer_main(rank: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
    if rank == 1:  # leaves between steps, without joining the next exchange
        q.put((1, "left"))
        return
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        q.put((0, "completed"))
    except Exception as e:  # the collective ends with an error once the timeout runs out
        q.put((0, type(e).__name__))


def test_absent_peer_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_absent_peer_main, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res[1] == "left" and res[0] != "completed"
