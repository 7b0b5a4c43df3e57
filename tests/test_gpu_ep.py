"""Expert parallelism on 2 and 4 GPUs (one process per GPU): each rank owns 1/N of the experts and its own tokens;
the EP forward (token rows out by the peer-store kernels over NVLink, or by NCCL send / recv with expert chunks or
ARTLITE_EP_EXCHANGE=nccl; local tcgen05 or GEMV experts, outputs back the same way, local combine) must
equal, on every rank, the single-GPU block over the same tokens with all experts, with one or four expert chunks and
with the rows regrouped expert-major before the experts (the default from 8 ranks, forced here), and with a shared
expert (held whole by every rank, run on its own tokens). Skipped with fewer GPUs than ranks.
NVLS is off (NCCL_NVLS_ENABLE=0); the ranks are child processes."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, E, K, F = 512, 16, 4, 256


def _rank(rank, world, uid, path, T, Tmax, chunks, regroup, shared, q, exchange="p2p"):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["ARTLITE_EP_EXCHANGE"] = exchange
    os.environ["ARTLITE_EP_CHUNKS"] = str(chunks)
    os.environ["ARTLITE_EP_REGROUP"] = regroup
    os.environ["ARTLITE_EP_TIMEOUT_MS"] = "20000"
    import torch
    torch.cuda.set_device(rank)
    from artlite_b200.moe.block import MoEBlock
    from oracle import moe_np
    layer, _, _ = moe_np.make_block(77, 1, qtype="Q4_0", E=E, H=H, F=F)
    x = moe_np.make_block(100 + rank, T, qtype="Q4_0", E=E, H=H, F=F)[1]
    # (max_tokens: the largest batch of any rank, which sizes what a rank can receive)
    ep = MoEBlock(hidden=H, n_experts=E, top_k=K, expert_ffn=F, max_tokens=Tmax, act_dtype="bf16", path=path,
                  device=rank, ep_rank=rank, ep_world=world)
    ep.set_weights(0, gate=layer.gate, up=layer.up, down=layer.down, router=layer.router, qtype="Q4_0")
    sh = None
    if shared:  # (the same shared expert on every rank: it is not sharded)
        rng = np.random.default_rng(9)
        Fs = 128
        sh = dict(gate=moe_np.random_blocks(rng, "Q4_0", Fs, H), up=moe_np.random_blocks(rng, "Q4_0", Fs, H),
                  down=moe_np.random_blocks(rng, "Q4_0", H, Fs), ffn=Fs, qtype="Q4_0",
                  gate_inp=(0.02 * rng.standard_normal(H)).astype(np.float32))
        ep.set_shared(0, **sh)
    ep.ep_init(uid)
    y_ep = ep.forward(x).copy()
    y_ep2 = ep.forward(x).copy()
    one = MoEBlock(hidden=H, n_experts=E, top_k=K, expert_ffn=F, max_tokens=T, act_dtype="bf16", path=path,
                   device=rank)
    one.set_weights(0, gate=layer.gate, up=layer.up, down=layer.down, router=layer.router, qtype="Q4_0")
    if sh:
        one.set_shared(0, **sh)
    y_one = one.forward(x)
    ep.close()
    one.close()
    a, b = moe_np.bf16_to_f32(y_ep), moe_np.bf16_to_f32(y_one)
    q.put((rank, float(moe_np.rel_max(a, b)), bool(np.array_equal(y_ep, y_one)), bool(np.array_equal(y_ep, y_ep2))))


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("path,T,chunks,regroup,shared,exchange", [
    ("tc", 300, 1, "0", False, "p2p"), ("tc", 300, 1, "0", False, "nccl"), ("tc", 300, 4, "0", False, "p2p"),
    ("tc", 300, 1, "1", False, "p2p"), ("gemv", 7, 1, "0", False, "p2p"), ("tc", 300, 1, "0", True, "p2p"),
    ("gemv", 7, 1, "0", True, "p2p")])
def test_ep_matches_single_gpu(path, T, chunks, regroup, shared, exchange, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from artlite_b200.moe.block import ep_unique_id
    uid = ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    Tmax = T + 13 * (world - 1)
    procs = [ctx.Process(target=_rank, args=(r, world, uid, path, T + 13 * r, Tmax, chunks, regroup, shared, q,
                                             exchange), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=10) for _ in range(world)]
    for rank, err, exact, repeat in res:
        assert err <= 1e-2 and exact and repeat, (rank, err, exact, repeat)


def _lonely_rank(uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["ARTLITE_EP_INIT_TIMEOUT_MS"] = "3000"
    import time
    import torch
    torch.cuda.set_device(0)
    from artlite_b200 import Error
    from artlite_b200.moe.block import MoEBlock
    ep = MoEBlock(hidden=H, n_experts=E, top_k=K, expert_ffn=F, max_tokens=8, act_dtype="bf16", device=0, ep_rank=0,
                  ep_world=2)
    t0 = time.monotonic()
    try:
        ep.ep_init(uid)
        q.put(("formed", 0.0))
    except Error as e:
        q.put((str(e), time.monotonic() - t0))
    ep.close()


def test_init_deadline_without_peers():
    """ep_init with a peer that never joins (rank 0 of 2 alone, one GPU): the communicator is non-blocking, the host's
    wait for it is bounded (ARTLITE_EP_INIT_TIMEOUT_MS = 3 s here), and past it the half-formed communicator is
    aborted and ep_init fails with ARTLITE_ETIMEOUT's message instead of waiting forever (nccl.h:151 non-blocking
    initialisation; SURVEY's failure-detection row: a watchdog on the communicator)."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    from artlite_b200.moe.block import ep_unique_id
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(ep_unique_id(), q), daemon=True)
    p.start()
    p.join(120)
    if p.exitcode is None:
        p.kill()
    assert p.exitcode == 0
    msg, took = q.get(timeout=10)
    assert "did not form within 3000 ms" in msg, msg
    assert 2.5 <= took <= 60, took


def _leaving_rank(rank, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["ARTLITE_EP_TIMEOUT_MS"] = "3000"
    import time
    import torch
    torch.cuda.set_device(rank)
    from artlite_b200 import Error
    from artlite_b200.moe.block import MoEBlock
    from oracle import moe_np
    layer, _, _ = moe_np.make_block(77, 1, qtype="Q4_0", E=E, H=H, F=F)
    x = moe_np.make_block(100 + rank, 6, qtype="Q4_0", E=E, H=H, F=F)[1]
    ep = MoEBlock(hidden=H, n_experts=E, top_k=K, expert_ffn=F, max_tokens=8, act_dtype="bf16", path="gemv",
                  device=rank, ep_rank=rank, ep_world=2)
    ep.set_weights(0, gate=layer.gate, up=layer.up, down=layer.down, router=layer.router, qtype="Q4_0")
    ep.ep_init(uid)
    ep.forward(x)  # (returns once the step is complete on this rank: nothing of it is in flight)
    if rank == 1:
        q.put((1, "left", 0.0))
        q.close()
        q.join_thread()  # (the message is out before the process ends)
        os._exit(0)  # leaves between steps, without a word to its peer
    time.sleep(2.0)
    t0 = time.monotonic()
    try:
        ep.forward(x)
        q.put((0, "returned", 0.0))
    except Error as e:
        q.put((0, str(e), time.monotonic() - t0))
    try:
        ep.forward(x)
        q.put((0, "again", 0.0))
    except Error as e:
        q.put((0, str(e), 0.0))
    ep.close()


def test_peer_leaves_between_steps():
    """Rank 1 of 2 leaves after a step; rank 0's next forward must not wait forever: its count exchange with the absent
    peer runs past ARTLITE_EP_TIMEOUT_MS (3 s), the library aborts the communicator (ncclCommAbort: the exchange's
    kernels on this GPU end) and the forward fails with ARTLITE_ETIMEOUT's message; the handle then refuses further
    expert-parallel forwards. NVLS off; the ranks are child processes on two GPUs."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from artlite_b200.moe.block import ep_unique_id
    uid = ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_leaving_rank, args=(r, uid, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = []
    while True:
        try:
            res.append(q.get(timeout=5))
        except Exception:
            break
    mine = [r for r in res if r[0] == 0]
    assert len(mine) == 2, res
    first, again = mine
    assert "did not complete within 3000 ms" in first[1], first
    assert 2.5 <= first[2] <= 60, first
    assert "expert parallelism needs artlite_moe_ep_init first" in again[1], again
