"""Expert parallelism on 2 and 4 GPUs (NCCL, one process per GPU): each rank owns 1/N of the experts and its own tokens;
the EP forward (token rows out by NCCL send / recv, local tcgen05 or GEMV experts, outputs back, local combine) must
equal, on every rank, the single-GPU block over the same tokens with all experts, with one or four expert chunks and
with the rows regrouped expert-major before the experts (the default from 8 ranks, forced here), and with a shared
expert (held whole by every rank, run on its own tokens). Skipped with fewer GPUs than ranks.
NVLS is off (NCCL_NVLS_ENABLE=0); the ranks are child processes."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, E, K, F = 512, 16, 4, 256


def _rank(rank, world, uid, path, T, Tmax, chunks, regroup, shared, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
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
@pytest.mark.parametrize("path,T,chunks,regroup,shared", [("tc", 300, 1, "0", False), ("tc", 300, 4, "0", False),
                                                          ("tc", 300, 1, "1", False), ("gemv", 7, 1, "0", False),
                                                          ("tc", 300, 1, "0", True), ("gemv", 7, 1, "0", True)])
def test_ep_matches_single_gpu(path, T, chunks, regroup, shared, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from artlite_b200.moe.block import ep_unique_id
    uid = ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    Tmax = T + 13 * (world - 1)
    procs = [ctx.Process(target=_rank, args=(r, world, uid, path, T + 13 * r, Tmax, chunks, regroup, shared, q), daemon=True)
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
