"""GPU parity of the whole block at the benchmarked configurations' full sizes, on every token.

The reference checks its whole block, not samples of it (tests/moe/test_prefill.py:287-407). Here every output row
of a full-size forward is compared with ``ref.moe_ffn`` evaluated in plain PyTorch fp32 on the GPU
(``tests.moe_helpers.torch_moe_ffn``: the weights dequantised exactly by the C oracle, fp32 products without TF32),
which is itself pinned to the NumPy oracle on a token subset in each test. Routing is checked bit for bit against the
oracle's routing of the GPU's own logits.

Tolerances (rel_max = max|a - b| / max|b|, tests/numerics.py:50-53): bf16 activations and the tcgen05 path (weights
rounded once to bf16 after the exact fp32 dequant, h and y in bf16): rel_max <= 1e-2; the torch fp32 reference
against the NumPy oracle: rel_max <= 1e-4 (summation order only).

Repetition: the config-3 case runs ten forwards, each in a new block whose device buffers were first poisoned (the
memory the block allocates last held 0xFF bytes: bf16 NaN patterns), and requires the ten outputs to be bit-identical
(a read of a row no kernel wrote, or a race between kernels, shows up as a difference)."""

import numpy as np
import pytest

from oracle import moe_np
from tests.moe_helpers import make_block, oracle_y, orc, torch_moe_ffn, x_f32

pytestmark = pytest.mark.gpu

BF16_TOL, REF_TOL = 1e-2, 1e-4
# router logits against the fp32 product: the reference's own router bound (within 5e-5, tests/moe/test_prefill.py:85-91);
# at H = 4096 the tensor cores' fp32 accumulation over three bf16 planes lands near 1.5e-5
LOGIT_TOL = 5e-5


def poison_device_memory(gib: float = 4.0) -> None:
    """Fill `gib` GiB of fresh device memory with 0xFF bytes and give it back to the driver, so that the next
    allocations (the block's workspaces) start from NaN patterns rather than zeros."""
    import torch
    buf = torch.empty(int(gib * (1 << 30)), dtype=torch.uint8, device="cuda")
    buf.fill_(0xFF)
    torch.cuda.synchronize()
    del buf
    torch.cuda.empty_cache()


def check_routing(dbg, x, layer, k, bias=None):
    want = x_f32(x) @ layer.router.T
    if bias is not None:
        want = want + bias
    assert moe_np.rel_max(dbg["logits"], want) < LOGIT_TOL
    ids, w = orc().route(dbg["logits"], k)
    assert np.array_equal(dbg["ids"], ids)
    assert np.abs(dbg["w"].astype(np.float64) - w).max() <= 2 ** -23
    off, perm, _ = orc().dispatch(ids, layer.E)
    assert np.array_equal(dbg["offsets"], off) and np.array_equal(dbg["perm"], perm)
    return ids, w


def check_against_references(layer, x, ids, w, y, stride_tokens):
    """y (fp32) against the torch fp32 reference on every token, and that reference against the NumPy oracle on
    the given tokens."""
    ref = torch_moe_ffn(layer, x, ids, w)
    err = moe_np.rel_max(y, ref)
    assert err <= BF16_TOL, f"rel_max {err} over all {y.shape[0]} tokens"
    rows_bad = np.nonzero(np.abs(y - ref).max(1) > BF16_TOL * np.abs(ref).max())[0]
    assert rows_bad.size == 0, f"tokens off: {rows_bad[:16]}"
    want = oracle_y(layer, x, ids, w, tokens=stride_tokens)
    assert moe_np.rel_max(ref[stride_tokens], want) <= REF_TOL
    assert moe_np.rel_max(y[stride_tokens], want) <= BF16_TOL
    return err


def test_config3_every_token_repeated():
    """Config 3 (T=4096, Q8_0, Zipf(1.1)-skewed routing, tcgen05 path): all 4096 tokens against the reference, and
    ten forwards in ten fresh blocks over poisoned memory, bit-identical."""
    T = 4096
    layer, x, bias = moe_np.make_block(3, T, qtype="Q8_0", zipf=1.1)
    outs = []
    dbg = None
    for rep in range(10):
        poison_device_memory()
        b = make_block(layer, T, act="bf16", path="tc")
        b.set_router_bias(0, bias)
        outs.append(b.forward(x).copy())
        if rep == 0:
            dbg = b.debug(T)
        b.close()
    for rep in range(1, 10):
        diff = np.nonzero(outs[rep] != outs[0])
        assert diff[0].size == 0, f"repeat {rep}: {diff[0].size} values differ, tokens {np.unique(diff[0])[:16]}"
    ids, w = check_routing(dbg, x, layer, 8, bias=bias)
    counts = np.bincount(ids.ravel(), minlength=128)
    assert counts.max() > 4 * counts.mean()  # (the skew is there)
    check_against_references(layer, x, ids, w, moe_np.bf16_to_f32(outs[0]), np.arange(0, T, T // 32))


def test_config3_same_block_repeated():
    """Config 3 forwarded ten times through one block (the workspaces reused with the last forward's contents):
    bit-identical outputs."""
    T = 4096
    layer, x, bias = moe_np.make_block(3, T, qtype="Q8_0", zipf=1.1)
    b = make_block(layer, T, act="bf16", path="tc")
    b.set_router_bias(0, bias)
    first = b.forward(x).copy()
    for rep in range(9):
        y = b.forward(x)
        assert np.array_equal(y, first), f"repeat {rep + 1}"
    b.close()


@pytest.mark.parametrize("qtype", ["Q4_0", "Q4_K"])
def test_config4_bench_shape(qtype):
    """Config 4's benchmarked layer shape exactly: T=16384, H=2048, E=128, K=8, F=768 on the tcgen05 path; every
    token against the reference, against the dequant-GEMV path on every token, and against the NumPy oracle on a
    256-token stride."""
    T = 16384
    poison_device_memory()
    layer, x, _ = moe_np.make_block(44, T, qtype=qtype)
    b = make_block(layer, T, act="bf16", path="tc")
    y_tc = b.forward(x).copy()
    dbg = b.debug(T)
    b.close()
    ids, w = check_routing(dbg, x, layer, 8)
    yf = moe_np.bf16_to_f32(y_tc)
    check_against_references(layer, x, ids, w, yf, np.arange(0, T, 256))
    b = make_block(layer, T, act="bf16", path="gemv")
    y_gemv = moe_np.bf16_to_f32(b.forward(x))
    b.close()
    assert moe_np.rel_max(yf, y_gemv) <= BF16_TOL


def test_config5_full_expert_count():
    """Config 5's block (H=4096, F=1536, Q4_0) at its full routing shape: E=128, K=8, an 8192-token prefill on the
    tcgen05 path (every token against the reference, the NumPy oracle on a stride) and a 64-token decode batch."""
    T = 8192
    layer, x, _ = moe_np.make_block(55, T, qtype="Q4_0", H=4096, F=1536)
    b = make_block(layer, T, act="bf16", path="tc")
    y = moe_np.bf16_to_f32(b.forward(x))
    dbg = b.debug(T)
    ids, w = check_routing(dbg, x, layer, 8)
    check_against_references(layer, x, ids, w, y, np.arange(0, T, 512))
    y64 = moe_np.bf16_to_f32(b.forward(x[:64]))
    dbg = b.debug(64)
    b.close()
    ids, w = check_routing(dbg, x[:64], layer, 8)
    assert moe_np.rel_max(y64, torch_moe_ffn(layer, x[:64], ids, w)) <= BF16_TOL


@pytest.mark.parametrize("qtype,T,zipf", [("Q4_0", 16384, 0.0), ("Q8_0", 4096, 1.1), ("Q4_K", 16384, 0.0)])
def test_tcgen05_many_repeats_bit_identical(qtype, T, zipf):
    """Forty forwards of a benchmarked shape in one block, device buffers in and out: every output bit-identical to
    the first, and the first within tolerance of the reference on every token. The tcgen05 pipeline's waits are the
    kind of code whose races show up as a rare wrong tile: this is the repetition harness for them."""
    import torch
    layer, x, bias = moe_np.make_block(45, T, qtype=qtype, zipf=zipf)
    b = make_block(layer, T, act="bf16", path="tc")
    if zipf:
        b.set_router_bias(0, bias)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    yd = torch.empty_like(xd)
    outs = []
    stream = torch.cuda.Stream()  # (the forwards and the copies in one stream order; not the legacy default stream,
    torch.cuda.synchronize()      # whose handle 0 would mean "the block's own stream" to forward_ptr)
    with torch.cuda.stream(stream):
        for _ in range(40):
            b.forward_ptr(xd.data_ptr(), yd.data_ptr(), T, stream=stream.cuda_stream)
            outs.append(yd.clone())
    torch.cuda.synchronize()
    b.sync()
    first = outs[0]
    bad = [i for i, o in enumerate(outs) if not torch.equal(o, first)]
    dbg = b.debug(T)
    b.close()
    assert not bad, f"forwards {bad} differ from the first"
    ids, w = check_routing(dbg, x, layer, 8, bias=bias if zipf else None)
    y = moe_np.bf16_to_f32(first.cpu().numpy().view(np.uint16))
    assert moe_np.rel_max(y, torch_moe_ffn(layer, x, ids, w)) <= BF16_TOL
