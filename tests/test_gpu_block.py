"""GPU parity of the whole block (router -> routing -> dispatch -> SwiGLU experts from raw GGUF blocks -> combine)
through the C ABI (artlite_b200.moe.block.MoEBlock), against the oracle: the reference's ref.moe_ffn restated in NumPy
with the reference-exact fp32 dequant (tests/moe_helpers.py), under the routing the oracle computes from the GPU's own
logits (which must equal the GPU's routing bit for bit).

Tolerances (max relative error rel_max = max|a - b| / max|b|, tests/numerics.py:50-53):
  - fp32 path (the dequant-GEMVs: fp32 dequant, fp32 accumulation, fp32 x and y): rel_max <= 2e-3;
  - bf16 (bf16 x / y, or the tcgen05 path: weights rounded to bf16 after the exact fp32 dequant, h and y in bf16):
    rel_max <= 1e-2."""

import numpy as np
import pytest

from oracle import moe_np
from tests.moe_helpers import expert_fn, make_block, oracle_y, orc, x_f32

pytestmark = pytest.mark.gpu

FP32_TOL, BF16_TOL = 2e-3, 1e-2


def run(layer, x, *, act, path, T, gating="softmax", k=8, bias=None):
    b = make_block(layer, T, act=act, path=path, gating=gating, top_k=k)
    if bias is not None:
        b.set_router_bias(0, bias)
    y = b.forward(x)
    dbg = b.debug(T)
    b.close()
    return (moe_np.bf16_to_f32(y) if act == "bf16" else y), dbg


def check_routing(dbg, x, layer, k, gating="softmax", bias=None):
    """GPU logits close to the fp32 product; GPU routing == the oracle's routing of those logits, bit for bit."""
    want = x_f32(x) @ layer.router.T
    if bias is not None:
        want = want + bias
    assert moe_np.rel_max(dbg["logits"], want) < 1e-5
    ids, w = orc().route(dbg["logits"], k, gating=gating)
    assert np.array_equal(dbg["ids"], ids)
    assert np.abs(dbg["w"].astype(np.float64) - w).max() <= 2 ** -23
    off, perm, _ = orc().dispatch(ids, layer.E)
    assert np.array_equal(dbg["offsets"], off) and np.array_equal(dbg["perm"], perm)
    return ids, w


def test_config1_fp32(golden):
    """benchmark config 1 (T=16, H=2048, E=128, K=8, F=768, Q4_0, fp32 x) against the reference's own moe_ffn output
    (tests/golden: ref.moe_route + ref.moe_ffn with gguf-py's dequant)."""
    layer, x, _ = moe_np.make_block(0, 16, qtype="Q4_0", x_bf16=False)
    y, dbg = run(layer, x, act="f32", path="gemv", T=16)
    ids, w = check_routing(dbg, x, layer, 8)
    assert np.array_equal(ids, golden["block_c1_ids"])
    assert moe_np.rel_max(y, golden["block_c1_y"]) <= FP32_TOL
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= FP32_TOL


@pytest.mark.parametrize("B", [1, 4, 12, 16, 64])
def test_decode_q4k(B):
    """Config 2's decode batches (Q4_K, bf16 x) on the dequant-GEMV path: below 16 tokens the small-batch tensor-core
    GEMVs (12: every token slot staged), from 16 the fused decode kernel."""
    layer, x, _ = moe_np.make_block(B, B, qtype="Q4_K")
    y, dbg = run(layer, x, act="bf16", path="gemv", T=B)
    ids, w = check_routing(dbg, x, layer, 8)
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


@pytest.mark.parametrize("qtype", ["Q4_0", "Q8_0", "Q4_K"])
def test_decode_fp32_tight(qtype):
    """fp32 activations through the GEMV path: the tight bound."""
    layer, x, _ = moe_np.make_block(5, 24, qtype=qtype, x_bf16=False, E=32, H=512, F=256)
    y, dbg = run(layer, x, act="f32", path="gemv", T=24)
    ids, w = check_routing(dbg, x, layer, 8)
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= FP32_TOL


@pytest.mark.parametrize("qtype", ["Q4_1", "Q5_K", "Q6_K", "Q3_K", "IQ4_NL", "IQ4_XS"])
def test_decode_generic_formats(qtype):
    """The formats without a register-decoding GEMV (the generic staged kernel) through the block, fp32 tight."""
    layer, x, _ = moe_np.make_block(6, 12, qtype=qtype, x_bf16=False, E=16, H=512, F=256)
    y, dbg = run(layer, x, act="f32", path="gemv", T=12)
    ids, w = check_routing(dbg, x, layer, 8)
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= FP32_TOL


@pytest.mark.parametrize("qtype,down", [("Q3_K", "Q3_K"), ("IQ4_XS", "IQ4_XS"), ("IQ4_NL", "Q6_K"), ("Q4_K", "Q3_K")])
def test_low_bit_formats_prefill_and_mixed(qtype, down):
    """Q3_K, IQ4_NL and IQ4_XS experts (the reference's low-bit files: dequant.cpp:103-140), alone and under another
    down type, through the block's automatic path at a prefill size and a decode size, bf16 activations."""
    for T in (300, 6):
        layer, x, _ = moe_np.make_block(40 + T, T, qtype=qtype, down_qtype=down, E=16, H=512, F=256)
        y, dbg = run(layer, x, act="bf16", path="auto", T=T)
        ids, w = check_routing(dbg, x, layer, 8)
        assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL, T


@pytest.mark.parametrize("qtype", ["Q4_0", "Q8_0", "Q4_K"])
def test_tcgen05_small(qtype):
    """The tcgen05 grouped GEMMs at a small shape: E=16, H=512, F=256, T=200 (ragged expert groups)."""
    layer, x, _ = moe_np.make_block(11, 200, qtype=qtype, E=16, H=512, F=256)
    y, dbg = run(layer, x, act="bf16", path="tc", T=200)
    ids, w = check_routing(dbg, x, layer, 8)
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


@pytest.mark.parametrize("qtype", ["Q4_0", "Q8_0"])
def test_tcgen05_full_shape(qtype):
    """The tcgen05 path at the Qwen3-30B-A3B shape (H=2048, E=128, K=8, F=768), T=512, checked on 48 tokens."""
    T = 512
    layer, x, _ = moe_np.make_block(21, T, qtype=qtype)
    y, dbg = run(layer, x, act="bf16", path="tc", T=T)
    ids, w = check_routing(dbg, x, layer, 8)
    tok = np.arange(0, T, T // 48)
    assert moe_np.rel_max(y[tok], oracle_y(layer, x, ids, w, tokens=tok)) <= BF16_TOL


@pytest.mark.parametrize("path", ["tc", "gemv"])
def test_large_expert_shape(path):
    """Config 5's expert shape (H=4096, F=1536, Q4_0) at E=8, K=2, T=64, on both paths."""
    layer, x, _ = moe_np.make_block(50, 64, qtype="Q4_0", E=8, H=4096, F=1536)
    y, dbg = run(layer, x, act="bf16", path=path, T=64, k=2)
    ids, w = check_routing(dbg, x, layer, 2)
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


@pytest.mark.parametrize("path,T,gated", [("tc", 200, True), ("gemv", 5, True), ("tc", 130, False)])
def test_shared_expert(path, T, gated):
    """The shared expert (ref.shared_expert, tests/moe/ref.py:55-60): the routed sum + sigmoid(x . g) swiglu_s(x),
    in one fp32 sum; gated and ungated, both expert paths; and through a captured graph."""
    import torch
    H, Fs = 512, 256
    layer, x, _ = moe_np.make_block(60, T, qtype="Q4_K", E=16, H=H, F=256)
    rng = np.random.default_rng(61)
    sg, su = moe_np.random_blocks(rng, "Q4_K", Fs, H), moe_np.random_blocks(rng, "Q4_K", Fs, H)
    sd = moe_np.random_blocks(rng, "Q4_K", H, Fs)
    g = (rng.standard_normal(H) * 0.05).astype(np.float32) if gated else None
    b = make_block(layer, T, act="bf16", path=path)
    b.set_shared(0, gate=sg, up=su, down=sd, ffn=Fs, qtype="Q4_K", gate_inp=g)
    y_raw = b.forward(x)
    dbg = b.debug(T)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    yd = torch.empty_like(xd)
    b.forward_graph(xd.data_ptr(), yd.data_ptr(), T)
    b.sync()
    y_graph = yd.cpu().numpy().view(np.uint16)
    b.close()
    assert np.array_equal(y_graph, y_raw)
    ids, w = check_routing(dbg, x, layer, 8)
    want = oracle_y(layer, x, ids, w) + moe_np.shared_expert(x_f32(x), moe_np.dequant("Q4_K", sg, H),
                                                             moe_np.dequant("Q4_K", su, H),
                                                             moe_np.dequant("Q4_K", sd, Fs), g)
    assert moe_np.rel_max(moe_np.bf16_to_f32(y_raw), want) <= BF16_TOL


@pytest.mark.parametrize("path,T", [("tc", 300), ("gemv", 6), ("gemv", 24)])
def test_flint_shape_sigmoid_top6(path, T):
    """The reference's other MoE family's routing shape: E=256 experts, sigmoid gating, top-6, F=512 (Q4_K)."""
    layer, x, _ = moe_np.make_block(70 + T, T, qtype="Q4_K", E=256, H=512, F=512)
    y, dbg = run(layer, x, act="bf16", path=path, T=T, gating="sigmoid", k=6)
    ids, w = check_routing(dbg, x, layer, 6, gating="sigmoid")
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


def test_prefill_zipf_q8():
    """Config 3 (T=4096, Q8_0, Zipf(1.1)-skewed routing, bf16): the dispatch in full, outputs on 32 tokens."""
    T = 4096
    layer, x, bias = moe_np.make_block(3, T, qtype="Q8_0", zipf=1.1)
    y, dbg = run(layer, x, act="bf16", path="tc", T=T, bias=bias)
    ids, w = check_routing(dbg, x, layer, 8, bias=bias)
    counts = np.bincount(ids.ravel(), minlength=128)
    assert counts.max() > 4 * counts.mean()  # (the skew is there)
    tok = np.arange(0, T, T // 32)
    assert moe_np.rel_max(y[tok], oracle_y(layer, x, ids, w, tokens=tok)) <= BF16_TOL


@pytest.mark.parametrize("qtype", ["Q4_0", "Q8_0", "Q4_K"])
def test_tcgen05_single_and_pair_agree(qtype, monkeypatch):
    """The one-CTA and the two-CTA (cta_group::2) tcgen05 kernels agree (the same bf16 operands and K order: equal up
    to the tensor core's accumulation within an instruction); the shape splits into pairs (F % 128 == 0,
    H % 256 == 0)."""
    layer, x, _ = moe_np.make_block(12, 333, qtype=qtype, E=16, H=512, F=256)
    monkeypatch.setenv("ARTLITE_TC_PAIR", "0")
    y1, _ = run(layer, x, act="bf16", path="tc", T=333)
    monkeypatch.setenv("ARTLITE_TC_PAIR", "1")
    y2, dbg = run(layer, x, act="bf16", path="tc", T=333)
    assert moe_np.rel_max(y2, y1) <= 2e-3
    ids, w = check_routing(dbg, x, layer, 8)
    assert moe_np.rel_max(y2, oracle_y(layer, x, ids, w)) <= BF16_TOL


def test_paths_agree():
    """The GEMV and the tcgen05 path on the same input (Q4_0, T=256)."""
    layer, x, _ = moe_np.make_block(8, 256, qtype="Q4_0", E=32, H=1024, F=512)
    y1, _ = run(layer, x, act="bf16", path="gemv", T=256)
    y2, _ = run(layer, x, act="bf16", path="tc", T=256)
    assert moe_np.rel_max(y2, y1) <= BF16_TOL


def test_tiny_and_sigmoid():
    """Tiny shapes (E=8, K=2, T=1 and 3) and sigmoid gating (Flint's), on both paths."""
    for T in (1, 3):
        layer, x, _ = moe_np.make_block(30 + T, T, qtype="Q4_0", E=8, H=256, F=256)
        for path in ("gemv", "tc"):
            for gating in ("softmax", "sigmoid"):
                y, dbg = run(layer, x, act="bf16", path=path, T=T, gating=gating, k=2)
                ids, w = check_routing(dbg, x, layer, 2, gating=gating)
                assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


def test_repeatable():
    """The same input twice: bit-identical outputs (the combine sums in slot order, no atomics)."""
    layer, x, _ = moe_np.make_block(9, 300, qtype="Q4_0", E=32, H=512, F=256)
    b = make_block(layer, 300, act="bf16", path="tc")
    y1 = b.forward(x).copy()
    y2 = b.forward(x)
    b.close()
    assert np.array_equal(y1, y2)


def test_zero_tokens_and_errors():
    from artlite_b200 import Error
    layer, x, _ = moe_np.make_block(1, 4, qtype="Q4_0", E=8, H=256, F=256)
    b = make_block(layer, 4, act="bf16", path="auto", top_k=2)
    assert b.forward(x[:0]).shape == (0, 256)
    with pytest.raises(Error, match="max_tokens"):
        b.forward(np.zeros((5, 256), np.uint16))
    b.close()


@pytest.mark.parametrize("path,T", [("gemv", 4), ("tc", 260)])
def test_forward_graph_matches_forward(path, T):
    """A forward captured as a CUDA graph (device x / y) gives the eager forward's output bit for bit, on its first
    (capturing) call and on replays with new input values in the same buffers."""
    import torch
    layer, x, _ = moe_np.make_block(40, T, qtype="Q4_K", E=32, H=512, F=256)
    b = make_block(layer, T, act="bf16", path=path)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    yd = torch.empty_like(xd)
    for rep in range(3):
        if rep:
            xd.copy_(torch.from_numpy(np.roll(x, rep, axis=0).view(np.int16)))
        want = b.forward(xd.cpu().numpy().view(np.uint16))
        b.forward_graph(xd.data_ptr(), yd.data_ptr(), T)
        b.sync()
        assert np.array_equal(yd.cpu().numpy().view(np.uint16), want)
    b.close()


@pytest.mark.parametrize("path,T,act", [("tc", 300, "bf16"), ("gemv", 1, "bf16"), ("gemv", 5, "bf16"),
                                        ("gemv", 24, "bf16"), ("gemv", 64, "bf16"), ("gemv", 3, "f32"),
                                        ("gemv", 16, "f32")])
def test_norm_and_residual(path, T, act):
    """A layer with its input norm and residual (artlite_moe_set_norm): y = x + moe(rms_norm(x, w, eps)), against
    np_ops.rms_norm restated and ref.moe_ffn on the normed rows (rounded to the activation dtype, as the block routes
    and computes on them); the norm in the CTA-per-expert router (T <= 16 below the fused kernel) and in the fused
    decode kernel's first phase, and the norm kernel before the tcgen05 path."""
    qtype = "Q4_K" if act == "bf16" else "Q4_0"
    layer, x, _ = moe_np.make_block(80 + T, T, qtype=qtype, E=16, H=512, F=256, x_bf16=act == "bf16")
    wn = (1.0 + 0.1 * np.random.default_rng(5).standard_normal(layer.H)).astype(np.float32)
    eps = 1e-6
    b = make_block(layer, T, act=act, path=path)
    b.set_norm(0, wn, eps=eps)
    y = b.forward(x)
    dbg = b.debug(T)
    b.close()
    xf = x_f32(x)
    xn = moe_np.rms_norm(xf, wn, eps)
    if act == "bf16":
        xn = moe_np.bf16_to_f32(moe_np.to_bf16_bits(xn))
    assert moe_np.rel_max(dbg["logits"], xn @ layer.router.T) < 1e-5
    ids, w = orc().route(dbg["logits"], 8)
    assert np.array_equal(dbg["ids"], ids)
    want = xf + moe_np.moe_ffn(xn, ids, w, expert_fn(layer))
    got = moe_np.bf16_to_f32(y) if act == "bf16" else y
    assert moe_np.rel_max(got, want) <= (BF16_TOL if act == "bf16" or path == "tc" else FP32_TOL)


@pytest.mark.parametrize("act", ["f32", "bf16"])
@pytest.mark.parametrize("T", [1, 5, 12, 16, 40, 300])
def test_norm_rows_exact(act, T):
    """The normed rows bit for bit against np_ops.rms_norm restated: a router equal to the identity (E = H = 256) makes
    each logit one normed value exactly, on every path that norms: the CTA-per-expert router (up to 16 tokens below the
    fused kernel), the fused decode kernel's phase 0, the norm kernel (prefill sizes). Random rows, and (f32) rows of
    equal values under an eps sweep that puts v / d within a few float64 units of a float32 midpoint, where the norm's
    one-product division must fall back to the division itself."""
    import dataclasses
    layer, x, _ = moe_np.make_block(900 + T, T, qtype="Q4_0", E=256, H=256, F=256, x_bf16=act == "bf16")
    layer = dataclasses.replace(layer, router=np.eye(256, dtype=np.float32))
    b = make_block(layer, T, act=act, path="auto")
    wn = (1.0 + 0.1 * np.random.default_rng(9).standard_normal(256)).astype(np.float32)
    b.set_norm(0, wn, eps=1e-6)
    b.forward(x)
    want = moe_np.rms_norm(x_f32(x), wn, 1e-6)
    if act == "bf16":
        want = moe_np.bf16_to_f32(moe_np.to_bf16_bits(want))
    assert np.array_equal(b.debug(T)["logits"].view(np.uint32), want.view(np.uint32))
    if act == "f32":
        x3 = np.full((T, 256), 3.0, np.float32)
        ones = np.ones(256, np.float32)
        for j in range(0, 26):
            eps = 9.0 * 2.0 ** -24 + j * 2.0 ** -49
            b.set_norm(0, ones, eps=eps)
            b.forward(x3)
            want = moe_np.rms_norm(x3, ones, eps)
            assert np.array_equal(b.debug(T)["logits"].view(np.uint32), want.view(np.uint32)), j
    b.close()


def _norm_case(qtype, down, act, T, shared):
    layer, x, _ = moe_np.make_block(500 + T, T, qtype=qtype, down_qtype=down or "", E=16, H=512, F=256,
                                    x_bf16=act == "bf16")
    b = make_block(layer, T, act=act, path="gemv")
    b.set_norm(0, (1.0 + 0.1 * np.random.default_rng(6).standard_normal(layer.H)).astype(np.float32), eps=1e-5)
    if shared:
        rng = np.random.default_rng(7)
        b.set_shared(0, gate=moe_np.random_blocks(rng, "Q4_K", 256, 512), up=moe_np.random_blocks(rng, "Q4_K", 256, 512),
                     down=moe_np.random_blocks(rng, "Q4_K", 512, 256), ffn=256, qtype="Q4_K",
                     gate_inp=(rng.standard_normal(512) * 0.02).astype(np.float32))
    return b, x


@pytest.mark.parametrize("qtype,down,act,T,shared", [
    ("Q4_K", None, "bf16", 1, False), ("Q4_K", None, "bf16", 5, False), ("Q4_K", None, "bf16", 16, False),
    ("Q4_K", None, "bf16", 40, False), ("Q4_K", "Q6_K", "bf16", 16, False), ("Q4_K", None, "bf16", 4, True),
    ("Q4_0", None, "f32", 3, False), ("Q4_0", None, "f32", 12, False), ("Q8_0", None, "bf16", 24, False)])
def test_norm_fused_equals_norm_kernel(monkeypatch, qtype, down, act, T, shared):
    """The norm done inside the kernel that first reads the rows (the CTA-per-expert router, the fused decode
    kernel's phase 0; with a shared expert and a Q6_K down too) gives the norm kernel's output bit for bit
    (ARTLITE_NORM_FUSE=0: the norm kernel first), on repeated forwards and on graph replays (the norm's counters
    start from zero every launch)."""
    import torch
    b, x = _norm_case(qtype, down, act, T, shared)
    monkeypatch.setenv("ARTLITE_NORM_FUSE", "0")
    want = b.forward(x)
    want_lg = b.debug(T)["logits"]
    monkeypatch.delenv("ARTLITE_NORM_FUSE")
    for _ in range(3):
        got = b.forward(x)
        assert np.array_equal(got.view(np.uint32 if act == "f32" else np.uint16),
                              want.view(np.uint32 if act == "f32" else np.uint16))
        assert np.array_equal(b.debug(T)["logits"].view(np.uint32), want_lg.view(np.uint32))
    xd = torch.from_numpy(x.view(np.int16 if act == "bf16" else np.int32)).cuda()
    yd = torch.empty_like(xd)
    for _ in range(3):
        b.forward_graph(xd.data_ptr(), yd.data_ptr(), T)
        b.sync()
        assert np.array_equal(yd.cpu().numpy(), want.view(np.int16 if act == "bf16" else np.int32))
    b.close()


@pytest.mark.parametrize("T,gated", [(16, True), (64, True), (24, False)])
def test_qwen35moe_decode_shared_fused(T, gated):
    """The reference's own MoE decode shape (qwen35moe: H=2048, E=256, K=8, F=512, a shared expert of FFN 512, Q4_K)
    at decode batches that take the fused decode kernel, the shared expert inside it: the routed sum plus
    sigmoid(x . g) swiglu_s(x) (ref.moe_ffn + ref.shared_expert, tests/moe/ref.py:43-60), gated and ungated."""
    H, E, F, Fs = 2048, 256, 512, 512
    layer, x, _ = moe_np.make_block(100 + T, T, qtype="Q4_K", E=E, H=H, F=F)
    rng = np.random.default_rng(101)
    sg, su = moe_np.random_blocks(rng, "Q4_K", Fs, H), moe_np.random_blocks(rng, "Q4_K", Fs, H)
    sd = moe_np.random_blocks(rng, "Q4_K", H, Fs)
    g = (rng.standard_normal(H) * 0.02).astype(np.float32) if gated else None
    b = make_block(layer, T, act="bf16", path="auto")
    b.set_shared(0, gate=sg, up=su, down=sd, ffn=Fs, qtype="Q4_K", gate_inp=g)
    y = moe_np.bf16_to_f32(b.forward(x))
    took = b.path(0)
    dbg = b.debug(T)
    b.close()
    assert took == "gemv"
    ids, w = check_routing(dbg, x, layer, 8)
    want = oracle_y(layer, x, ids, w) + moe_np.shared_expert(x_f32(x), moe_np.dequant("Q4_K", sg, H),
                                                             moe_np.dequant("Q4_K", su, H),
                                                             moe_np.dequant("Q4_K", sd, Fs), g)
    assert moe_np.rel_max(y, want) <= BF16_TOL
