"""GPU parity of the block for the k-quant formats of the reference's real MoE files, and for layers whose down
tensor has its own type (Qwen3.6-35B-A3B Q4_K_M: Q4_K gate / up with Q5_K or Q6_K downs, tests/moe/test_prefill.py:1-5;
the formats' dequant: csrc/artlite/dequant.cpp:64-101), on the tcgen05 path where the format has a tensor-core stage
and on the decode path, against the oracle (ref.moe_ffn with the reference-exact fp32 dequant).

Tolerance: bf16 activations / the tcgen05 path's bf16 operands: rel_max <= 1e-2 (tests/numerics.py:50-53)."""

import numpy as np
import pytest

from oracle import moe_np
from tests.moe_helpers import make_block, oracle_y, orc, torch_moe_ffn, x_f32

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2


def run_checked(layer, x, T, path, k=8):
    b = make_block(layer, T, act="bf16", path=path, top_k=k)
    y = moe_np.bf16_to_f32(b.forward(x))
    dbg = b.debug(T)
    took = b.path(0)
    b.close()
    want = x_f32(x) @ layer.router.T
    assert moe_np.rel_max(dbg["logits"], want) < 1e-5
    ids, w = orc().route(dbg["logits"], k)
    assert np.array_equal(dbg["ids"], ids)
    return y, ids, w, took


@pytest.mark.parametrize("qtype,down", [("Q5_K", "Q5_K"), ("Q4_K", "Q5_K"), ("Q5_K", "Q4_K"), ("Q4_0", "Q5_K"),
                                        ("Q8_0", "Q5_K"), ("Q6_K", "Q6_K"), ("Q4_K", "Q6_K"), ("Q8_0", "Q6_K"),
                                        ("Q3_K", "Q3_K"), ("Q4_K", "Q3_K"), ("Q3_K", "Q6_K"), ("IQ4_NL", "IQ4_NL"),
                                        ("IQ4_XS", "IQ4_XS"), ("Q4_K", "IQ4_XS"), ("IQ4_NL", "Q6_K"), ("Q4_1", "Q4_1"),
                                        ("Q4_1", "Q6_K")])
def test_tcgen05_q5_k_q6_k_and_mixed(qtype, down):
    """Q5_K, Q6_K, Q3_K, IQ4_NL, IQ4_XS and Q4_1 on the tensor cores, alone and mixed with the other formats (E=16,
    H=512, F=256, T=200: ragged groups; Q6_K, Q3_K and IQ4_XS rows (420 / 210, 220 / 110, 272 / 136 bytes) are not
    16-byte pitched and go through the copy warp; the IQ4 code values by byte permutes)."""
    layer, x, _ = moe_np.make_block(90, 200, qtype=qtype, down_qtype=down, E=16, H=512, F=256)
    y, ids, w, took = run_checked(layer, x, 200, "tc")
    assert took == "tc"
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


@pytest.mark.parametrize("down", ["Q6_K", "Q5_K"])
def test_q4_k_m_prefill_shape(down):
    """A Q4_K_M-style layer at config 3's size (T=4096, H=2048, E=128, K=8, F=768, Q4_K gate / up, Q6_K or Q5_K down)
    on the tcgen05 path, every token against the torch fp32 reference, which is pinned to the NumPy oracle on a
    stride."""
    T = 4096
    layer, x, _ = moe_np.make_block(91, T, qtype="Q4_K", down_qtype=down)
    y, ids, w, took = run_checked(layer, x, T, "auto")
    assert took == "tc"
    ref = torch_moe_ffn(layer, x, ids, w)
    assert moe_np.rel_max(y, ref) <= BF16_TOL
    tok = np.arange(0, T, 128)
    want = oracle_y(layer, x, ids, w, tokens=tok)
    assert moe_np.rel_max(ref[tok], want) <= 1e-4


@pytest.mark.parametrize("down,T", [("Q6_K", 16), ("Q6_K", 300), ("Q5_K", 16), ("Q5_K", 5), ("Q6_K", 1), ("Q6_K", 4),
                                    ("Q6_K", 64)])
def test_mixed_down_decode_and_prefill(down, T):
    """Q4_K gate / up with a Q6_K or Q5_K down through the block's automatic path choice, decode and prefill sizes."""
    layer, x, _ = moe_np.make_block(92 + T, T, qtype="Q4_K", down_qtype=down, E=32, H=1024, F=512)
    y, ids, w, _ = run_checked(layer, x, T, "auto")
    assert moe_np.rel_max(y, oracle_y(layer, x, ids, w)) <= BF16_TOL


@pytest.mark.parametrize("T", [1, 16, 64])
def test_q4_k_m_decode_shape(T):
    """A Q4_K_M-style layer (Q4_K gate / up, Q6_K down) at the benchmark's decode shape (H=2048, E=128, K=8, F=768) on
    the small-batch tensor-core GEMVs (the Q6_K down kernel: whole items by one bulk copy, h in the mma's natural k
    order), every token against the torch fp32 reference, which is pinned to the NumPy oracle on a stride."""
    layer, x, _ = moe_np.make_block(93 + T, T, qtype="Q4_K", down_qtype="Q6_K")
    y, ids, w, took = run_checked(layer, x, T, "auto")
    assert took == "gemv"
    ref = torch_moe_ffn(layer, x, ids, w)
    assert moe_np.rel_max(y, ref) <= BF16_TOL
    tok = np.arange(0, T, max(1, T // 4))
    assert moe_np.rel_max(ref[tok], oracle_y(layer, x, ids, w, tokens=tok)) <= 1e-4


def test_q3_k_prefill_shape():
    """Q3_K experts (the reference's low-bit MoE files: dequant.cpp:103-117) at a prefill size of the benchmark's shape
    (T=2048, H=2048, E=128, K=8, F=768) on the tensor cores, every token against the torch fp32 reference, which is
    pinned to the NumPy oracle on a stride."""
    T = 2048
    layer, x, _ = moe_np.make_block(95, T, qtype="Q3_K")
    y, ids, w, took = run_checked(layer, x, T, "auto")
    assert took == "tc"
    ref = torch_moe_ffn(layer, x, ids, w)
    assert moe_np.rel_max(y, ref) <= BF16_TOL
    tok = np.arange(0, T, 128)
    assert moe_np.rel_max(ref[tok], oracle_y(layer, x, ids, w, tokens=tok)) <= 1e-4
