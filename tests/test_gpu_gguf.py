"""A GGUF file to HBM to a forward, on the GPU: the path from the reference's loader (GGUFFile.tensor's zero-copy raw
views, src/artlite/gguf_model.py:494-506, and the MoE configuration from the metadata, model_config.py:853-898) into
the block.

The file is written by gguf-py's own GGUFWriter (the reference's pinned dependency), read by artlite_b200.gguf, and
its raw views are handed to set_weights as they are: the bytes in HBM must equal the file's bytes (no conversion),
and a forward must match the oracle (ref.moe_ffn with the reference-exact dequant of the file's tensors) on the
tcgen05 path and on the decode path. The down tensor has its own type (Q8_0 under Q4_0 gate / up), as the
reference's mixed-type files have."""

import ctypes

import numpy as np
import pytest

from artlite_b200.gguf import GGUFFile
from oracle import moe_np
from tests.moe_helpers import orc, x_f32
from tests.test_gguf import write_with_gguf_py

pytestmark = pytest.mark.gpu


def device_bytes(ptr: int, n: int) -> np.ndarray:
    rt = ctypes.CDLL("libcudart.so.12")
    out = np.empty(n, np.uint8)
    rc = rt.cudaMemcpy(ctypes.c_void_p(out.ctypes.data), ctypes.c_void_p(ptr), ctypes.c_size_t(n), 2)
    assert rc == 0
    return out


@pytest.mark.parametrize("qtypes", [("Q4_0", "Q4_0", "Q8_0"), ("Q4_K", "Q4_K", "Q4_K")])
def test_gguf_file_to_hbm_to_forward(tmp_path, qtypes):
    from artlite_b200.moe.block import MoEBlock
    H, E, F, K, layers = 1024, 32, 512, 4, 2
    p = str(tmp_path / "moe.gguf")
    write_with_gguf_py(p, E, F, H, K, layers, qtypes=qtypes, seed=7)
    g = GGUFFile(p)
    cfg = g.moe_config()
    T = 200
    b = MoEBlock(hidden=cfg["hidden"], n_experts=cfg["n_experts"], top_k=cfg["top_k"], expert_ffn=cfg["expert_ffn"],
                 n_layers=cfg["n_layers"], max_tokens=T, act_dtype="bf16", path="auto")
    lays = [g.moe_layer(L) for L in range(cfg["n_layers"])]
    for L, lay in enumerate(lays):
        assert all(np.shares_memory(t.raw, g.data) for t in lay.values())  # (views of the map, no host copy)
        b.set_weights(L, gate=lay["gate"].raw, up=lay["up"].raw, down=lay["down"].raw, router=lay["router"].raw,
                      qtype=lay["gate"].qtype, down_qtype=lay["down"].qtype, router_qtype=lay["router"].qtype)
    for L, lay in enumerate(lays):
        for which in ("gate", "up", "down", "router"):
            ptr, n = b.weights(L, which)
            want = lay[which].raw.reshape(-1)
            assert n == want.size and np.array_equal(device_bytes(ptr, n), want), (L, which)

    rng = np.random.default_rng(3)
    for T_run, want_path in ((T, "tc"), (6, "gemv")):
        x = moe_np.to_bf16_bits(rng.standard_normal((T_run, H)).astype(np.float32))
        for L, lay in enumerate(lays):
            y = moe_np.bf16_to_f32(b.forward(x, layer=L))
            assert b.path(L) == want_path
            dbg = b.debug(T_run)
            ids, w = orc().route(dbg["logits"], K)
            assert np.array_equal(ids, dbg["ids"])
            qg, qd = lay["gate"].qtype, lay["down"].qtype

            def expert(e, lay=lay, qg=qg, qd=qd):
                return (orc().dequant_rows(qg, lay["gate"].raw[e * F:(e + 1) * F], H),
                        orc().dequant_rows(qg, lay["up"].raw[e * F:(e + 1) * F], H),
                        orc().dequant_rows(qd, lay["down"].raw[e * H:(e + 1) * H], F))

            want = moe_np.moe_ffn(x_f32(x), ids, w, expert)
            assert moe_np.rel_max(y, want) <= 1e-2, (T_run, L)
    b.close()
