"""The GGUF reader (artlite_b200.gguf, after src/artlite/gguf_model.py:396-506) on a synthetic MoE file written by its
writer: metadata, the MoE configuration keys (model_config.py:853-898), zero-copy raw tensor views equal to the bytes
written, tensor data alignment. CPU only."""

import numpy as np

from artlite_b200.gguf import GGUFFile, write_gguf
from oracle import moe_np


def test_roundtrip(tmp_path):
    rng = np.random.default_rng(0)
    H, E, F, K = 256, 8, 256, 2
    tensors = []
    for L in range(2):
        tensors += [(f"blk.{L}.ffn_gate_exps.weight", "Q4_0", (H, F, E), moe_np.random_blocks(rng, "Q4_0", E * F, H)),
                    (f"blk.{L}.ffn_up_exps.weight", "Q4_0", (H, F, E), moe_np.random_blocks(rng, "Q4_0", E * F, H)),
                    (f"blk.{L}.ffn_down_exps.weight", "Q8_0", (F, H, E), moe_np.random_blocks(rng, "Q8_0", E * H, F)),
                    (f"blk.{L}.ffn_gate_inp.weight", "F32", (H, E), rng.standard_normal((E, H)).astype(np.float32))]
    meta = {"general.architecture": "qwen3moe", "general.alignment": 64, "qwen3moe.block_count": 2,
            "qwen3moe.embedding_length": H, "qwen3moe.expert_count": E, "qwen3moe.expert_used_count": K,
            "qwen3moe.expert_feed_forward_length": F}
    p = str(tmp_path / "moe.gguf")
    write_gguf(p, meta, tensors, alignment=64)
    g = GGUFFile(p)
    assert g.arch == "qwen3moe"
    assert g.moe_config() == {"hidden": H, "n_experts": E, "top_k": K, "expert_ffn": F, "n_layers": 2}
    for name, qtype, dims, raw in tensors:
        t = g.tensor(name)
        assert t.qtype == qtype and t.cols == dims[0]
        assert np.array_equal(t.raw.reshape(-1), np.ascontiguousarray(raw).view(np.uint8).reshape(-1))
        assert g.tensor_info[name][2] % 64 == 0
    lay = g.moe_layer(1)
    assert lay["gate"].rows == E * F and lay["down"].qtype == "Q8_0" and lay["router"].rows == E
