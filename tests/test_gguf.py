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


def write_with_gguf_py(path, E, F, H, K, layers, qtypes=("Q4_0", "Q4_0", "Q8_0"), seed=0):
    """A qwen3moe file written by gguf-py's own GGUFWriter (the reference's pinned dependency, gguf>=0.19.0,
    pyproject.toml:23), not by this repository's writer: (path, {name: raw bytes (rows, row_bytes)})."""
    import gguf
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(path, "qwen3moe")
    w.add_block_count(layers)
    w.add_embedding_length(H)
    w.add_expert_count(E)
    w.add_expert_used_count(K)
    w.add_expert_feed_forward_length(F)
    raws = {}
    for L in range(layers):
        for (n, rows, cols, qt, shape) in ((f"blk.{L}.ffn_gate_exps.weight", E * F, H, qtypes[0], (E, F)),
                                           (f"blk.{L}.ffn_up_exps.weight", E * F, H, qtypes[1], (E, F)),
                                           (f"blk.{L}.ffn_down_exps.weight", E * H, F, qtypes[2], (E, H))):
            raw = moe_np.random_blocks(rng, qt, rows, cols)
            w.add_tensor(n, raw.reshape(*shape, -1), raw_dtype=gguf.GGMLQuantizationType[qt])
            raws[n] = raw
        r = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
        w.add_tensor(f"blk.{L}.ffn_gate_inp.weight", r)
        raws[f"blk.{L}.ffn_gate_inp.weight"] = r
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return raws


def test_reads_gguf_py_file(tmp_path):
    """A file written by an independent writer (gguf-py's GGUFWriter): the MoE configuration, every tensor's dims,
    type and raw bytes as zero-copy views of the map, and the data offsets gguf-py's own GGUFReader finds."""
    import gguf
    H, E, F, K = 512, 8, 256, 2
    p = str(tmp_path / "gguf_py.gguf")
    raws = write_with_gguf_py(p, E, F, H, K, 2, qtypes=("Q4_K", "Q4_K", "Q6_K"))
    g = GGUFFile(p)
    assert g.moe_config() == {"hidden": H, "n_experts": E, "top_k": K, "expert_ffn": F, "n_layers": 2}
    rd = gguf.GGUFReader(p)
    offs = {t.name: int(t.data_offset) for t in rd.tensors}
    for name, raw in raws.items():
        t = g.tensor(name)
        assert np.shares_memory(t.raw, g.data)  # (a view of the map, not a copy)
        assert np.array_equal(t.raw.reshape(-1), np.ascontiguousarray(raw).view(np.uint8).reshape(-1))
        assert g.tensor_info[name][2] == offs[name]
    lay = g.moe_layer(1)
    assert (lay["gate"].qtype, lay["down"].qtype, lay["router"].qtype) == ("Q4_K", "Q6_K", "F32")
    assert lay["gate"].cols == H and lay["down"].cols == F and lay["gate"].rows == E * F
