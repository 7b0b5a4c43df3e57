"""Writes the golden vectors of tests/golden/ from the REFERENCE itself (run in a container that holds the reference
tree; the vectors are committed, so the tests need neither the reference nor this script):

- the reference's NumPy oracle ``tests/moe/ref.py`` (``moe_route``, ``moe_ffn``) imported from its tree;
- the reference's compiled host code ``csrc/artlite/moe_host.cpp`` / ``dequant.cpp`` (``oracle/_ref``, built by
  ``make -C oracle ref``): routing ids / weights, the plan, row dequant;
- gguf-py (``gguf.quants.dequantize``, the reference's pinned ``gguf>=0.19.0``, pyproject.toml:23) as an independent
  dequant of the same blocks;
- the reference's ``tests/np_ops.py`` ``rms_norm`` (the block's optional input norm).

Inputs follow the reference's own seeded fixtures (``tests/moe/test_plan.py:18-57``, ``tests/moe/test_route.py:16-26``)
with the benchmark's E=128 added, and the seeded synthetic blocks of ``oracle.moe_np``.

    python tests/golden/make_golden.py [--ref <the reference's source tree>]
"""

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import lib as olib  # noqa: E402
from oracle import moe_np  # noqa: E402


def route_cases() -> dict[str, np.ndarray]:
    """Logits of the reference's routing fixtures: test_plan.py:21-26 (ties, all-tied, -0/+0) at E=256 and E=128."""
    out = {}
    for E, T in ((256, 256), (128, 256)):
        rng = np.random.default_rng(0)
        lg = rng.standard_normal((T, E)).astype(np.float32) * 2
        lg[0, [3, 9, E - 56]] = lg[0].max() + 1  # (a three-way tie at the top)
        lg[1, :] = 0.5  # (all tied: the lowest ids)
        lg[2, :8], lg[2, 8:] = -0.0, -1  # (-0 and +0 tie)
        lg[2, 5] = 0.0
        out[f"E{E}"] = lg
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=olib.reference_tree(), help="the reference checkout (default: ARTLITE_REF, "
                    "else reference/ beside this repository)")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    from tests.moe import ref  # the reference's NumPy oracle  # noqa: E402
    import gguf.quants  # noqa: E402

    rl = olib.reference()
    assert rl is not None, "build oracle/_ref first: make -C oracle ref"
    g: dict[str, np.ndarray] = {}

    # --- routing: the reference's NumPy oracle and its compiled moe_route (softmax k = 8, sigmoid k = 6, k = 4)
    for name, lg in route_cases().items():
        g[f"route_{name}_logits"] = lg
        ids, w = ref.moe_route(lg, 8)
        g[f"route_{name}_ref_ids"], g[f"route_{name}_ref_w"] = ids.astype(np.int32), w
        ids, w = rl.route(lg, 8)
        g[f"route_{name}_cpp_ids"], g[f"route_{name}_cpp_w"] = ids, w
        ids, w = rl.route(lg, 6, gating="sigmoid")
        g[f"route_{name}_cpp_sig6_ids"], g[f"route_{name}_cpp_sig6_w"] = ids, w
        ids, w = ref.moe_route(lg, 6, gating="sigmoid")
        g[f"route_{name}_ref_sig6_ids"], g[f"route_{name}_ref_sig6_w"] = ids.astype(np.int32), w
        ids, w = rl.route(lg, 4)
        g[f"route_{name}_cpp_k4_ids"], g[f"route_{name}_cpp_k4_w"] = ids, w
    # the router GEMM's layout (test_plan.py:28-30): per column 32 experts at a pitch of 64, NaN padding
    lg = g["route_E256_logits"]
    rows = np.full((lg.shape[0], 8, 64), np.nan, np.float32)
    rows[:, :, :32] = lg.reshape(lg.shape[0], 8, 32)
    ids, w = rl.route(rows.reshape(lg.shape[0], -1), 8, E=256, per_col=32, pitch=64)
    g["route_pitch_ids"], g["route_pitch_w"] = ids, w

    # --- plan: test_plan.py:36-46 (logits + linspace(0, 3, E) bias, seed T), chunk 192, 8 columns
    for T, E in ((24, 256), (300, 256), (200, 128)):
        rng = np.random.default_rng(T)
        lg = rng.standard_normal((T, E)).astype(np.float32) + np.linspace(0, 3, E, dtype=np.float32)
        ids, _ = rl.route(lg, 8)
        cap = -(-(E + -(-T * 8 // 192)) // 8)
        ex, counts, sizes, rws, pos = rl.plan(ids, E=E, cap=cap)
        p = f"plan_T{T}_E{E}"
        g[p + "_ids"], g[p + "_cap"] = ids, np.array([cap], np.int32)
        g[p + "_experts"], g[p + "_counts"], g[p + "_sizes"], g[p + "_rows"], g[p + "_pos"] = ex, counts, sizes, rws, pos

    # --- dequant: random blocks (bytes uniform, fp16 scales N(0, 0.01) as tests/tensors.py:30-35), 8 rows of 512
    qt = {"Q4_0": gguf.GGMLQuantizationType.Q4_0, "Q4_1": gguf.GGMLQuantizationType.Q4_1,
          "Q8_0": gguf.GGMLQuantizationType.Q8_0, "Q4_K": gguf.GGMLQuantizationType.Q4_K,
          "Q5_K": gguf.GGMLQuantizationType.Q5_K, "Q6_K": gguf.GGMLQuantizationType.Q6_K,
          "Q3_K": gguf.GGMLQuantizationType.Q3_K, "IQ4_NL": gguf.GGMLQuantizationType.IQ4_NL,
          "IQ4_XS": gguf.GGMLQuantizationType.IQ4_XS}
    f16_at = {"Q4_0": (0,), "Q4_1": (0, 2), "Q8_0": (0,), "Q4_K": (0, 2), "Q5_K": (0, 2), "Q6_K": (208,),
              "Q3_K": (108,), "IQ4_NL": (0,), "IQ4_XS": (0,)}
    for i, (name, t) in enumerate(qt.items()):
        per, nb = moe_np.BLOCKS[name]
        rows, cols = 8, 512
        rng = np.random.default_rng(100 + i)
        raw = rng.integers(0, 256, (rows, cols // per, nb), dtype=np.uint8)
        for o in f16_at[name]:
            d = (rng.standard_normal((rows, cols // per)) * 0.01).astype(np.float16)
            raw[..., o:o + 2] = d.view(np.uint8).reshape(rows, cols // per, 2)
        raw = raw.reshape(rows, -1)
        g[f"dq_{name}_raw"] = raw
        g[f"dq_{name}_cpp"] = rl.dequant_rows(name, raw, cols)
        g[f"dq_{name}_ggufpy"] = np.asarray(gguf.quants.dequantize(raw, t), np.float32).reshape(rows, cols)

    # --- the block (config 1: T=16, H=2048, E=128, K=8, F=768, Q4_0, fp32 x, seed 0): the reference's moe_route and
    # moe_ffn with the experts dequantized by gguf-py (independent of this repository's dequant)
    layer, x, _ = moe_np.make_block(0, 16, qtype="Q4_0", x_bf16=False)
    logits = x @ layer.router.T
    ids, w = ref.moe_route(logits, 8)

    def expert(e: int):
        F, H = layer.F, layer.H
        dq = lambda raw: np.asarray(gguf.quants.dequantize(raw, gguf.GGMLQuantizationType.Q4_0), np.float32)
        return dq(layer.gate[e * F:(e + 1) * F]), dq(layer.up[e * F:(e + 1) * F]), dq(layer.down[e * H:(e + 1) * H])

    y = ref.moe_ffn(x, ids, w, expert)
    g["block_c1_logits"], g["block_c1_ids"], g["block_c1_w"], g["block_c1_y"] = logits, ids.astype(np.int32), w, y
    h = hashlib.sha256()
    for arr in (layer.router, x, layer.gate, layer.up, layer.down):
        h.update(np.ascontiguousarray(arr).tobytes())
    g["block_c1_sha256"] = np.frombuffer(h.digest(), np.uint8)

    # --- the block's input norm: the reference's np_ops.rms_norm (tests/np_ops.py:27-32) on seeded rows
    from tests import np_ops  # noqa: E402
    rng = np.random.default_rng(11)
    g["norm_x"] = (3 * rng.standard_normal((16, 2048))).astype(np.float32)
    g["norm_w"] = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    g["norm_y"] = np_ops.rms_norm(g["norm_x"], g["norm_w"], 1e-6)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **g)
    print("wrote", os.path.join(HERE, "golden.npz"), len(g), "arrays")


if __name__ == "__main__":
    main()
