"""Helpers of the block tests: synthetic layers (oracle.moe_np), the oracle's y for the GPU's own routing."""

import numpy as np

from oracle import lib as olib
from oracle import moe_np

_ORC = None


def orc():
    global _ORC
    if _ORC is None:
        _ORC = olib.oracle()
    return _ORC


def expert_fn(layer: moe_np.Layer):
    """expert(e) -> fp32 (gate, up, down) by the C oracle's dequant (bit-identical to the reference's)."""
    o = orc()
    F, H = layer.F, layer.H

    def get(e: int):
        return (o.dequant_rows(layer.qtype, layer.gate[e * F:(e + 1) * F], H),
                o.dequant_rows(layer.qtype, layer.up[e * F:(e + 1) * F], H),
                o.dequant_rows(layer.dqtype, layer.down[e * H:(e + 1) * H], F))
    return get


def x_f32(x: np.ndarray) -> np.ndarray:
    return moe_np.bf16_to_f32(x) if x.dtype == np.uint16 else np.asarray(x, np.float32)


def oracle_y(layer: moe_np.Layer, x: np.ndarray, ids: np.ndarray, w: np.ndarray, tokens=None) -> np.ndarray:
    """ref.moe_ffn's y (fp32) of the tokens (all, or the given subset) under the routing (ids, w)."""
    xf = x_f32(x)
    if tokens is not None:
        xf, ids, w = xf[tokens], ids[tokens], w[tokens]
    return moe_np.moe_ffn(xf, ids, w, expert_fn(layer))


def make_block(layer: moe_np.Layer, T: int, *, act: str, path: str, gating: str = "softmax", n_layers: int = 1,
               top_k: int = 8):
    from artlite_b200.moe.block import MoEBlock
    b = MoEBlock(hidden=layer.H, n_experts=layer.E, top_k=top_k, expert_ffn=layer.F, max_tokens=T, act_dtype=act,
                 path=path, gating=gating, n_layers=n_layers)
    for L in range(n_layers):
        b.set_weights(L, gate=layer.gate, up=layer.up, down=layer.down, router=layer.router, qtype=layer.qtype,
                      down_qtype=layer.dqtype)
    return b


def torch_moe_ffn(layer: moe_np.Layer, x: np.ndarray, ids: np.ndarray, w: np.ndarray, device: int = 0) -> np.ndarray:
    """ref.moe_ffn (tests/moe/ref.py:43-52) as a plain PyTorch fp32 computation on the GPU, for every token of a
    full-size batch: each expert's weights dequantised exactly on the CPU by the C oracle (bit-identical to the
    reference's dequant_rows), its rows' SwiGLU in fp32 (no TF32), the weighted rows added into y in expert order.
    It differs from the NumPy oracle only in the fp32 summation order (tests pin the two against each other)."""
    import torch
    prev = torch.backends.cuda.matmul.fp32_precision
    torch.backends.cuda.matmul.fp32_precision = "ieee"
    try:
        dev = torch.device("cuda", device)
        xf = torch.from_numpy(x_f32(x)).to(dev)
        y = torch.zeros_like(xf)
        get = expert_fn(layer)
        ids_t = torch.from_numpy(np.ascontiguousarray(ids, np.int64)).to(dev)
        w_t = torch.from_numpy(np.ascontiguousarray(w, np.float32)).to(dev)
        for e in np.unique(ids):
            t, i = torch.nonzero(ids_t == int(e), as_tuple=True)
            g, u, d = (torch.from_numpy(a).to(dev) for a in get(int(e)))
            xe = xf[t]
            h = torch.nn.functional.silu(xe @ g.T) * (xe @ u.T)
            y.index_add_(0, t, w_t[t, i][:, None] * (h @ d.T))
        out = y.cpu().numpy()
    finally:
        torch.backends.cuda.matmul.fp32_precision = prev
    return out
