"""TEST INFRASTRUCTURE ONLY: the NumPy oracle of the GGUF MoE block, restated from the reference.

- ``softmax`` / ``silu`` / ``sigmoid``: ``tests/np_ops.py:10-19,35-39`` (float32, the softmax's sum in float64).
- ``moe_route``: ``tests/moe/ref.py:11-18`` (softmax over all E, a stable argsort of -p, w / max(sum, 2^-14)).
- ``swiglu`` / ``moe_ffn`` / ``shared_expert``: ``tests/moe/ref.py:21-24,43-52,55-60`` (float32 matmuls).
- ``dequant``: ``src/artlite/gguf_model.py:50-129`` (``QTensor.fields``) and ``:278-330`` (``QTensor.dequantize``)
  for Q4_0, Q4_1, Q8_0, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_NL, IQ4_XS, F32, F16, BF16 (Q3_K :141-162,297-299; IQ4_NL
  :195-200,320-321; IQ4_XS :201-212,322-324).
- ``rel`` / ``rel_max``: ``tests/numerics.py:24-27,50-53``.
- Block generators: the synthetic GGUF blocks of the benchmark configurations (fp16 d from |N(0, 0.02)|; Q4_0 nibbles
  uniform 0..15; Q4_K 6-bit scales / mins uniform 0..63 packed as ``gguf_model.py:116-121`` reads them; Q8_0 int8
  uniform -127..127), drawn from one ``default_rng(seed)`` stream in the order router, x, gate, up, down. The other
  block formats (test cases only): Q4_1 m = -8 d; Q5_K as Q4_K with uniform high bits; Q6_K int8 scales uniform
  -32..31 with d from |N(0, 0.002)|; Q3_K d from |N(0, 0.004)|; IQ4_NL d from |N(0, 0.0005)|, IQ4_XS d from
  |N(0, 0.00005)|; all quant and scale bits uniform.
"""

from dataclasses import dataclass

import numpy as np

# (values per block, bytes per block) of the GGUF types (gguf_model.py:385-390)
BLOCKS = {"F32": (1, 4), "F16": (1, 2), "BF16": (1, 2), "Q4_0": (32, 18), "Q4_1": (32, 20), "Q8_0": (32, 34),
          "Q3_K": (256, 110), "Q4_K": (256, 144), "Q5_K": (256, 176), "Q6_K": (256, 210), "IQ4_NL": (32, 18),
          "IQ4_XS": (256, 136)}

# IQ4_NL / IQ4_XS code values (gguf_model.py's IQ4_VALUES, ggml's non-linear 4-bit grid)
IQ4_GRID = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float32)


def row_bytes(qtype: str, cols: int) -> int:
    per, nb = BLOCKS[qtype]
    assert cols % per == 0, (qtype, cols)
    return cols // per * nb


# ---------------------------------------------------------------- np_ops / moe.ref

def f32(x: object) -> np.ndarray:
    return np.asarray(x, np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x = f32(x)
    return x / (np.float32(1) + np.exp(-x))


def sigmoid(x: np.ndarray) -> np.ndarray:
    x = f32(x)
    return np.float32(1) / (np.float32(1) + np.exp(-x))


def rms_norm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    """tests/np_ops.py:27-32: x / sqrt(mean(x^2) + eps) * w over the last axis, the mean of the squares in float64,
    the quotient rounded to float32, then times w in float32."""
    x = f32(x)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    y = (x / np.sqrt(ms + eps)).astype(np.float32)
    return y if w is None else y * f32(w)


def softmax(x: np.ndarray) -> np.ndarray:
    x = f32(x)
    e = np.exp(x - x.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True, dtype=np.float64)).astype(np.float32)


def moe_route(logits: np.ndarray, k: int, gating: str = "softmax") -> tuple[np.ndarray, np.ndarray]:
    p = softmax(logits) if gating == "softmax" else sigmoid(logits)
    ids = np.argsort(-p, axis=-1, kind="stable")[:, :k]
    w = np.take_along_axis(p, ids, -1)
    return ids, (w / np.maximum(w.sum(-1, keepdims=True), np.float32(6.103515625e-5))).astype(np.float32)


def swiglu(x: np.ndarray, gate: np.ndarray, up: np.ndarray, down: np.ndarray) -> np.ndarray:
    x = f32(x)
    return (silu(x @ f32(gate).T) * (x @ f32(up).T)) @ f32(down).T


def moe_ffn(x: np.ndarray, ids: np.ndarray, weights: np.ndarray, expert, ffn=swiglu) -> np.ndarray:
    x = f32(x)
    y = np.zeros_like(x)
    for e in np.unique(ids):
        t, i = np.nonzero(ids == e)
        y[t] += f32(weights)[t, i][:, None] * ffn(x[t], *expert(int(e)))
    return y


def shared_expert(x, gate, up, down, gate_inp):
    y = swiglu(x, gate, up, down)
    return y if gate_inp is None else sigmoid(f32(x) @ f32(gate_inp).reshape(-1, 1)) * y


# ---------------------------------------------------------------- numerics

def rel(a: object, b: object) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def rel_max(a: object, b: object) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


# ---------------------------------------------------------------- dequant (QTensor.fields / dequantize)

def _f16(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b).view(np.float16)[..., 0].astype(np.float32)


def dequant(qtype: str, raw: np.ndarray, cols: int) -> np.ndarray:
    """(rows, cols) fp32 of raw GGUF rows ((rows, row_bytes) uint8, or the plain types' values)."""
    if qtype == "F32":
        return np.asarray(raw).view(np.float32).reshape(raw.shape[0], -1)[:, :cols].astype(np.float32)
    if qtype == "F16":
        return np.asarray(raw).view(np.float16).reshape(raw.shape[0], -1)[:, :cols].astype(np.float32)
    if qtype == "BF16":
        u = np.asarray(raw).view(np.uint16).reshape(raw.shape[0], -1)[:, :cols].astype(np.uint32) << 16
        return u.view(np.float32)
    per, nb = BLOCKS[qtype]
    rows = raw.shape[0]
    b = np.ascontiguousarray(raw, np.uint8)[:, :cols // per * nb].reshape(rows, -1, nb)
    if qtype in ("Q4_0", "Q4_1"):
        o = 2 if qtype == "Q4_0" else 4
        q = np.empty((rows, b.shape[1], 32), np.uint8)
        q[..., :16] = b[..., o:] & 0xF
        q[..., 16:] = b[..., o:] >> 4
        d = _f16(b[..., 0:2])
        if qtype == "Q4_0":
            w = d[..., None] * (q.astype(np.float32) - 8.0)
        else:
            w = d[..., None] * q + _f16(b[..., 2:4])[..., None]
    elif qtype == "Q8_0":
        q = np.ascontiguousarray(b[..., 2:]).view(np.int8)
        w = _f16(b[..., 0:2])[..., None] * q.astype(np.float32)
    elif qtype in ("Q4_K", "Q5_K"):
        s = b[..., 4:16]
        lo, hi, top = s[..., 0:4], s[..., 4:8], s[..., 8:12]
        sc = np.concatenate([lo & 63, (top & 0xF) | ((lo >> 6) << 4)], axis=-1)
        mn = np.concatenate([hi & 63, (top >> 4) | ((hi >> 6) << 4)], axis=-1)
        qs = b[..., 16 if qtype == "Q4_K" else 48:].reshape(rows, -1, 4, 32)
        q = np.stack([qs & 0xF, qs >> 4], axis=3)
        if qtype == "Q5_K":
            qh = b[..., 16:48]
            hb = (qh[..., None, :] >> np.arange(8, dtype=np.uint8)[:, None]) & 1
            q = q | (hb.reshape(q.shape) << 4)
        a = _f16(b[..., 0:2])[..., None] * sc
        m = _f16(b[..., 2:4])[..., None] * mn
        w = a[..., None] * q.reshape(rows, -1, 8, 32) - m[..., None]
    elif qtype == "Q6_K":
        ql = b[..., 0:128].reshape(rows, -1, 2, 64)
        qh = b[..., 128:192].reshape(rows, -1, 2, 32)
        q = np.empty((rows, b.shape[1], 2, 4, 32), np.uint8)
        q[..., 0, :] = (ql[..., :32] & 0xF) | (((qh >> 0) & 3) << 4)
        q[..., 1, :] = (ql[..., 32:] & 0xF) | (((qh >> 2) & 3) << 4)
        q[..., 2, :] = (ql[..., :32] >> 4) | (((qh >> 4) & 3) << 4)
        q[..., 3, :] = (ql[..., 32:] >> 4) | (((qh >> 6) & 3) << 4)
        sc = np.ascontiguousarray(b[..., 192:208]).view(np.int8)
        a = _f16(b[..., 208:210])[..., None] * sc.astype(np.float32)
        w = a[..., None] * (q.reshape(rows, -1, 16, 16).astype(np.float32) - 32.0)
    elif qtype == "Q3_K":
        nbk = b.shape[1]
        # value 128 n + 32 j + i: crumb j of qs[32 n + i], bit (4 n + j) of hmask[i] as bit 2
        qs = b[..., 32:96].reshape(rows, nbk, 2, 1, 32)
        j = np.arange(4, dtype=np.uint8).reshape(1, 1, 1, 4, 1)
        n = np.arange(2, dtype=np.uint8).reshape(1, 1, 2, 1, 1)
        hm = b[..., 0:32].reshape(rows, nbk, 1, 1, 32)
        q = ((qs >> (2 * j)) & 3) | (((hm >> (4 * n + j)) & 1) << 2)  # (rows, nbk, n, j, i)
        sb = b[..., 96:108]
        low = np.concatenate([sb[..., :8] & 0xF, sb[..., :8] >> 4], axis=-1)  # sub-blocks 0 .. 15
        top = (sb[..., 8:12, None] >> (2 * np.arange(4, dtype=np.uint8))) & 3  # [i, k]: sub-block 4 k + i
        sc = (low | (top.transpose(0, 1, 3, 2).reshape(rows, nbk, 16) << 4)).astype(np.float32) - 32.0
        a = _f16(b[..., 108:110])[..., None] * sc
        w = a[..., None] * (q.reshape(rows, nbk, 16, 16).astype(np.float32) - 4.0)
    elif qtype == "IQ4_NL":
        q = np.concatenate([b[..., 2:] & 0xF, b[..., 2:] >> 4], axis=-1)
        w = _f16(b[..., 0:2])[..., None] * IQ4_GRID[q]
    elif qtype == "IQ4_XS":
        nbk = b.shape[1]
        hi = (np.ascontiguousarray(b[..., 2:4]).view("<u2") >> (2 * np.arange(8, dtype=np.uint16))) & 3
        lo = np.stack([b[..., 4:8] & 0xF, b[..., 4:8] >> 4], axis=-1).reshape(rows, nbk, 8)
        ls = (lo | (hi.astype(np.uint8) << 4)).astype(np.float32)
        qs = b[..., 8:].reshape(rows, nbk, 8, 16)
        q = np.concatenate([qs & 0xF, qs >> 4], axis=-1)
        dl = _f16(b[..., 0:2])[..., None] * (ls - 32.0)
        w = dl[..., None] * IQ4_GRID[q]
    else:
        raise ValueError(qtype)
    return np.ascontiguousarray(w, dtype=np.float32).reshape(rows, cols)


# ---------------------------------------------------------------- synthetic blocks

def _fp16_abs_normal(rng: np.random.Generator, shape, scale: float = 0.02) -> np.ndarray:
    return np.abs(rng.standard_normal(shape) * scale).astype(np.float16)


def random_blocks(rng: np.random.Generator, qtype: str, rows: int, cols: int) -> np.ndarray:
    """(rows, row_bytes) uint8 of synthetic GGUF blocks of ``qtype`` (the module docstring's distributions)."""
    per, nb = BLOCKS[qtype]
    n = cols // per
    raw = np.empty((rows, n, nb), np.uint8)
    if qtype == "Q4_0":
        raw[..., 0:2] = _fp16_abs_normal(rng, (rows, n)).view(np.uint8).reshape(rows, n, 2)
        raw[..., 2:] = rng.integers(0, 256, (rows, n, 16), dtype=np.uint8)
    elif qtype == "Q8_0":
        raw[..., 0:2] = _fp16_abs_normal(rng, (rows, n)).view(np.uint8).reshape(rows, n, 2)
        raw[..., 2:] = rng.integers(-127, 128, (rows, n, 32), dtype=np.int8).view(np.uint8)
    elif qtype == "Q4_K":
        raw[..., 0:2] = _fp16_abs_normal(rng, (rows, n)).view(np.uint8).reshape(rows, n, 2)
        raw[..., 2:4] = _fp16_abs_normal(rng, (rows, n)).view(np.uint8).reshape(rows, n, 2)
        sc = rng.integers(0, 64, (rows, n, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, (rows, n, 8), dtype=np.uint8)
        raw[..., 4:8] = (sc[..., :4] & 63) | ((sc[..., 4:] >> 4) << 6)
        raw[..., 8:12] = (mn[..., :4] & 63) | ((mn[..., 4:] >> 4) << 6)
        raw[..., 12:16] = (sc[..., 4:] & 15) | ((mn[..., 4:] & 15) << 4)
        raw[..., 16:] = rng.integers(0, 256, (rows, n, 128), dtype=np.uint8)
    elif qtype == "Q4_1":
        d = _fp16_abs_normal(rng, (rows, n))
        raw[..., 0:2] = d.view(np.uint8).reshape(rows, n, 2)
        raw[..., 2:4] = (-8 * d).astype(np.float16).view(np.uint8).reshape(rows, n, 2)
        raw[..., 4:] = rng.integers(0, 256, (rows, n, 16), dtype=np.uint8)
    elif qtype == "Q5_K":
        raw[..., :144] = random_blocks(rng, "Q4_K", rows * n, 256).reshape(rows, n, 144)
        raw[..., 144:] = rng.integers(0, 256, (rows, n, 32), dtype=np.uint8)
        raw[..., 16:] = np.concatenate([raw[..., 144:], raw[..., 16:144]], axis=-1)  # d, dmin, scales, qh, qs
    elif qtype == "Q6_K":
        raw[..., :192] = rng.integers(0, 256, (rows, n, 192), dtype=np.uint8)
        raw[..., 192:208] = rng.integers(-32, 32, (rows, n, 16), dtype=np.int8).view(np.uint8)
        raw[..., 208:] = _fp16_abs_normal(rng, (rows, n), 0.002).view(np.uint8).reshape(rows, n, 2)
    elif qtype == "Q3_K":
        raw[..., :108] = rng.integers(0, 256, (rows, n, 108), dtype=np.uint8)
        raw[..., 108:] = _fp16_abs_normal(rng, (rows, n), 0.004).view(np.uint8).reshape(rows, n, 2)
    elif qtype in ("IQ4_NL", "IQ4_XS"):
        scale = 0.0005 if qtype == "IQ4_NL" else 0.00005
        raw[..., 0:2] = _fp16_abs_normal(rng, (rows, n), scale).view(np.uint8).reshape(rows, n, 2)
        raw[..., 2:] = rng.integers(0, 256, (rows, n, nb - 2), dtype=np.uint8)
    else:
        raise ValueError(qtype)
    return raw.reshape(rows, n * nb)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), rounded to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class Layer:
    """One synthetic MoE layer: raw GGUF blocks of the expert tensors as the GGUF stores them (gate / up: (E F,
    row_bytes(H)); down: (E H, row_bytes(F))) and the router (E, H) fp32."""

    qtype: str
    H: int
    E: int
    F: int
    router: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    down_qtype: str = ""  # (the down tensor's own type, as mixed files have it; "": qtype)

    @property
    def dqtype(self) -> str:
        return self.down_qtype or self.qtype

    def expert(self, e: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(gate (F, H), up (F, H), down (H, F)) fp32 of expert e (``tests/moe/ref.py:27-40``'s row ranges)."""
        F, H = self.F, self.H
        return (dequant(self.qtype, self.gate[e * F:(e + 1) * F], H),
                dequant(self.qtype, self.up[e * F:(e + 1) * F], H),
                dequant(self.dqtype, self.down[e * H:(e + 1) * H], F))


def make_block(seed: int, T: int, *, H: int = 2048, E: int = 128, F: int = 768, qtype: str = "Q4_0",
               x_bf16: bool = True, zipf: float = 0.0, down_qtype: str = "") -> tuple[Layer, np.ndarray, np.ndarray]:
    """(layer, x (T, H): bf16 bits if ``x_bf16`` else fp32, router bias (E,) fp32) from one seeded stream: router,
    x, gate, up, down; ``zipf`` s > 0 adds bias_e = -s ln(r_e), r a seeded permutation of 1..E (drawn last);
    ``down_qtype`` the down tensor's own type (default: qtype)."""
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    gate = random_blocks(rng, qtype, E * F, H)
    up = random_blocks(rng, qtype, E * F, H)
    down = random_blocks(rng, down_qtype or qtype, E * H, F)
    bias = np.zeros(E, np.float32)
    if zipf:
        r = rng.permutation(E) + 1
        bias = (-zipf * np.log(r)).astype(np.float32)
    return Layer(qtype, H, E, F, router, gate, up, down, down_qtype), (to_bf16_bits(x) if x_bf16 else x), bias
