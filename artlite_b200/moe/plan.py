"""The routing and the plan of an MoE layer, with the signatures of the reference's ``artlite.moe.plan``
(src/artlite/moe/plan.py:25-57): ``route`` and ``Plan.of``, computed by the CUDA kernels of
``libartlite_moe_cuda.so`` (``artlite_moe_route`` / ``artlite_moe_plan``) instead of the host C++ (``_native``).

``route``: per token the k largest logits (ties to the lower id, -0 == +0), weights e^(l - l_max) over the k in
double, normalised in numpy's pairwise order (or sigmoid(l) over their sum, at least 2^-14), fp32.
``Plan``: the (token, slot) pairs of each expert in token order, in chunks of at most ``CHUNK``, dealt to ``COLS``
columns in turn; ``pos[t, i]`` the row (c cap + k) CHUNK + j of each pair."""

from dataclasses import dataclass

import numpy as np

from .._lib import check, lib

CHUNK = 192  # tokens of a chunk (src/artlite/moe/expert_gemm.py:75: 3 MAC rows x 64)
COLS = 8  # the reference's array columns (src/artlite/operators/design.py:18)


def route(logits: np.ndarray, k: int, *, E: int = 0, per_col: int = 0, pitch: int = 0,
          gating: str = "softmax") -> tuple[np.ndarray, np.ndarray]:
    """(ids (T, k) int32, largest first, ties to the lower id; weights (T, k) float32 summing to 1) of fp32 logits:
    (T, E), or rows of the router GEMM's layout (expert e at (e / per_col) pitch + e % per_col of its row)."""
    assert gating in ("softmax", "sigmoid"), gating
    lg = np.ascontiguousarray(logits, np.float32)
    T = lg.shape[0]
    E = E or lg.shape[1]
    ids, w = np.empty((T, k), np.int32), np.empty((T, k), np.float32)
    check(lib().artlite_moe_route(lg.ctypes.data, T, lg.shape[1], per_col or E, pitch, E, k, int(gating == "sigmoid"),
                                  ids.ctypes.data, w.ctypes.data))
    return ids, w


@dataclass
class Plan:
    """An MoE layer's chunks for T tokens' routing (``ids`` (T, k)), dealt to the columns of ``cap`` slots each:
    ``experts[c]`` the experts of column c's chunks, ``sizes[c]`` their pairs, ``rows[c]`` (n_c, CHUNK) their tokens
    (padding: the chunk's first), ``pos`` (T, k) the row (c cap CHUNK + k CHUNK + j) of each (token, slot)."""

    experts: list[np.ndarray]
    sizes: list[np.ndarray]
    rows: list[np.ndarray]
    pos: np.ndarray

    @classmethod
    def of(cls, ids: np.ndarray, *, cap: int, E: int, cols: int = COLS, chunk: int = CHUNK) -> "Plan":
        ids = np.ascontiguousarray(ids, np.int32)
        ex, counts, sizes = np.zeros((cols, cap), np.int32), np.zeros(cols, np.int32), np.zeros((cols, cap), np.int32)
        rows, pos = np.zeros((cols, cap, chunk), np.int32), np.zeros(ids.shape, np.int64)
        check(lib().artlite_moe_plan(ids.ctypes.data, ids.shape[0], ids.shape[1], E, cols, cap, chunk,
                                     ex.ctypes.data, counts.ctypes.data, sizes.ctypes.data, rows.ctypes.data,
                                     pos.ctypes.data))
        return cls(*([a[c, :counts[c]] for c in range(cols)] for a in (ex, sizes, rows)), pos)

    @property
    def counts(self) -> list[int]:
        return [len(e) for e in self.experts]


def dispatch(ids: np.ndarray, E: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The block's own dispatch (``artlite_moe_dispatch``): (offsets (E + 1,) int64, perm (T k,) int32, slot (T k,)
    int32), the pairs t k + i grouped by expert, stable in pair order."""
    ids = np.ascontiguousarray(ids, np.int32)
    off = np.zeros(E + 1, np.int64)
    perm, slot = np.zeros(ids.size, np.int32), np.zeros(ids.size, np.int32)
    check(lib().artlite_moe_dispatch(ids.ctypes.data, ids.shape[0], ids.shape[1], E, off.ctypes.data,
                                     perm.ctypes.data, slot.ctypes.data))
    return off, perm, slot


def dequant_supported(qtype: str) -> bool:
    return bool(lib().artlite_dequant_supported(qtype.encode()))


def dequant_rows(qtype: str, raw: np.ndarray, cols: int) -> np.ndarray:
    """(n, cols) fp32 of n raw GGUF rows ((n, row_bytes) uint8) on the GPU (``_native.dequant_rows``)."""
    raw = np.ascontiguousarray(raw, np.uint8)
    out = np.empty((raw.shape[0], cols), np.float32)
    check(lib().artlite_dequant_rows(qtype.encode(), raw.ctypes.data, raw.shape[0], raw.shape[1], cols,
                                     out.ctypes.data))
    return out
