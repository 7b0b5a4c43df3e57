"""The whole GGUF MoE block on the GPU: router logits, routing, dispatch, SwiGLU experts read from the raw GGUF blocks,
the weighted combine (``artlite_moe_create`` / ``set_weights`` / ``forward``, include/artlite_moe.h).

The block the reference composes from ``MoEPrefill.items`` with its host steps (src/artlite/moe/prefill.py:102-195)
and defines in its oracle (``ref.moe_route`` + ``ref.moe_ffn``, tests/moe/ref.py:11-52), as one object. Host side:
NumPy + ctypes; activations are fp32 or bf16 (NumPy uint16 bit patterns); the GGUF tensors are passed as their raw
bytes (``GGUFFile.tensor(name).raw`` views, or ``artlite_b200.gguf``'s) and copied to HBM verbatim."""

import ctypes

import numpy as np

from .._lib import QTYPES, Error, MoeDesc, check, lib

PATHS = {"auto": 0, "gemv": 1, "tc": 2}


def ep_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes) for ``MoEBlock.ep_init``."""
    buf = ctypes.create_string_buffer(128)
    check(lib().artlite_moe_ep_unique_id(buf, 128))
    return buf.raw


def ep_plan(send_counts: np.ndarray, recv_counts: np.ndarray, world: int, rank: int, E: int):
    """The exchange plan of one rank (``artlite_moe_ep_plan``, host only): (send_off (E,), recv_pos (world, E / world),
    local_off (E / world + 1,), local_counts (E / world,))."""
    El = E // world
    sc = np.ascontiguousarray(send_counts, np.int32)
    rc = np.ascontiguousarray(recv_counts, np.int32).reshape(world * El)
    send_off, recv_pos = np.zeros(E, np.int64), np.zeros((world, El), np.int64)
    local_off, local_counts = np.zeros(El + 1, np.int64), np.zeros(El, np.int32)
    check(lib().artlite_moe_ep_plan(sc.ctypes.data, rc.ctypes.data, world, rank, E, send_off.ctypes.data,
                                    recv_pos.ctypes.data, local_off.ctypes.data, local_counts.ctypes.data))
    return send_off, recv_pos, local_off, local_counts


def _ptr(a) -> int | None:
    """A host array's address, or a device address given as an int / an object with ``data_ptr()`` (None: NULL)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return int(a.data_ptr())
    raise TypeError(type(a))


class MoEBlock:
    """``n_layers`` MoE blocks of one shape (a stack, each with its own weights) on one CUDA device.

    ``act_dtype``: "f32" (x / y float32) or "bf16" (x / y uint16 bf16 bits); ``path``: "auto" (tcgen05 grouped GEMMs
    for prefill-sized batches, the dequant-GEMVs for decode batches), "gemv" or "tc"."""

    def __init__(self, *, hidden: int, n_experts: int, top_k: int, expert_ffn: int, max_tokens: int,
                 n_layers: int = 1, gating: str = "softmax", act_dtype: str = "bf16", device: int = -1,
                 path: str = "auto", ep_rank: int = 0, ep_world: int = 1):
        assert gating in ("softmax", "sigmoid") and act_dtype in ("f32", "bf16") and path in PATHS
        self.H, self.E, self.K, self.F = hidden, n_experts, top_k, expert_ffn
        self.act = act_dtype
        self.max_tokens = max_tokens
        d = MoeDesc(hidden=hidden, n_experts=n_experts, top_k=top_k, expert_ffn=expert_ffn, n_layers=n_layers,
                    gating=int(gating == "sigmoid"), act_dtype=QTYPES["BF16" if act_dtype == "bf16" else "F32"],
                    max_tokens=max_tokens, device=device, path=PATHS[path], ep_rank=ep_rank, ep_world=ep_world)
        h = ctypes.c_void_p()
        check(lib().artlite_moe_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h

    def ep_init(self, unique_id: bytes) -> None:
        """Joins this rank's block to the NCCL communicator of ``unique_id`` (from ``ep_unique_id`` on one rank,
        shared with the others by the caller): collective over the ``ep_world`` ranks."""
        buf = ctypes.create_string_buffer(bytes(unique_id), len(unique_id))
        check(lib().artlite_moe_ep_init(self._h, buf, len(unique_id)))

    @property
    def np_dtype(self):
        return np.uint16 if self.act == "bf16" else np.float32

    def set_weights(self, layer: int, *, gate, up, down, router, qtype: str, down_qtype: str | None = None,
                    router_qtype: str = "F32") -> None:
        """Layer ``layer``'s raw GGUF tensors (blk.L.ffn_gate_exps / ffn_up_exps / ffn_down_exps / ffn_gate_inp)."""
        keep = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a for a in (gate, up, down, router)]
        check(lib().artlite_moe_set_weights(self._h, layer, QTYPES[qtype], _ptr(keep[0]), _ptr(keep[1]),
                                            QTYPES[down_qtype or qtype], _ptr(keep[2]), _ptr(keep[3]),
                                            QTYPES[router_qtype]))

    def set_shared(self, layer: int, *, gate, up, down, ffn: int, qtype: str, down_qtype: str | None = None,
                   gate_inp=None, gate_dtype: str = "F32") -> None:
        """Layer ``layer``'s shared expert (ref.shared_expert): raw GGUF rows gate / up (ffn x hidden), down (hidden x
        ffn) (blk.L.ffn_{gate,up,down}_shexp), and the optional gate vector (blk.L.ffn_gate_inp_shexp, hidden values of
        ``gate_dtype``); numpy arrays or device pointers. ``gate=None`` removes it."""
        keep = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a for a in (gate, up, down, gate_inp)]
        check(lib().artlite_moe_set_shared(self._h, layer, ffn, QTYPES[qtype], _ptr(keep[0]), _ptr(keep[1]),
                                            QTYPES[down_qtype or qtype], _ptr(keep[2]), _ptr(keep[3]),
                                            QTYPES[gate_dtype]))

    def set_norm(self, layer: int, w, *, eps: float = 1e-6, dtype: str = "F32") -> None:
        """RMSNorm of layer ``layer``'s input before the router and the experts (np_ops.rms_norm: the mean of the
        squares in float64), and the input added back to the output as the residual: y = x + moe(rms_norm(x, w, eps)).
        ``w``: hidden values of ``dtype`` (F32 or BF16), a numpy array or a device pointer; None removes it."""
        keep = np.ascontiguousarray(w) if isinstance(w, np.ndarray) else w
        check(lib().artlite_moe_set_norm(self._h, layer, _ptr(keep), QTYPES[dtype], float(eps)))

    def set_router_bias(self, layer: int, bias: np.ndarray | None) -> None:
        """A per-expert bias added to the router logits (None: none)."""
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        check(lib().artlite_moe_set_router_bias(self._h, layer, None if b is None else b.ctypes.data))

    def forward(self, x: np.ndarray, layer: int = 0, out: np.ndarray | None = None) -> np.ndarray:
        """y (T, H) of x (T, H) (host arrays: the call returns when y is back)."""
        x = np.ascontiguousarray(x, self.np_dtype)
        T = x.shape[0]
        if x.shape[1] != self.H:
            raise Error(f"moe_forward: x has {x.shape[1]} columns, H is {self.H}")
        y = out if out is not None else np.empty((T, self.H), self.np_dtype)
        check(lib().artlite_moe_forward(self._h, layer, x.ctypes.data, y.ctypes.data, T, None))
        return y

    def forward_ptr(self, x, y, T: int, layer: int = 0, stream: int = 0) -> None:
        """The forward on device (or pinned host) buffers given by address; enqueued on ``stream`` (0: the block's)."""
        check(lib().artlite_moe_forward(self._h, layer, _ptr(x), _ptr(y), T, ctypes.c_void_p(stream or None)))

    def forward_graph(self, x, y, T: int, layer: int = 0, stream: int = 0) -> None:
        """``forward_ptr`` as a CUDA graph, captured on the first call per (layer, T, x, y) and replayed after."""
        check(lib().artlite_moe_forward_graph(self._h, layer, _ptr(x), _ptr(y), T, ctypes.c_void_p(stream or None)))

    def sync(self, timeout_ms: int = 0) -> None:
        check(lib().artlite_moe_sync(self._h, timeout_ms))

    def debug(self, T: int) -> dict[str, np.ndarray]:
        """The last forward's logits, routing and dispatch (T: its tokens)."""
        out = {"logits": np.empty((T, self.E), np.float32), "ids": np.empty((T, self.K), np.int32),
               "w": np.empty((T, self.K), np.float32), "offsets": np.empty(self.E + 1, np.int64),
               "perm": np.empty(T * self.K, np.int32)}
        check(lib().artlite_moe_debug(self._h, *(out[k].ctypes.data for k in ("logits", "ids", "w", "offsets",
                                                                              "perm"))))
        return out

    def stage_times(self, layer: int = 0) -> list[float]:
        """Layer ``layer``'s per-stage device times (ms) of its last forward (ARTLITE_MOE_TIMING=1 at creation)."""
        ms = (ctypes.c_float * 16)()
        n = ctypes.c_int()
        check(lib().artlite_moe_stage_times(self._h, layer, ms, ctypes.byref(n)))
        return list(ms[:n.value])

    def weights(self, layer: int, which: str) -> tuple[int, int]:
        """(device address, bytes) of layer ``layer``'s tensor ``which`` ("gate", "up", "down", "router") as it sits
        in HBM: the GGUF bytes set_weights copied, unconverted (this rank's experts' rows)."""
        ptr, n = ctypes.c_void_p(), ctypes.c_int64()
        check(lib().artlite_moe_weights(self._h, layer, ("gate", "up", "down", "router").index(which),
                                        ctypes.byref(ptr), ctypes.byref(n)))
        return ptr.value, n.value

    def path(self, layer: int = 0) -> str:
        return {0: "none", 1: "gemv", 2: "tc"}[lib().artlite_moe_path(self._h, layer)]

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().artlite_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
