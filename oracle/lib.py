"""TEST INFRASTRUCTURE ONLY: ctypes bindings of the C oracle (``liboracle.so``) and, when it was built, of the
reference's own compiled host code (``_ref/libartlite_ref.so``, see ``oracle/Makefile``).

Both expose the same three operations with the reference's argument meaning (``csrc/artlite/moe_host.h:13-22``,
``csrc/artlite/dequant.h:16``): ``route``, ``plan``, ``dequant_rows``; ``dispatch`` (C oracle only) is the
expert-contiguous permutation the CUDA path builds (the first half of ``moe_plan``)."""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libartlite_ref.so")

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int


class OracleError(RuntimeError):
    pass


def reference_tree() -> str:
    """The reference checkout: ``ARTLITE_REF``, else ``reference/`` beside this repository's root."""
    return os.environ.get("ARTLITE_REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def build() -> None:
    """Compile the C oracle (and the reference's host code when its tree is present) with ``oracle/Makefile``."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    ref = reference_tree()
    if os.path.isdir(os.path.join(ref, "csrc", "artlite")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + ref], check=True)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.path = path
        self.lib = ctypes.CDLL(path)
        self.prefix = prefix
        f = self._f
        f("moe_route").argtypes = [_P, _I64, _I64, _I, _I64, _I, _I, _I, _P, _P]
        f("moe_plan").argtypes = [_P, _I64, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P]
        f("dequant_rows").argtypes = [ctypes.c_char_p, _P, _I64, _I64, _I64, _P]
        for n in ("moe_route", "moe_plan", "dequant_rows"):
            f(n).restype = _I

    def _f(self, name: str):
        return getattr(self.lib, self.prefix + name)

    def _check(self, rc: int, what: str) -> None:
        if rc:
            msg = what
            if hasattr(self.lib, "artlite_ref_last_error"):
                self.lib.artlite_ref_last_error.restype = ctypes.c_char_p
                msg = self.lib.artlite_ref_last_error().decode()
            raise OracleError(f"{msg} (status {rc})")

    def route(self, logits: np.ndarray, k: int, *, E: int = 0, per_col: int = 0, pitch: int = 0,
              gating: str = "softmax") -> tuple[np.ndarray, np.ndarray]:
        """``moe_route`` on (T, row) fp32 logits (``artlite.moe.plan.route``'s arguments, ``plan.py:25-36``)."""
        lg = np.ascontiguousarray(logits, np.float32)
        T = lg.shape[0]
        E = E or lg.shape[1]
        ids, w = np.empty((T, k), np.int32), np.empty((T, k), np.float32)
        rc = self._f("moe_route")(_ptr(lg), T, lg.shape[1], per_col or E, pitch, E, k, int(gating == "sigmoid"),
                                  _ptr(ids), _ptr(w))
        self._check(rc, "moe_route: k / E / per_col")
        return ids, w

    def plan(self, ids: np.ndarray, *, E: int, cols: int = 8, cap: int, chunk: int = 192):
        """``moe_plan``: (experts (cols, cap), counts (cols), sizes (cols, cap), rows (cols, cap, chunk), pos (T, k))."""
        ids = np.ascontiguousarray(ids, np.int32)
        ex, counts = np.zeros((cols, cap), np.int32), np.zeros(cols, np.int32)
        sizes, rows = np.zeros((cols, cap), np.int32), np.zeros((cols, cap, chunk), np.int32)
        pos = np.zeros(ids.shape, np.int64)
        rc = self._f("moe_plan")(_ptr(ids), ids.shape[0], ids.shape[1], E, cols, cap, chunk, _ptr(ex), _ptr(counts),
                                 _ptr(sizes), _ptr(rows), _ptr(pos))
        self._check(rc, "moe_plan")
        return ex, counts, sizes, rows, pos

    def dequant_rows(self, qtype: str, raw: np.ndarray, cols: int) -> np.ndarray:
        """(n, cols) fp32 of n raw GGUF rows (a (n, row_bytes) uint8 array)."""
        raw = np.ascontiguousarray(raw, np.uint8)
        out = np.empty((raw.shape[0], cols), np.float32)
        rc = self._f("dequant_rows")(qtype.encode(), _ptr(raw), raw.shape[0], raw.shape[1], cols, _ptr(out))
        self._check(rc, f"dequant_rows {qtype}")
        return out


class Oracle(_Lib):
    """The C restatement (``oracle.c``)."""

    def __init__(self):
        super().__init__(LIB, "oracle_")
        self.lib.oracle_moe_dispatch.argtypes = [_P, _I64, _I, _I, _P, _P, _P]
        self.lib.oracle_moe_dispatch.restype = _I

    def dispatch(self, ids: np.ndarray, E: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(offsets (E + 1,) int64, perm (T k,) int32, slot (T k,) int32): pairs in expert-then-pair order."""
        ids = np.ascontiguousarray(ids, np.int32)
        offsets = np.zeros(E + 1, np.int64)
        perm, slot = np.zeros(ids.size, np.int32), np.zeros(ids.size, np.int32)
        rc = self.lib.oracle_moe_dispatch(_ptr(ids), ids.shape[0], ids.shape[1], E, _ptr(offsets), _ptr(perm),
                                          _ptr(slot))
        self._check(rc, "dispatch: expert id")
        return offsets, perm, slot


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = next((line for line in f if line.startswith("flags")), "").split()
    except OSError:
        return False
    return all(x in flags for x in ("avx512f", "avx512dq", "avx512bw", "avx512vl"))


def oracle() -> Oracle:
    if not os.path.exists(LIB):
        build()
    return Oracle()


def reference() -> _Lib | None:
    """The reference's compiled host code, or None (not built, or a host CPU without AVX-512: its vector routing path
    is compiled in unconditionally)."""
    if not os.path.exists(REF_LIB) or not _cpu_has_avx512():
        return None
    return _Lib(REF_LIB, "artlite_ref_")
