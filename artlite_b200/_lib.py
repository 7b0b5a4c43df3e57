"""ctypes binding of ``lib/libartlite_moe_cuda.so`` (the C ABI of ``include/artlite_moe.h``).

Errors: a non-zero status raises ``Error`` with the library's message, as the reference's bindings translate
``artlite::Error`` into the Python exception ``artlite.Error`` (csrc/bindings/errors.cpp, src/artlite/__init__.py:48).
The library location can be overridden with ``ARTLITE_CUDA_LIB``. Loading never falls back to anything else."""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_LIB = os.path.join(HERE, "lib", "libartlite_moe_cuda.so")

OK, EINVAL, ECAPACITY, ECUDA, ENCCL, ETIMEOUT, EDEVICE, EUNSUPPORTED = 0, -1, -2, -3, -4, -5, -6, -7
# ggml tensor type ids (include/artlite_moe.h; gguf_model.py:385-390)
QTYPES = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q8_0": 8, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ4_NL": 20,
          "IQ4_XS": 23, "BF16": 30}

# every entry point include/artlite_moe.h declares (tests check the library exports each of them)
EXPORTS = ("artlite_moe_last_error", "artlite_moe_version", "artlite_moe_route", "artlite_moe_plan",
           "artlite_moe_dispatch", "artlite_moe_dispatch_noalloc", "artlite_dequant_supported", "artlite_dequant_rows", "artlite_moe_create",
           "artlite_moe_set_weights", "artlite_moe_set_router_bias", "artlite_moe_set_shared", "artlite_moe_set_norm",
           "artlite_moe_forward",
           "artlite_moe_forward_graph", "artlite_moe_sync", "artlite_moe_debug",
           "artlite_moe_stage_times", "artlite_moe_path", "artlite_moe_weights", "artlite_moe_launch_count", "artlite_moe_destroy",
           "artlite_moe_ep_unique_id", "artlite_moe_ep_init", "artlite_moe_ep_plan")


class Error(RuntimeError):
    """A failed library call (the reference's ``artlite.Error``); ``code`` is the ARTLITE_E* status."""

    def __init__(self, msg: str, code: int = EINVAL):
        super().__init__(msg)
        self.code = code


class CapacityError(Error):
    """``moe_plan``: a column needs more than ``cap`` chunks (moe_host.cpp:223)."""


class MoeDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("hidden", "n_experts", "top_k", "expert_ffn", "n_layers", "gating",
                                              "act_dtype", "max_tokens", "device", "path", "ep_rank", "ep_world")]


_P, _I64, _I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
_SIGS = {
    "artlite_moe_last_error": ([], ctypes.c_char_p),
    "artlite_moe_version": ([], ctypes.c_char_p),
    "artlite_moe_route": ([_P, _I64, _I64, _I, _I64, _I, _I, _I, _P, _P], _I),
    "artlite_moe_plan": ([_P, _I64, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P], _I),
    "artlite_moe_dispatch": ([_P, _I64, _I, _I, _P, _P, _P], _I),
    "artlite_moe_dispatch_noalloc": ([_P, _I64, _I, _I, _P, _P, _P, _P], _I),
    "artlite_dequant_supported": ([ctypes.c_char_p], _I),
    "artlite_dequant_rows": ([ctypes.c_char_p, _P, _I64, _I64, _I64, _P], _I),
    "artlite_moe_create": ([ctypes.POINTER(MoeDesc), ctypes.POINTER(_P)], _I),
    "artlite_moe_set_weights": ([_P, _I, _I, _P, _P, _I, _P, _P, _I], _I),
    "artlite_moe_set_router_bias": ([_P, _I, _P], _I),
    "artlite_moe_set_shared": ([_P, _I, _I, _I, _P, _P, _I, _P, _P, _I], _I),
    "artlite_moe_set_norm": ([_P, _I, _P, _I, ctypes.c_double], _I),
    "artlite_moe_forward": ([_P, _I, _P, _P, _I64, _P], _I),
    "artlite_moe_forward_graph": ([_P, _I, _P, _P, _I64, _P], _I),
    "artlite_moe_sync": ([_P, _I], _I),
    "artlite_moe_debug": ([_P, _P, _P, _P, _P, _P], _I),
    "artlite_moe_stage_times": ([_P, _I, _P, ctypes.POINTER(_I)], _I),
    "artlite_moe_path": ([_P, _I], _I),
    "artlite_moe_weights": ([_P, _I, _I, ctypes.POINTER(_P), ctypes.POINTER(_I64)], _I),
    "artlite_moe_launch_count": ([], _I64),
    "artlite_moe_destroy": ([_P], _I),
    "artlite_moe_ep_unique_id": ([_P, _I], _I),
    "artlite_moe_ep_init": ([_P, _P, _I], _I),
    "artlite_moe_ep_plan": ([_P, _P, _I, _I, _I, _P, _P, _P, _P], _I),
}

_lib = None


def lib_path() -> str:
    return os.environ.get("ARTLITE_CUDA_LIB", DEFAULT_LIB)


def lib() -> ctypes.CDLL:
    """The loaded library (raises Error when it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        path = lib_path()
        if not os.path.exists(path):
            raise Error(f"{path} is missing: build it with __graft_entry__.build() (make -C artlite_b200/csrc)")
        lb = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            f = getattr(lb, name)
            f.argtypes, f.restype = args, res
        _lib = lb
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        msg = lib().artlite_moe_last_error().decode(errors="replace")
        raise (CapacityError if rc == ECAPACITY else Error)(msg, rc)
