"""artlite_b200: artlite's GGUF mixture-of-experts block on NVIDIA B200 (sm_100a).

The host side is NumPy + ctypes only (no torch): ``artlite_b200.moe.plan`` mirrors ``artlite.moe.plan`` (``route``,
``Plan``), ``artlite_b200.moe.block.MoEBlock`` runs the whole block, ``artlite_b200.gguf`` reads GGUF files; all of them
call ``lib/libartlite_moe_cuda.so`` through the C ABI of ``include/artlite_moe.h``. There is no CPU fallback: without
the built library (or without a GPU) every call raises ``Error``.
"""

from ._lib import Error, CapacityError, lib  # noqa: F401

__all__ = ["Error", "CapacityError", "lib"]
