"""The C ABI on CPU (no compute calls): libartlite_moe_cuda.so exists, loads, and exports every entry point that
include/artlite_moe.h declares; the host package stays torch-free (the reference's tests/test_no_torch.py:7-43 rule
for its src/artlite); the Python mirror keeps the reference's signatures."""

import ctypes
import importlib
import inspect
import os
import re
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared() -> list[str]:
    text = open(os.path.join(REPO, "include", "artlite_moe.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(artlite_\w+)\s*\(", text)))


def test_header_matches_binding_table():
    from artlite_b200 import _lib
    assert declared() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    from artlite_b200 import _lib
    path = _lib.lib_path()
    assert os.path.exists(path), f"{path}: run __graft_entry__.build()"
    lb = ctypes.CDLL(path)
    for name in declared():
        assert hasattr(lb, name), name
    # and exports nothing else of its own (visibility hidden)
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True).stdout
    ours = sorted({ln.split()[-1] for ln in out.splitlines() if " T artlite_" in ln})
    assert ours == declared()


def test_version_and_last_error_without_gpu():
    from artlite_b200 import _lib
    lb = _lib.lib()
    assert b"sm_100a" in lb.artlite_moe_version()
    assert lb.artlite_moe_last_error() is not None


def test_argument_errors_need_no_gpu():
    """The reference's artlite::Error cases are checked before any CUDA call (moe_host.cpp:188)."""
    from artlite_b200 import Error
    from artlite_b200.moe import plan
    import numpy as np
    with pytest.raises(Error, match="moe_route: k 9 of E 8"):
        plan.route(np.zeros((2, 8), np.float32), 9)
    with pytest.raises(Error, match="per column"):
        plan.route(np.zeros((2, 8), np.float32), 2, E=8, per_col=3)


def test_host_package_is_torch_free():
    code = (
        "import sys, importlib.abc\n"
        "class Block(importlib.abc.MetaPathFinder):\n"
        "    def find_spec(self, name, path, target=None):\n"
        "        if name == 'torch' or name.startswith('torch.'):\n"
        "            raise ImportError('torch is refused')\n"
        "sys.meta_path.insert(0, Block())\n"
        "import artlite_b200, artlite_b200.moe.plan, artlite_b200.moe.block, artlite_b200.gguf\n"
        "assert 'torch' not in sys.modules\n"
    )
    r = subprocess.run([sys.executable, "-c", code], cwd=REPO, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_mirror_signatures():
    """route / Plan.of keep the reference's parameters (src/artlite/moe/plan.py:25-57)."""
    from artlite_b200.moe import plan
    p = inspect.signature(plan.route).parameters
    assert list(p)[:2] == ["logits", "k"] and all(p[n].kind == p[n].KEYWORD_ONLY for n in ("E", "per_col", "pitch",
                                                                                           "gating"))
    q = inspect.signature(plan.Plan.of).parameters
    assert list(q)[:1] == ["ids"] and q["cap"].kind == q["cap"].KEYWORD_ONLY and q["E"].kind == q["E"].KEYWORD_ONLY
    assert plan.CHUNK == 192 and plan.COLS == 8
