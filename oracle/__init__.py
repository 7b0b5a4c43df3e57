"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the GGUF MoE block.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm import this package,
and only as the checker; the product (``artlite_b200``) never does.

- ``oracle.lib``: ctypes bindings of ``liboracle.so`` (``oracle.c``: the C restatement of the reference's
  ``moe_route`` / ``moe_plan`` / ``dequant_rows``) and of ``_ref/libartlite_ref.so`` (the reference's own
  ``csrc/artlite/moe_host.cpp`` and ``dequant.cpp`` compiled from its tree, when present).
- ``oracle.moe_np``: the NumPy restatement of the reference's MoE oracle (``tests/moe/ref.py``, ``tests/np_ops.py``),
  the GGUF block dequant of ``src/artlite/gguf_model.py`` and the seeded synthetic block generators.
"""
