"""The MoE block's host API: ``plan`` (the reference's ``artlite.moe.plan``: ``route``, ``Plan``) and ``block``
(``MoEBlock``: the whole block on the GPU)."""
