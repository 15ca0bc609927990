"""CPU oracle for the fused-RoPE causal attention path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this package, and only as the checker or as the timed
CPU baseline. The product path (``dominusultra_b200``) never imports it.
"""

from .oracle import (  # noqa: F401
    apply_rope,
    apply_rope_backward,
    decode,
    decode_kvcache,
    decode_partial,
    merge_partials,
    precompute_rope_cos_sin,
    prefill,
    prefill_block,
    prefill_rows,
)
