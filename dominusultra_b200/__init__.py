"""B200-native (sm_100a) fused-RoPE causal attention: the DominusUltra hot path.

Public API (drop-in for the reference module ``dominus_ultra``):
``precompute_rope_cos_sin``, ``dominus_ultra_prefill``, ``dominus_ultra_decode``; the
generation-loop step ``dominus_ultra_decode_kvcache`` (per-sequence lengths, KV append);
multi-shard decode helpers ``decode_partial`` / ``merge_partials``; sharding in ``dist``.
"""

from .attention import (  # noqa: F401
    decode_partial,
    dominus_ultra_decode,
    dominus_ultra_decode_kvcache,
    dominus_ultra_prefill,
    merge_partials,
    precompute_rope_cos_sin,
)

__version__ = "0.1.0"
