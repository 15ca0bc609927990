"""Half-split Rotary Position Embedding (drop-in for the reference's ``rope`` module).

``make_half_split_pos_emb`` and ``make_interleaved_pos_emb`` keep the reference's signatures
and produce bit-identical tables (``rope.py:124-166`` of the reference); ``apply_rope`` and
``apply_rope_backward`` (``rope.py:179-220``) run the sm_100a rotary kernel. Implementation:
``dominusultra_b200.rope``.
"""

from dominusultra_b200.rope import (  # noqa: F401
    apply_rope,
    apply_rope_backward,
    make_half_split_pos_emb,
    make_interleaved_pos_emb,
)

__all__ = ["apply_rope", "apply_rope_backward", "make_half_split_pos_emb", "make_interleaved_pos_emb"]
