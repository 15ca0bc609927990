"""Half-split Rotary Position Embedding tables (drop-in for the reference's ``rope`` module).

``make_half_split_pos_emb`` and ``make_interleaved_pos_emb`` keep the reference's signatures
and produce bit-identical tables (``rope.py:124-166`` of the reference); the fused attention
path uses the same half-split convention (``dominus_ultra.precompute_rope_cos_sin``).
"""

from __future__ import annotations

from typing import Tuple

import torch

__all__ = ["make_half_split_pos_emb", "make_interleaved_pos_emb"]


def make_half_split_pos_emb(
    seq_len: int,
    head_dim: int,
    device: str = "cuda",
    dtype: torch.dtype = torch.float32,
    base: float = 10000.0,
    scale_factor: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Create half-width cosine and sine tables used by half-split RoPE."""
    if seq_len <= 0:
        raise ValueError("seq_len must be positive")
    if head_dim <= 0 or head_dim % 2:
        raise ValueError("head_dim must be a positive even integer")
    if base <= 0 or scale_factor <= 0:
        raise ValueError("base and scale_factor must be positive")
    inv_freq = 1.0 / (
        base ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim)
    )
    inv_freq = inv_freq * scale_factor
    angles = torch.arange(seq_len, device=device, dtype=torch.float32)[:, None] * inv_freq[None, :]
    return angles.cos().to(dtype), angles.sin().to(dtype)


def make_interleaved_pos_emb(
    seq_len: int,
    head_dim: int,
    device: str = "cuda",
    dtype: torch.dtype = torch.float32,
    base: float = 10000.0,
    scale_factor: float = 1.0,
) -> torch.Tensor:
    """Compatibility helper returning ``[cos_0, sin_0, ...]`` columns."""
    cos, sin = make_half_split_pos_emb(seq_len, head_dim, device, dtype, base, scale_factor)
    output = torch.empty((seq_len, head_dim), device=device, dtype=dtype)
    output[:, 0::2] = cos
    output[:, 1::2] = sin
    return output
