"""Standalone half-split RoPE on the B200 (drop-in for the reference's ``rope`` module).

``apply_rope`` / ``apply_rope_backward`` keep the reference's signatures, validation order and
messages (reference ``rope.py:110-121``, ``:179-220``) and run the sm_100a rotary kernel
(``du_rope``, ``csrc/rope_sm100.cuh``) once per tensor. Tables come from
``make_half_split_pos_emb`` in the input dtype exactly as the reference builds them
(``rope.py:124-144``), cached per (length, head_dim, device, dtype, base, scale_factor).
The same kernel rotates the keys of every prefill (``du_prefill``) once per (b, kv head).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from .attention import _OnDevice, _dtype_code, _ptr, _stream

__all__ = ["apply_rope", "apply_rope_backward", "make_half_split_pos_emb", "make_interleaved_pos_emb"]


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


def _validate_pair(first: torch.Tensor, second: torch.Tensor) -> None:
    if first.ndim != 4 or second.ndim != 4 or first.shape != second.shape:
        raise ValueError("Q and K must have the same rank-4 [B, H, T, D] shape")
    if not first.is_cuda or not second.is_cuda:
        raise ValueError("the standalone RoPE kernels require CUDA tensors")
    if first.device != second.device or first.dtype != second.dtype:
        raise ValueError("Q and K must have the same device and dtype")
    if first.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("Q and K must use float16 or bfloat16")
    if not first.is_contiguous() or not second.is_contiguous():
        raise ValueError("Q and K must be contiguous")
    head_dim = first.shape[-1]
    if head_dim < 16 or head_dim > 256 or head_dim & (head_dim - 1):
        raise ValueError("head_dim must be a power of two between 16 and 256")


def _validate_output(output: torch.Tensor, reference: torch.Tensor, name: str) -> None:
    if (
        output.shape != reference.shape
        or output.device != reference.device
        or output.dtype != reference.dtype
        or not output.is_contiguous()
    ):
        raise ValueError(f"{name} must be contiguous and match its input shape/device/dtype")


_TABLES: dict = {}


def _tables(T: int, D: int, device: torch.device, dtype: torch.dtype, base: float, scale: float):
    key = (T, D, device, dtype, float(base), float(scale))
    tab = _TABLES.get(key)
    if tab is None:
        if len(_TABLES) >= 32:
            _TABLES.clear()
        tab = make_half_split_pos_emb(T, D, str(device), dtype, base, scale)
        tab = (tab[0].contiguous(), tab[1].contiguous())
        _TABLES[key] = tab
    return tab


def _launch(
    first: torch.Tensor,
    second: torch.Tensor,
    output_first: torch.Tensor,
    output_second: torch.Tensor,
    base: float,
    scale_factor: float,
    backward: bool,
) -> Tuple[torch.Tensor, torch.Tensor]:
    _validate_pair(first, second)
    _validate_output(output_first, first, "first output")
    _validate_output(output_second, second, "second output")
    B, H, T, D = first.shape
    cos, sin = _tables(T, D, first.device, first.dtype, base, scale_factor)
    lib = _lib.load()
    code = _dtype_code(first.dtype)
    with _OnDevice(first.device):
        stream = _stream(first.device)
        for src, dst in ((first, output_first), (second, output_second)):
            rc = lib.du_rope(
                _ptr(src), _ptr(cos), _ptr(sin), _ptr(dst), B, H, T, D, code, code, 0, T,
                1 if backward else 0, stream,
            )
            _lib.check(rc, "du_rope")
    return output_first, output_second


def apply_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    base: float = 10000.0,
    scale_factor: float = 1.0,
    out_q: Optional[torch.Tensor] = None,
    out_k: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Apply half-split RoPE to Q and K (positions 0..T-1)."""
    out_q = torch.empty_like(q) if out_q is None else out_q
    out_k = torch.empty_like(k) if out_k is None else out_k
    return _launch(q, k, out_q, out_k, base, scale_factor, backward=False)


def apply_rope_backward(
    grad_out_q: torch.Tensor,
    grad_out_k: torch.Tensor,
    base: float = 10000.0,
    scale_factor: float = 1.0,
    grad_q: Optional[torch.Tensor] = None,
    grad_k: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Apply the exact transpose rotation to Q/K output gradients."""
    grad_q = torch.empty_like(grad_out_q) if grad_q is None else grad_q
    grad_k = torch.empty_like(grad_out_k) if grad_k is None else grad_k
    return _launch(grad_out_q, grad_out_k, grad_q, grad_k, base, scale_factor, backward=True)
