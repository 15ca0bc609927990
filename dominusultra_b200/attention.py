"""Drop-in Python API of DominusUltra's fused-RoPE attention, backed by sm_100a CUDA.

Same names, signatures, argument meaning, validation order and error messages as the reference
module ``dominus_ultra.py``; the Triton launches are replaced by calls into the C ABI of
``libdominus_b200.so`` (``include/dominus_ultra_b200.h``). Launches go to torch's current
stream of the tensors' device and return without synchronising, like the reference.
There is no CPU path: CPU tensors are rejected exactly as the reference rejects them.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import torch

from . import _lib

__all__ = [
    "precompute_rope_cos_sin",
    "dominus_ultra_prefill",
    "dominus_ultra_decode",
    "dominus_ultra_decode_kvcache",
    "decode_partial",
    "merge_partials",
]


def precompute_rope_cos_sin(
    max_seq_len: int, dim: int, device, dtype=torch.float32, base: float = 10000.0
) -> Tuple[torch.Tensor, torch.Tensor]:
    """
    Pre-compute RoPE (Rotary Position Embedding) cos/sin values.

    Same contract as the reference (``dominus_ultra.py:25-58``): returns ``(cos, sin)``, each
    ``[max_seq_len, dim // 2]``, computed in fp32 as ``cos/sin(t * base ** (-2j / dim))`` and
    cast to ``dtype``; bit-identical to the reference on CPU. Runs on any device.
    """
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be positive")
    if dim <= 0 or dim % 2 != 0:
        raise ValueError("dim must be a positive even integer")
    if base <= 0:
        raise ValueError("base must be positive")

    inv_freq = 1.0 / (
        base ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim)
    )
    t = torch.arange(max_seq_len, device=device, dtype=torch.float32)
    freqs = torch.einsum("i,j->ij", t, inv_freq)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def _validate_head_dim(head_dim: int) -> None:
    # dominus_ultra.py:70-72
    if head_dim < 16 or head_dim > 256 or head_dim & (head_dim - 1):
        raise ValueError("head_dim must be a power of two between 16 and 256")


def _validate_rope_tables(
    cos: torch.Tensor,
    sin: torch.Tensor,
    positions: int,
    head_dim: int,
    device: torch.device,
    dtype: torch.dtype,
) -> None:
    # dominus_ultra.py:75-101
    expected_tail = (head_dim // 2,)
    if cos.ndim != 2 or sin.ndim != 2:
        raise ValueError("cos and sin must be rank-2 [positions, head_dim // 2] tensors")
    if cos.shape[0] < positions or sin.shape[0] < positions:
        raise ValueError(f"cos and sin must contain at least {positions} positions")
    if cos.shape[1:] != expected_tail or sin.shape[1:] != expected_tail:
        raise ValueError(f"cos and sin must have trailing shape {expected_tail}")
    if cos.device != device or sin.device != device:
        raise ValueError("cos and sin must be on the same device as the attention tensors")
    if cos.dtype != dtype or sin.dtype != dtype:
        raise ValueError("cos and sin must have the same dtype as the attention tensors")
    if not cos.is_contiguous() or not sin.is_contiguous():
        raise ValueError("cos and sin must be contiguous")


def _validate_attention_tensors(*tensors: torch.Tensor) -> None:
    # dominus_ultra.py:104-116
    first = tensors[0]
    if not first.is_cuda:
        raise ValueError("DominusUltra kernels require CUDA tensors")
    if first.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("attention tensors must use float16 or bfloat16")
    for tensor in tensors:
        if tensor.device != first.device:
            raise ValueError("all attention tensors must be on the same CUDA device")
        if tensor.dtype != first.dtype:
            raise ValueError("all attention tensors must have the same dtype")
        if not tensor.is_contiguous():
            raise ValueError("attention tensors must be contiguous")


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _lib.DU_DTYPE_BF16
    if dtype == torch.float16:
        return _lib.DU_DTYPE_F16
    if dtype == torch.float32:
        return _lib.DU_DTYPE_F32
    raise ValueError(f"unsupported dtype {dtype}")


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The kernels read through TMA / 128-bit loads, which need 16-byte aligned bases.

    A contiguous view at an odd storage offset is copied into a fresh (aligned) buffer.
    """
    return t if t.data_ptr() % 16 == 0 else t.clone()


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """Handle of torch's current stream on `device` (without building a Stream object when the
    raw getter is available: this is on every call's host path)."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


# Workspace sizes by (entry point, sizes, device): a ctypes call per launch otherwise.
_WS_SIZES = {}


def _ws_size(fn_name: str, B: int, Hq: int, Hkv: int, L: int, D: int, device) -> int:
    key = (fn_name, B, Hq, Hkv, L, D, device.index)
    n = _WS_SIZES.get(key)
    if n is None:
        n = int(getattr(_lib.load(), fn_name)(B, Hq, Hkv, L, D))
        _WS_SIZES[key] = n
    return n


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


class _OnDevice:
    """Make `device` current only when it is not already (the common case costs one call)."""

    __slots__ = ("index", "prev")

    def __init__(self, device: torch.device):
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


# Workspace per (kind, device, stream): [buffer, used under a graph capture], reused across
# calls, since kernels on one stream run in order; grown on demand.
_WORKSPACES = {}
# Outgrown buffers that a captured CUDA graph may still reference: never freed.
_RETIRED = []


def dominus_ultra_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """
    Prefill phase attention with RoPE and optional Grouped Query Attention.

    Computes causal multi-head attention with fused Rotary Position Embeddings on the B200
    tensor cores (``du_prefill``). Supports Grouped Query Attention (GQA) and Multi-Query
    Attention (MQA). Reference: ``dominus_ultra.py:416-501``.

    Args:
        q: Query tensor of shape [batch, num_heads, seq_len, head_dim]
        k: Key tensor of shape [batch, num_kv_heads, seq_len, head_dim]
        v: Value tensor of shape [batch, num_kv_heads, seq_len, head_dim]
        cos: Pre-computed cosine values from precompute_rope_cos_sin
        sin: Pre-computed sine values from precompute_rope_cos_sin
        num_kv_heads: Number of KV heads for GQA. If None, uses num_query_heads (MHA)

    Returns:
        Tuple of:
            - out: Output tensor of shape [batch, num_heads, seq_len, head_dim]
            - lse: Log-sum-exp values (natural log, fp32) of shape [batch, num_heads, seq_len]
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must be rank-4 tensors")

    B, Hq, T, D = q.shape
    _, Hk, _, _ = k.shape
    KvH = num_kv_heads if num_kv_heads is not None else Hq
    if B <= 0 or Hq <= 0 or T <= 0:
        raise ValueError("batch, heads, and sequence length must be positive")
    if KvH <= 0 or Hq % KvH != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if k.shape != (B, KvH, T, D) or v.shape != (B, KvH, T, D):
        raise ValueError("k and v must have shape [batch, num_kv_heads, seq_len, head_dim]")
    if Hk != KvH:
        raise ValueError("k head count does not match num_kv_heads")

    _validate_head_dim(D)
    _validate_attention_tensors(q, k, v)
    _validate_rope_tables(cos, sin, T, D, q.device, q.dtype)

    lib = _lib.load()
    q, k, v, cos, sin = (_aligned(t) for t in (q, k, v, cos, sin))
    out = torch.empty_like(q)
    lse = torch.empty((B, Hq, T), dtype=torch.float32, device=q.device)
    scale = 1.0 / (D**0.5)
    with _OnDevice(q.device):
        stream = _stream(q.device)
        ws, ws_bytes = _cached_workspace(
            "prefill", _ws_size("du_prefill_workspace_size", B, Hq, KvH, T, D, q.device), q.device,
            stream,
        )
        rc = lib.du_prefill(
            _ptr(q), _ptr(k), _ptr(v), _ptr(cos), _ptr(sin), _ptr(out), _ptr(lse),
            B, Hq, KvH, T, D, _dtype_code(q.dtype), scale,
            min(cos.shape[0], sin.shape[0]), ws, ws_bytes, stream,
        )
    _lib.check(rc, "du_prefill")
    return out, lse


def _cached_workspace(kind: str, nbytes: int, device, stream: int):
    """(pointer, bytes) of a per-(kind, device, stream) scratch buffer of at least nbytes, grown on
    demand. Calls on one stream are ordered, so reusing the buffer across them is safe.

    A buffer that a CUDA graph capture has used stays referenced by that graph's kernels, so
    when it is outgrown it is kept alive (``_RETIRED``) instead of being returned to the caching
    allocator, where a later allocation could take the memory the graph still writes on every
    replay. Buffers only ever used eagerly are released when outgrown (stream order makes that
    safe). Growth is at least geometric, so few buffers are ever retired.
    """
    if nbytes == 0:
        return 0, 0
    key = (kind, device.index, stream)
    entry = _WORKSPACES.get(key)
    capturing = torch.cuda.is_current_stream_capturing()
    if entry is None or entry[0].numel() < nbytes:
        if entry is not None and entry[1]:
            _RETIRED.append(entry[0])
        size = max(nbytes, 1 << 20, 2 * entry[0].numel() if entry is not None else 0)
        # zero-filled: the decode split walk keeps its ticket counters at the front, and every
        # call leaves them zero
        entry = [torch.zeros(size, dtype=torch.uint8, device=device), capturing]
        _WORKSPACES[key] = entry
    elif capturing:
        entry[1] = True
    return entry[0].data_ptr(), entry[0].numel()


def _workspace(B: int, Hq: int, Hkv: int, L: int, D: int, device, stream: int):
    nbytes = _ws_size("du_decode_workspace_size", B, Hq, Hkv, L, D, device)
    return _cached_workspace("decode", nbytes, device, stream)


def dominus_ultra_decode(
    q_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int] = None,
) -> torch.Tensor:
    """
    Decode phase attention for autoregressive generation with KV cache.

    Computes attention for a single new token (rotated at position ``past_len``) against
    cached keys (rotated at positions ``0..past_len-1``) with a split-KV streaming kernel
    (``du_decode``). Reference: ``dominus_ultra.py:504-583``.

    Args:
        q_new: New query tensor of shape [batch, num_heads, 1, head_dim]
        k_cache: Cached key tensor of shape [batch, num_kv_heads, past_len, head_dim]
        v_cache: Cached value tensor of shape [batch, num_kv_heads, past_len, head_dim]
        cos: Pre-computed cosine values from precompute_rope_cos_sin
        sin: Pre-computed sine values from precompute_rope_cos_sin
        num_kv_heads: Number of KV heads for GQA. If None, uses num_query_heads (MHA)

    Returns:
        Output tensor of shape [batch, num_heads, 1, head_dim]
    """
    if q_new.ndim != 4 or k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("q_new, k_cache, and v_cache must be rank-4 tensors")

    B, Hq, _, D = q_new.shape
    _, Hk, past_T, _ = k_cache.shape
    KvH = num_kv_heads if num_kv_heads is not None else Hq
    if q_new.shape[2] != 1:
        raise ValueError("q_new must contain exactly one sequence position")
    if B <= 0 or Hq <= 0 or past_T <= 0:
        raise ValueError("batch, heads, and cache length must be positive")
    if KvH <= 0 or Hq % KvH != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if k_cache.shape != (B, KvH, past_T, D) or v_cache.shape != (B, KvH, past_T, D):
        raise ValueError("k_cache and v_cache must have matching GQA cache shapes")
    if Hk != KvH:
        raise ValueError("cache head count does not match num_kv_heads")

    _validate_head_dim(D)
    _validate_attention_tensors(q_new, k_cache, v_cache)
    _validate_rope_tables(cos, sin, past_T + 1, D, q_new.device, q_new.dtype)

    lib = _lib.load()
    q_new, k_cache, v_cache, cos, sin = (_aligned(t) for t in (q_new, k_cache, v_cache, cos, sin))
    out = torch.empty_like(q_new).squeeze(2)
    scale = 1.0 / (D**0.5)
    with _OnDevice(q_new.device):
        stream = _stream(q_new.device)
        ws, nbytes = _workspace(B, Hq, KvH, past_T, D, q_new.device, stream)
        rc = lib.du_decode(
            _ptr(q_new), _ptr(k_cache), _ptr(v_cache), _ptr(cos), _ptr(sin), _ptr(out),
            B, Hq, KvH, past_T, D, _dtype_code(q_new.dtype), scale,
            min(cos.shape[0], sin.shape[0]), ws, nbytes, stream,
        )
    _lib.check(rc, "du_decode")
    return out.unsqueeze(2)


def dominus_ultra_decode_kvcache(
    q_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    cache_seqlens: torch.Tensor,
    k_new: Optional[torch.Tensor] = None,
    v_new: Optional[torch.Tensor] = None,
    num_kv_heads: Optional[int] = None,
) -> torch.Tensor:
    """
    One decode step of a generation loop: per-sequence cache lengths, new token appended.

    The caller step around ``dominus_ultra_decode`` (``dominus_ultra.py:504-583``), which takes
    one length for the whole batch and attends to the cache without the current token
    (``dominus_ultra.py:350``). Here ``k_cache`` / ``v_cache`` are preallocated to a capacity
    ``max_len`` and sequence ``b`` holds ``s_b = cache_seqlens[b]`` tokens:

    * with ``k_new`` / ``v_new`` (``[batch, num_kv_heads, 1, head_dim]``) the new token's key
      and value are written in place to row ``s_b`` of the caches, and the query attends to
      keys ``0..s_b`` (itself included);
    * without them the query attends to keys ``0..s_b-1`` (``dominus_ultra_decode`` of that
      prefix).

    The query rotates at position ``s_b`` and cached key ``j`` at ``j``. ``cache_seqlens`` is
    not advanced (the caller adds 1 after an append). When it is a CUDA tensor it is read on
    the GPU: the call never synchronises, and a captured CUDA graph stays valid as the lengths
    change. A length out of range (``s_b < 0`` or ``s_b + 1 > max_len`` with an append) cannot
    raise without a sync: that sequence's output is zero, nothing is appended, and
    ``_lib.read_status()`` reports code 6. A CPU ``cache_seqlens`` is checked here instead.

    Args:
        q_new: [batch, num_heads, 1, head_dim]
        k_cache, v_cache: [batch, num_kv_heads, max_len, head_dim], contiguous, updated in place
        cos, sin: tables from precompute_rope_cos_sin covering max_len positions (max_len + 1
            without an append)
        cache_seqlens: [batch] integer tokens already cached per sequence
        k_new, v_new: [batch, num_kv_heads, 1, head_dim] or None (both)
        num_kv_heads: Number of KV heads for GQA. If None, uses num_query_heads (MHA)

    Returns:
        Output tensor of shape [batch, num_heads, 1, head_dim]
    """
    if q_new.ndim != 4 or k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("q_new, k_cache, and v_cache must be rank-4 tensors")
    if (k_new is None) != (v_new is None):
        raise ValueError("k_new and v_new must be given together")
    append = k_new is not None
    B, Hq, _, D = q_new.shape
    _, Hk, max_len, _ = k_cache.shape
    KvH = num_kv_heads if num_kv_heads is not None else Hq
    if q_new.shape[2] != 1:
        raise ValueError("q_new must contain exactly one sequence position")
    if B <= 0 or Hq <= 0 or max_len <= 0:
        raise ValueError("batch, heads, and cache length must be positive")
    if KvH <= 0 or Hq % KvH != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if k_cache.shape != (B, KvH, max_len, D) or v_cache.shape != (B, KvH, max_len, D):
        raise ValueError("k_cache and v_cache must have matching GQA cache shapes")
    if Hk != KvH:
        raise ValueError("cache head count does not match num_kv_heads")
    if append and (k_new.shape != (B, KvH, 1, D) or v_new.shape != (B, KvH, 1, D)):
        raise ValueError("k_new and v_new must have shape [batch, num_kv_heads, 1, head_dim]")
    if cache_seqlens.ndim != 1 or cache_seqlens.shape[0] != B:
        raise ValueError("cache_seqlens must have shape [batch]")
    if cache_seqlens.dtype not in (torch.int32, torch.int64):
        raise ValueError("cache_seqlens must be an int32 or int64 tensor")

    _validate_head_dim(D)
    tensors = (q_new, k_cache, v_cache) + ((k_new, v_new) if append else ())
    _validate_attention_tensors(*tensors)
    _validate_rope_tables(cos, sin, max_len + (0 if append else 1), D, q_new.device, q_new.dtype)
    if k_cache.data_ptr() % 16 or v_cache.data_ptr() % 16:
        raise ValueError("k_cache and v_cache must be 16-byte aligned (they are updated in place)")
    if cache_seqlens.device.type == "cpu":
        lens = cache_seqlens.tolist()
        hi = max_len - (1 if append else 0)
        bad = [i for i, s in enumerate(lens) if s < 0 or s > hi]
        if bad:
            raise ValueError(
                f"cache_seqlens[{bad[0]}] = {lens[bad[0]]} is outside [0, {hi}] "
                f"for a cache of {max_len} positions" + (" with an append" if append else "")
            )
        cache_seqlens = cache_seqlens.to(q_new.device)
    elif cache_seqlens.device != q_new.device:
        raise ValueError("cache_seqlens must be on the device of q_new (or on the CPU)")
    if cache_seqlens.dtype != torch.int32:
        cache_seqlens = cache_seqlens.to(torch.int32)
    seqlens = cache_seqlens.contiguous()

    lib = _lib.load()
    q_new, cos, sin = (_aligned(t) for t in (q_new, cos, sin))
    if append:
        k_new, v_new = _aligned(k_new), _aligned(v_new)
    out = torch.empty_like(q_new).squeeze(2)
    scale = 1.0 / (D**0.5)
    with _OnDevice(q_new.device):
        stream = _stream(q_new.device)
        ws, nbytes = _cached_workspace(
            "decode_kvcache",
            _ws_size("du_decode_kvcache_workspace_size", B, Hq, KvH, max_len, D, q_new.device),
            q_new.device,
            stream,
        )
        rc = lib.du_decode_kvcache(
            _ptr(q_new), _ptr(k_new), _ptr(v_new), _ptr(k_cache), _ptr(v_cache), _ptr(seqlens),
            _ptr(cos), _ptr(sin), _ptr(out), B, Hq, KvH, max_len, D, _dtype_code(q_new.dtype),
            scale, min(cos.shape[0], sin.shape[0]), ws, nbytes, stream,
        )
    _lib.check(rc, "du_decode_kvcache")
    return out.unsqueeze(2)


def decode_partial(
    q_new: torch.Tensor,
    k_shard: torch.Tensor,
    v_shard: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int],
    q_pos: int,
    kv_pos_offset: int,
    out: Optional[torch.Tensor] = None,
    lse: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Decode over one shard of the KV sequence (``du_decode_partial``).

    Keys of the shard sit at absolute positions ``kv_pos_offset + j`` and the query at
    ``q_pos``. Returns fp32 ``(out [B, Hq, D], lse [B, Hq])`` normalised over the shard, for
    ``merge_partials``. ``out`` / ``lse`` may be preallocated views (e.g. of a packed buffer).
    """
    B, Hq, _, D = q_new.shape
    L = k_shard.shape[2]
    KvH = num_kv_heads if num_kv_heads is not None else Hq
    _validate_head_dim(D)
    _validate_attention_tensors(q_new, k_shard, v_shard)
    _validate_rope_tables(cos, sin, max(q_pos, kv_pos_offset + L - 1) + 1, D, q_new.device, q_new.dtype)
    lib = _lib.load()
    q_new, k_shard, v_shard, cos, sin = (_aligned(t) for t in (q_new, k_shard, v_shard, cos, sin))
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.float32, device=q_new.device)
    if lse is None:
        lse = torch.empty((B, Hq), dtype=torch.float32, device=q_new.device)
    with _OnDevice(q_new.device):
        stream = _stream(q_new.device)
        ws, nbytes = _workspace(B, Hq, KvH, L, D, q_new.device, stream)
        rc = lib.du_decode_partial(
            _ptr(q_new), _ptr(k_shard), _ptr(v_shard), _ptr(cos), _ptr(sin), _ptr(out), _ptr(lse),
            B, Hq, KvH, L, D, _dtype_code(q_new.dtype), 1.0 / (D**0.5),
            int(q_pos), int(kv_pos_offset), min(cos.shape[0], sin.shape[0]),
            ws, nbytes, stream,
        )
    _lib.check(rc, "du_decode_partial")
    return out, lse


def merge_partials(
    o_parts: torch.Tensor,
    lse_parts: torch.Tensor,
    out_dtype: torch.dtype,
    with_lse: bool = False,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """LSE-weighted merge of ``R`` partials (``du_merge_partials``).

    ``o_parts`` is fp32 ``[R, *rows, D]`` and ``lse_parts`` fp32 ``[R, *rows]`` (any strides
    along R and a contiguous row block). Returns ``out [*rows, D]`` in ``out_dtype`` and, with
    ``with_lse``, the merged fp32 ``lse [*rows]``.
    """
    if o_parts.dtype != torch.float32 or lse_parts.dtype != torch.float32:
        raise ValueError("partials must be float32")
    if not o_parts.is_cuda or not lse_parts.is_cuda:
        raise ValueError("DominusUltra kernels require CUDA tensors")
    R = o_parts.shape[0]
    D = o_parts.shape[-1]
    row_shape: Sequence[int] = tuple(o_parts.shape[1:-1])
    if tuple(lse_parts.shape) != (R, *row_shape):
        raise ValueError("lse_parts must have shape [R, *rows] matching o_parts")
    o2 = o_parts.reshape(R, -1, D)
    l2 = lse_parts.reshape(R, -1)
    if o2.stride(2) != 1 or o2.stride(1) != D or l2.stride(1) != 1:
        raise ValueError("each partial must be a contiguous [rows, D] / [rows] block")
    rows = o2.shape[1]
    out = torch.empty((*row_shape, D), dtype=out_dtype, device=o_parts.device)
    lse = torch.empty(row_shape, dtype=torch.float32, device=o_parts.device) if with_lse else None
    lib = _lib.load()
    with _OnDevice(o_parts.device):
        rc = lib.du_merge_partials(
            _ptr(o2), _ptr(l2), R, rows, D, o2.stride(0), o2.stride(1), l2.stride(0), l2.stride(1),
            _ptr(out), _dtype_code(out_dtype), _ptr(lse), _stream(o_parts.device),
        )
    _lib.check(rc, "du_merge_partials")
    return out, lse
