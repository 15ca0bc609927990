"""fp32 CPU restatement of DominusUltra's fused-RoPE causal attention.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA path and the timed CPU
baseline; nothing in ``dominusultra_b200`` imports it.

The reference checks its Triton kernels against a torch restatement: half-split RoPE applied
in fp32 with the same (low-precision) cos/sin tables upcast, then
``F.scaled_dot_product_attention`` in fp32. This module restates exactly that path, plus the
log-sum-exp the reference's evidence runner uses:

* RoPE table precompute ............ ``dominus_ultra.py:25-58``
* half-split rotation .............. ``test_dominus.py:32-50`` (== ``gpu_evidence.py:73-80``)
* causal prefill (out) ............. ``test_dominus.py:133-137`` (SDPA, ``is_causal=True``)
* GQA head mapping ................. ``test_dominus.py:180-183`` (``repeat_interleave``),
                                     ``dominus_ultra.py:168`` (``kv_h = h // (H // KvH)``)
* prefill LSE (natural log) ........ ``gpu_evidence.py:277-281`` (``logsumexp`` of masked scores),
                                     kernel store ``dominus_ultra.py:284-285``
* decode ........................... ``test_dominus.py:270-285``: q rotated at position
                                     ``past_len``, keys at ``0..past_len-1``, no mask
* split-KV partial / merge ......... not in the reference; the LSE-weighted merge is the
                                     standard identity used by the build's multi-GPU decode.
* context-parallel block ........... not in the reference: ``prefill`` restricted to a query row
                                     range at given positions against a key range (ring prefill).
* KV-cache step (append + lengths) . not in the reference (its decode excludes the current
                                     token, ``dominus_ultra.py:350``); restated as the reference
                                     decode of each sequence over its own cache prefix
                                     (``test_dominus.py:270-285`` with ``past_len = s_b``), after
                                     writing the new key / value at row ``s_b``.

Pinning: ``tests/test_oracle_golden.py`` checks this module against golden vectors produced by
the reference itself (``tests/golden/make_golden.py``: the reference's own
``precompute_rope_cos_sin`` on CPU, bit-exact, and its Triton ``prefill_kernel`` /
``decode_kernel`` run under Triton's CPU interpreter in fp16).

Everything is computed per (batch, head) block so that memory stays bounded at the larger
benchmark shapes.
"""

from __future__ import annotations

import math
from typing import Iterable, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

__all__ = [
    "precompute_rope_cos_sin",
    "apply_rope",
    "prefill",
    "prefill_rows",
    "prefill_block",
    "decode",
    "decode_partial",
    "decode_kvcache",
    "merge_partials",
]


def precompute_rope_cos_sin(
    max_seq_len: int, dim: int, dtype: torch.dtype = torch.float32, base: float = 10000.0
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Half-width cos/sin tables, ``[max_seq_len, dim // 2]`` (``dominus_ultra.py:53-58``).

    ``inv_freq[j] = 1 / base ** (2j / dim)`` in fp32; ``angle = t * inv_freq`` via an outer
    product; cos/sin evaluated in fp32 and then cast to ``dtype``.
    """
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.einsum("i,j->ij", t, inv_freq)
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotation in fp32 (``test_dominus.py:32-50``).

    For ``i < D/2``: ``x_i * c_i - x_{i+D/2} * s_i``; for ``i >= D/2``:
    ``x_i * c_{i-D/2} + x_{i-D/2} * s_{i-D/2}``. ``cos``/``sin`` rows align with the
    sequence axis of ``x`` and are upcast to fp32.
    """
    x = x.float()
    cos = cos.float()
    sin = sin.float()
    half = x.shape[-1] // 2
    x1 = x[..., :half]
    x2 = x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def apply_rope_backward(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Transpose of ``apply_rope`` in fp32 (the BACKWARD branch of the reference ``_rope_kernel``,
    ``rope.py:62-72``, and its ``_reference(..., backward=True)``, ``rope.py:239-246``):
    ``x_i c_i + x_{i+D/2} s_i`` and ``x_{i+D/2} c_i - x_i s_i``."""
    x = x.float()
    cos = cos.float()
    sin = sin.float()
    half = x.shape[-1] // 2
    x1 = x[..., :half]
    x2 = x[..., half:]
    return torch.cat([x1 * cos + x2 * sin, x2 * cos - x1 * sin], dim=-1)


def _kv_head(h: int, hq: int, hkv: int) -> int:
    # dominus_ultra.py:168
    return h // (hq // hkv)


def prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int] = None,
    heads: Optional[Iterable[Tuple[int, int]]] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal fused-RoPE prefill in fp32: returns ``(out fp32 [B,Hq,T,D], lse fp32 [B,Hq,T])``.

    ``out`` follows ``test_dominus.py:133-137`` (SDPA, ``is_causal=True``); ``lse`` follows
    ``gpu_evidence.py:277-281`` (natural-log ``logsumexp`` of the causally masked, scaled
    scores). ``heads`` optionally restricts the work to a list of ``(b, h)`` pairs; rows of
    other heads are left as NaN.
    """
    B, Hq, T, D = q.shape
    Hkv = num_kv_heads if num_kv_heads is not None else Hq
    scale = 1.0 / math.sqrt(D)
    cos_t = cos[:T].float()
    sin_t = sin[:T].float()
    out = torch.full((B, Hq, T, D), float("nan"), dtype=torch.float32)
    lse = torch.full((B, Hq, T), float("nan"), dtype=torch.float32)
    mask = torch.ones((T, T), dtype=torch.bool).triu(1)
    pairs = list(heads) if heads is not None else [(b, h) for b in range(B) for h in range(Hq)]
    cache = {}
    for b, h in pairs:
        kvh = _kv_head(h, Hq, Hkv)
        key = (b, kvh)
        if key not in cache:
            cache.clear()
            cache[key] = (
                apply_rope(k[b, kvh].cpu(), cos_t, sin_t),
                v[b, kvh].cpu().float(),
            )
        kr, vf = cache[key]
        qr = apply_rope(q[b, h].cpu(), cos_t, sin_t)
        out[b, h] = F.scaled_dot_product_attention(
            qr[None, None], kr[None, None], vf[None, None], is_causal=True
        )[0, 0]
        scores = (qr @ kr.transpose(0, 1)) * scale
        lse[b, h] = torch.logsumexp(scores.masked_fill(mask, float("-inf")), dim=-1)
    return out, lse


def prefill_block(
    q: torch.Tensor,
    k_rot: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    q_row0: int,
    tq: int,
    tk: int,
    causal: bool,
    pos_split: int,
    pos_off0: int,
    pos_off1: int,
    num_kv_heads: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """One block of a context-parallel prefill in fp32: ``(out [B,Hq,tq,D], lse [B,Hq,tq])``.

    Not in the reference (single-GPU); the same mathematics as ``prefill`` restricted to query
    rows ``[q_row0, q_row0 + tq)`` of ``q`` — row ``t`` rotated at ``pos_off0 + t`` below
    ``pos_split`` and ``pos_off1 + (t - pos_split)`` from it — against keys ``[0, tk)`` of
    ``k_rot`` (already rotated at their positions) and ``v``. ``causal``: key ``j`` visible to
    row ``t`` iff ``j <= t``; otherwise all keys are visible.
    """
    B, Hq, T, D = q.shape
    Hkv = num_kv_heads if num_kv_heads is not None else Hq
    scale = 1.0 / math.sqrt(D)
    rows = torch.arange(q_row0, q_row0 + tq)
    pos = torch.where(rows < pos_split, pos_off0 + rows, pos_off1 + (rows - pos_split))
    qr = apply_rope(q[:, :, q_row0 : q_row0 + tq].cpu(), cos[pos], sin[pos])
    kr = k_rot[:, :, :tk].cpu().float()
    vf = v[:, :, :tk].cpu().float()
    out = torch.empty((B, Hq, tq, D), dtype=torch.float32)
    lse = torch.empty((B, Hq, tq), dtype=torch.float32)
    mask = (torch.arange(tk)[None, :] > rows[:, None]) if causal else None
    for h in range(Hq):
        kvh = _kv_head(h, Hq, Hkv)
        sc = torch.einsum("btd,bjd->btj", qr[:, h], kr[:, kvh]) * scale
        if mask is not None:
            sc = sc.masked_fill(mask, float("-inf"))
        l = torch.logsumexp(sc, dim=-1)
        out[:, h] = torch.einsum("btj,bjd->btd", torch.exp(sc - l[..., None]), vf[:, kvh])
        lse[:, h] = l
    return out, lse


def prefill_rows(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int],
    b: int,
    h: int,
    rows: Sequence[int],
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact oracle for selected query rows of one ``(b, h)`` at sizes too large for ``prefill``.

    Causal row ``i`` depends only on keys ``0..i``, so each sampled row is computed against its
    own key prefix: this is the same arithmetic as ``prefill`` restricted to those rows.
    Returns ``(out fp32 [len(rows), D], lse fp32 [len(rows)])``.
    """
    _, Hq, T, D = q.shape
    Hkv = num_kv_heads if num_kv_heads is not None else Hq
    kvh = _kv_head(h, Hq, Hkv)
    scale = 1.0 / math.sqrt(D)
    rows_t = torch.as_tensor(list(rows), dtype=torch.long)
    top = int(rows_t.max().item()) + 1
    kr = apply_rope(k[b, kvh, :top].cpu(), cos[:top], sin[:top])
    vf = v[b, kvh, :top].cpu().float()
    qr = apply_rope(q[b, h, rows_t].cpu(), cos[rows_t], sin[rows_t])
    scores = (qr @ kr.transpose(0, 1)) * scale
    keep = torch.arange(top)[None, :] <= rows_t[:, None]
    scores = scores.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    p = torch.exp(scores - lse[:, None])
    return p @ vf, lse


def decode_partial(
    q_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int] = None,
    q_pos: Optional[int] = None,
    kv_pos_offset: int = 0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Attention of one new token over a (shard of a) KV cache, in fp32.

    Query rotated at ``q_pos`` (default: the cache length, ``test_dominus.py:276-280``), key
    ``j`` of the shard rotated at ``kv_pos_offset + j`` (``test_dominus.py:272-274`` for offset
    0). No mask (``is_causal=False``, ``test_dominus.py:283-285``). Returns
    ``(out fp32 [B,Hq,D], lse fp32 [B,Hq])`` with ``out`` normalised over this shard only.
    """
    B, Hq, _, D = q_new.shape
    L = k_cache.shape[2]
    Hkv = num_kv_heads if num_kv_heads is not None else Hq
    qp = L if q_pos is None else q_pos
    scale = 1.0 / math.sqrt(D)
    group = Hq // Hkv
    k_rot = apply_rope(
        k_cache.cpu(), cos[kv_pos_offset : kv_pos_offset + L], sin[kv_pos_offset : kv_pos_offset + L]
    )  # [B,Hkv,L,D]
    q_rot = apply_rope(q_new.cpu(), cos[qp : qp + 1], sin[qp : qp + 1])[:, :, 0]  # [B,Hq,D]
    vf = v_cache.cpu().float()
    out = torch.empty((B, Hq, D), dtype=torch.float32)
    lse = torch.empty((B, Hq), dtype=torch.float32)
    for kvh in range(Hkv):
        qg = q_rot[:, kvh * group : (kvh + 1) * group]  # [B,G,D]
        s = torch.einsum("bgd,bld->bgl", qg, k_rot[:, kvh]) * scale
        l = torch.logsumexp(s, dim=-1)
        p = torch.exp(s - l[..., None])
        out[:, kvh * group : (kvh + 1) * group] = torch.einsum("bgl,bld->bgd", p, vf[:, kvh])
        lse[:, kvh * group : (kvh + 1) * group] = l
    return out, lse


def decode(
    q_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int] = None,
) -> torch.Tensor:
    """Reference decode output, fp32 ``[B,Hq,1,D]`` (``test_dominus.py:270-285``).

    Uses SDPA exactly as the reference test does, with GQA by ``repeat_interleave``.
    """
    B, Hq, _, D = q_new.shape
    L = k_cache.shape[2]
    Hkv = num_kv_heads if num_kv_heads is not None else Hq
    group = Hq // Hkv
    k_rot = apply_rope(k_cache.cpu(), cos[:L], sin[:L]).repeat_interleave(group, dim=1)
    q_rot = apply_rope(q_new.cpu(), cos[L : L + 1], sin[L : L + 1])
    vf = v_cache.cpu().float().repeat_interleave(group, dim=1)
    return F.scaled_dot_product_attention(q_rot, k_rot, vf, is_causal=False)


def decode_kvcache(
    q_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    cache_seqlens: Sequence[int],
    k_new: Optional[torch.Tensor] = None,
    v_new: Optional[torch.Tensor] = None,
    num_kv_heads: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One generation step over a KV cache with per-sequence lengths, in fp32.

    Sequence ``b`` holds ``s_b = cache_seqlens[b]`` tokens. With ``k_new`` / ``v_new``
    (``[B,Hkv,1,D]``) they are first written to row ``s_b`` of copies of the caches and the
    query attends to keys ``0..s_b``; otherwise to keys ``0..s_b-1``. The query rotates at
    position ``s_b`` and key ``j`` at ``j``: the reference decode (``test_dominus.py:270-285``)
    of each sequence over its own prefix, with the query position fixed at ``s_b``. A sequence
    with no keys gives zeros. Returns ``(out fp32 [B,Hq,1,D], k_cache', v_cache')``.
    """
    B, Hq, _, D = q_new.shape
    Hkv = num_kv_heads if num_kv_heads is not None else Hq
    kc = k_cache.cpu().clone()
    vc = v_cache.cpu().clone()
    out = torch.zeros((B, Hq, 1, D), dtype=torch.float32)
    for b in range(B):
        s_b = int(cache_seqlens[b])
        n = s_b
        if k_new is not None:
            kc[b, :, s_b] = k_new.cpu()[b, :, 0]
            vc[b, :, s_b] = v_new.cpu()[b, :, 0]
            n = s_b + 1
        if n == 0:
            continue
        o, _ = decode_partial(
            q_new[b : b + 1], kc[b : b + 1, :, :n], vc[b : b + 1, :, :n], cos, sin,
            num_kv_heads=Hkv, q_pos=s_b, kv_pos_offset=0,
        )
        out[b, :, 0] = o[0]
    return out, kc, vc


def merge_partials(
    outs: Sequence[torch.Tensor], lses: Sequence[torch.Tensor]
) -> Tuple[torch.Tensor, torch.Tensor]:
    """LSE-weighted merge of per-shard decode partials.

    ``lse = logsumexp_r lse_r`` and ``out = sum_r exp(lse_r - lse) * out_r``; shards with
    ``lse_r = -inf`` (no keys) contribute nothing.
    """
    lse_stack = torch.stack([x.float() for x in lses], dim=0)
    out_stack = torch.stack([x.float() for x in outs], dim=0)
    lse = torch.logsumexp(lse_stack, dim=0)
    w = torch.exp(lse_stack - lse[None])
    w = torch.nan_to_num(w, nan=0.0)
    return (w[..., None] * out_stack).sum(dim=0), lse
