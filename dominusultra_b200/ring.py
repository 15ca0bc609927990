"""Context-parallel (ring) causal prefill across the ranks of a process group.

For sequences beyond one GPU (or batches with fewer (batch, kv-head) units than GPUs), the
sequence itself is split. It extends the single-GPU prefill (reference ``dominus_ultra.py:416-501``,
kernel ``:119-285``) to N ranks:

* **Zigzag sharding.** The sequence is cut into 2N chunks of ``Tc`` positions; rank r holds
  chunks ``r`` and ``2N-1-r``, concatenated along T (``zigzag_shard``). Under the causal mask
  every rank then has the same work at every ring step.
* **Keys rotated once.** Each rank rotates its own keys at their absolute positions into fp16
  (``du_rope_segments``: two position segments); the rotated keys and the raw values travel.
* **Ring.** Step 0 attends the rank's queries to its own keys (a causal block over the local
  2·Tc rows: with the chunks in position order, local causality is global causality). At step
  s the rank holds the keys of ``src = (r - s) mod N`` and attends, with no mask,
  - all its query rows to src's first chunk when ``src < r``;
  - its second query chunk to both of src's chunks when ``src > r``
  (every other chunk pair lies above the diagonal). Meanwhile the buffers move one rank on with
  NCCL point-to-point (``batch_isend_irecv``; no multicast), double-buffered.
* **Merge in the epilogue.** Each block (``du_prefill_block``) LSE-merges its rows into fp32
  accumulators and writes the merged output in the input dtype, so after the last step ``out``
  and ``lse`` are final with no extra pass.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch

from . import _lib
from .attention import (
    _OnDevice,
    _aligned,
    _dtype_code,
    _ptr,
    _stream,
    _validate_attention_tensors,
    _validate_head_dim,
    _validate_rope_tables,
)

__all__ = [
    "RingBlock",
    "zigzag_chunks",
    "zigzag_positions",
    "zigzag_shard",
    "zigzag_unshard",
    "ring_schedule",
    "rotate_keys",
    "prefill_block",
    "ring_prefill",
]


def zigzag_chunks(rank: int, world: int) -> Tuple[int, int]:
    """The two sequence chunks (of 2·world) that ``rank`` holds, in position order."""
    return rank, 2 * world - 1 - rank


def zigzag_positions(rank: int, world: int, tc: int) -> Tuple[int, int, int]:
    """(pos_split, pos_off0, pos_off1) of the rank's local rows: row t < tc sits at
    ``a·tc + t``, row t >= tc at ``b·tc + (t - tc)``."""
    a, b = zigzag_chunks(rank, world)
    return tc, a * tc, b * tc


def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """Rank ``rank``'s zigzag shard of ``x`` along ``dim`` (length divisible by 2·world)."""
    T = x.shape[dim]
    if T % (2 * world):
        raise ValueError(f"sequence length {T} is not divisible by 2 * world = {2 * world}")
    tc = T // (2 * world)
    a, b = zigzag_chunks(rank, world)
    return torch.cat([x.narrow(dim, a * tc, tc), x.narrow(dim, b * tc, tc)], dim).contiguous()


def zigzag_unshard(parts: List[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Inverse of ``zigzag_shard``: the full tensor from every rank's shard (rank order)."""
    world = len(parts)
    tc = parts[0].shape[dim] // 2
    chunks: List[Optional[torch.Tensor]] = [None] * (2 * world)
    for r, p in enumerate(parts):
        a, b = zigzag_chunks(r, world)
        chunks[a] = p.narrow(dim, 0, tc)
        chunks[b] = p.narrow(dim, tc, tc)
    return torch.cat(chunks, dim)


@dataclass(frozen=True)
class RingBlock:
    """One attention block of a ring step: query rows [q_row0, q_row0 + tq) of the local shard
    against keys [0, tk) of the buffer received from ``src``."""

    step: int
    src: int
    q_row0: int
    tq: int
    tk: int
    causal: bool
    acc_mode: int  # 1: first block of every row (overwrite the accumulators), 2: merge


def ring_schedule(rank: int, world: int, tc: int) -> List[RingBlock]:
    """The blocks rank ``rank`` computes, one per ring step (2·tc·tc key pairs per row pair at
    every step after the first, so the ranks stay in step)."""
    blocks = [RingBlock(0, rank, 0, 2 * tc, 2 * tc, True, 1)]
    for s in range(1, world):
        src = (rank - s) % world
        if src < rank:  # src's first chunk precedes both of ours; its second follows both
            blocks.append(RingBlock(s, src, 0, 2 * tc, tc, False, 2))
        else:  # both of src's chunks precede our second chunk and follow our first
            blocks.append(RingBlock(s, src, tc, tc, 2 * tc, False, 2))
    return blocks


def rotate_keys(k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rank: int,
                world: int) -> torch.Tensor:
    """The rank's keys ``[B, Hkv, 2·tc, D]`` rotated at their zigzag positions, as fp16
    (``du_rope_segments``)."""
    B, H, T2, D = k.shape
    split, off0, off1 = zigzag_positions(rank, world, T2 // 2)
    lib = _lib.load()
    k = _aligned(k.contiguous())
    out = torch.empty(k.shape, dtype=torch.float16, device=k.device)
    with _OnDevice(k.device):
        rc = lib.du_rope_segments(
            _ptr(k), _ptr(cos), _ptr(sin), _ptr(out), B, H, T2, D, _dtype_code(k.dtype),
            _lib.DU_DTYPE_F16, split, off0, off1, min(cos.shape[0], sin.shape[0]), 0,
            _stream(k.device),
        )
    _lib.check(rc, "du_rope_segments")
    return out


def prefill_block(q, k_rot, v, cos, sin, out, lse, acc_o, acc_lse, blk: RingBlock,
                  pos: Tuple[int, int, int], num_kv_heads: int) -> None:
    """Launch ``du_prefill_block`` for one ring block (tensors already validated, on one
    device, contiguous and 16-byte aligned)."""
    B, Hq, T, D = q.shape
    Tkv = k_rot.shape[2]
    lib = _lib.load()
    with _OnDevice(q.device):
        rc = lib.du_prefill_block(
            _ptr(q), _ptr(k_rot), _ptr(v), _ptr(cos), _ptr(sin), _ptr(out), _ptr(lse),
            _ptr(acc_o), _ptr(acc_lse), blk.acc_mode, B, Hq, num_kv_heads, T, Tkv, blk.q_row0,
            blk.tq, blk.tk, 1 if blk.causal else 0, pos[0], pos[1], pos[2], D,
            _dtype_code(q.dtype), 1.0 / (D**0.5), min(cos.shape[0], sin.shape[0]),
            _stream(q.device),
        )
    _lib.check(rc, "du_prefill_block")


def ring_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int] = None,
    group=None,
    rotate_fn: Optional[Callable] = None,
    block_fn: Optional[Callable] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal fused-RoPE prefill of a sequence zigzag-sharded over the ranks of ``group``.

    ``q [B, Hq, 2·tc, D]``, ``k, v [B, Hkv, 2·tc, D]``: this rank's ``zigzag_shard`` of the
    sequence (length ``2·world·tc``); ``cos, sin``: tables covering the whole sequence.
    Returns this rank's ``(out [B, Hq, 2·tc, D], lse [B, Hq, 2·tc])`` — the rows of the
    single-GPU ``dominus_ultra_prefill`` of the full sequence that the shard holds.
    ``rotate_fn`` / ``block_fn`` replace the CUDA key rotation / block launch (host tests).
    """
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
    else:  # no process group: a ring of one rank (the causal prefill of the local sequence)
        world, rank = 1, 0
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must be rank-4 tensors")
    B, Hq, T2, D = q.shape
    KvH = num_kv_heads if num_kv_heads is not None else Hq
    if KvH <= 0 or Hq % KvH != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if k.shape != (B, KvH, T2, D) or v.shape != (B, KvH, T2, D):
        raise ValueError("k and v must have shape [batch, num_kv_heads, seq_len, head_dim]")
    if T2 % 2:
        raise ValueError("a zigzag shard holds two chunks of equal length")
    tc = T2 // 2
    if block_fn is None:
        _validate_head_dim(D)
        if D > 128:
            raise ValueError("ring prefill supports head_dim up to 128")
        _validate_attention_tensors(q, k, v)
        _validate_rope_tables(cos, sin, 2 * world * tc, D, q.device, q.dtype)
        q, v = _aligned(q), _aligned(v)
        cos, sin = _aligned(cos), _aligned(sin)
    rotate_fn = rotate_fn or rotate_keys
    block_fn = block_fn or prefill_block
    pos = zigzag_positions(rank, world, tc)
    nxt_rank = (rank + 1) % world
    prv_rank = (rank - 1) % world
    if group is not None:
        nxt_rank = dist.get_global_rank(group, nxt_rank)
        prv_rank = dist.get_global_rank(group, prv_rank)

    cur = (rotate_fn(k, cos, sin, rank, world), v.contiguous())
    nxt = (torch.empty_like(cur[0]), torch.empty_like(cur[1]))
    out = torch.empty_like(q)
    lse = torch.empty((B, Hq, T2), dtype=torch.float32, device=q.device)
    acc_o = torch.empty((B, Hq, T2, D), dtype=torch.float32, device=q.device)
    acc_lse = torch.empty((B, Hq, T2), dtype=torch.float32, device=q.device)
    for blk in ring_schedule(rank, world, tc):
        reqs = []
        if blk.step < world - 1:
            # The transfer is queued after the previous block on this stream (the receive
            # overwrites the buffer that block read) and overlaps this block.
            ops = [dist.P2POp(dist.isend, t, nxt_rank, group) for t in cur]
            ops += [dist.P2POp(dist.irecv, t, prv_rank, group) for t in nxt]
            reqs = dist.batch_isend_irecv(ops)
        block_fn(q, cur[0], cur[1], cos, sin, out, lse, acc_o, acc_lse, blk, pos, KvH)
        for r in reqs:
            r.wait()
        cur, nxt = nxt, cur
    return out, lse
