"""Multi-GPU sharding of the attention hot path (one process per GPU, torch.distributed).

The reference has no multi-GPU code; this module follows the partitioning the path allows:

* **Prefill** shards over independent ``(batch, kv-head)`` units with no communication. A rank's
  contiguous range of units is one contiguous slab of q (``[B*Hkv, G, T, D]`` view) and of k/v
  (``[B*Hkv, 1, T, D]``), so the rank runs one ``dominus_ultra_prefill`` on its slab. When there
  are fewer units than ranks (MQA), the G query heads of each group are split into chunks and the
  group's single KV head is replicated to the ranks that share it.
* **Long-context decode** splits the KV *sequence* into contiguous shards. Each rank computes an
  fp32 partial ``(out, lse)`` for its shard at absolute key positions (``decode_partial``), the
  partials are packed into one ``[B*Hq*(D+1)]`` fp32 buffer and exchanged with a single
  ``all_gather_into_tensor`` (NCCL over NVLink), and each rank merges them by LSE
  (``merge_partials``). This is the only collective on the path.

  ``PeerExchange`` replaces that collective and the merge launch with one kernel over NVLink
  peer memory (``du_exchange_merge``): each rank stores its partial into every rank's exchange
  buffer (mapped once through CUDA IPC) and merges the world's partials as soon as they are in.

The compute functions are injectable so the host logic (unit ranges, packing, collective,
merge) is testable on CPU ranks with the gloo backend and the oracle.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Balanced contiguous split of ``n`` items: rank gets ``[start, end)`` (may be empty)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class PrefillPlan:
    """How a prefill of ``B x Hq`` query heads over ``Hkv`` KV heads is cut into units."""

    B: int
    Hq: int
    Hkv: int
    chunks: int  # query-head chunks per KV group (1 unless units < ranks)

    @property
    def group(self) -> int:
        return self.Hq // self.Hkv

    @property
    def heads_per_unit(self) -> int:
        return self.group // self.chunks

    @property
    def n_units(self) -> int:
        return self.B * self.Hkv * self.chunks

    def unit_kv_index(self, u: int) -> int:
        """Flattened ``b * Hkv + kvh`` of unit ``u``."""
        return u // self.chunks


def plan_prefill(B: int, Hq: int, Hkv: int, world: int) -> PrefillPlan:
    """Units are ``(b, kvh)``; if that gives fewer units than ranks, split each KV group's query
    heads into the smallest number of chunks (a divisor of the group size) that covers them."""
    if Hq % Hkv:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    G = Hq // Hkv
    chunks = 1
    if B * Hkv < world:
        for c in range(1, G + 1):
            if G % c == 0:
                chunks = c
                if B * Hkv * c >= world:
                    break
    return PrefillPlan(B, Hq, Hkv, chunks)


def prefill_shard_inputs(plan: PrefillPlan, q, k, v, rank: int, world: int):
    """Rank's slab: ``(q_s [U, Hpu, T, D], k_s [U', 1 or U, ...], v_s, (u0, u1))``.

    With ``chunks == 1`` the K/V slab is a view; otherwise the replicated KV head of each unit
    is gathered (one copy of that head per unit on this rank).
    """
    B, Hq, T, D = q.shape
    u0, u1 = shard_range(plan.n_units, world, rank)
    qs = q.reshape(plan.n_units, plan.heads_per_unit, T, D)[u0:u1]
    kv_k = k.reshape(B * plan.Hkv, 1, T, D)
    kv_v = v.reshape(B * plan.Hkv, 1, T, D)
    if plan.chunks == 1:
        return qs, kv_k[u0:u1], kv_v[u0:u1], (u0, u1)
    idx = torch.tensor([plan.unit_kv_index(u) for u in range(u0, u1)], dtype=torch.long,
                       device=k.device)
    return qs, kv_k.index_select(0, idx), kv_v.index_select(0, idx), (u0, u1)


def sharded_prefill(q, k, v, cos, sin, num_kv_heads: Optional[int], rank: int, world: int,
                    prefill_fn: Optional[Callable] = None):
    """This rank's share of a causal prefill: returns ``(out_s, lse_s, (u0, u1), plan)`` where
    ``out_s`` is ``[U, heads_per_unit, T, D]`` for units ``u0..u1-1``. No communication."""
    if prefill_fn is None:
        from .attention import dominus_ultra_prefill as prefill_fn
    Hkv = num_kv_heads if num_kv_heads is not None else q.shape[1]
    plan = plan_prefill(q.shape[0], q.shape[1], Hkv, world)
    qs, ks, vs, rng = prefill_shard_inputs(plan, q, k, v, rank, world)
    if qs.shape[0] == 0:
        return qs.new_empty(qs.shape), None, rng, plan
    out, lse = prefill_fn(qs.contiguous(), ks.contiguous(), vs.contiguous(), cos, sin, 1)
    return out, lse, rng, plan


def kv_shard(L: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous KV-sequence shard ``[start, end)`` of rank ``rank``."""
    return shard_range(L, world, rank)


def pack_partial(out_f32: torch.Tensor, lse_f32: torch.Tensor) -> torch.Tensor:
    """``[rows*D]`` out followed by ``[rows]`` lse in one fp32 buffer (one collective)."""
    return torch.cat([out_f32.reshape(-1), lse_f32.reshape(-1)])


def unpack_gathered(gathered: torch.Tensor, world: int, rows_shape, D: int):
    """Views ``(o [world, *rows, D], lse [world, *rows])`` into an all-gathered buffer."""
    rows = 1
    for s in rows_shape:
        rows *= s
    per = rows * (D + 1)
    g = gathered.reshape(world, per)
    o = g[:, : rows * D].reshape(world, *rows_shape, D)
    lse = g[:, rows * D:].reshape(world, *rows_shape)
    return o, lse


class PeerExchange:
    """Exchange buffers of the sequence-split decode, mapped on every rank of ``group`` (one
    node, one GPU per rank, at most 8 ranks) for ``rows`` partial rows of ``D`` values.

    Set-up is collective (every rank constructs it, in the same order as its other collectives):
    each rank allocates its buffer (``du_exchange_buffer_alloc``), the 64-byte CUDA IPC handles
    travel with ``all_gather_object``, and each rank opens the others'. ``merge`` then runs
    ``du_exchange_merge`` on the current stream. ``close`` (also collective) unmaps and frees.
    """

    def __init__(self, rows: int, D: int, group=None, device=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self._lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.D = rows, D
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        nbytes = int(self._lib.du_exchange_buffer_bytes(self.world, rows, D))
        if nbytes == 0:
            raise ValueError("peer exchange supports 1..8 ranks and D a multiple of 4")
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            _lib.check(self._lib.du_exchange_buffer_alloc(nbytes, ctypes.byref(own)), "du_exchange_buffer_alloc")
            handle = ctypes.create_string_buffer(64)
            _lib.check(self._lib.du_ipc_get_handle(own, handle), "du_ipc_get_handle")
            handles: list = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            ptrs = []
            self._opened = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(own.value)
                    continue
                peer = ctypes.c_void_p()
                _lib.check(self._lib.du_ipc_open_handle(ctypes.create_string_buffer(h, 64), ctypes.byref(peer)),
                           "du_ipc_open_handle")
                self._opened.append(peer.value)
                ptrs.append(peer.value)
        self._own = own.value
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)

    def merge(self, o_local: torch.Tensor, lse_local: torch.Tensor, out_dtype: torch.dtype,
              with_lse: bool = False):
        """Merge every rank's ``(o [*rows, D], lse [*rows])`` fp32 partial; returns ``out`` in
        ``out_dtype`` (and the merged lse with ``with_lse``) on every rank."""
        import ctypes

        from . import _lib
        from .attention import _dtype_code

        if self._own is None:
            raise RuntimeError("this PeerExchange is closed")
        if o_local.dtype != torch.float32 or lse_local.dtype != torch.float32:
            raise ValueError("partials must be float32")
        o2 = o_local.reshape(-1, self.D)
        l2 = lse_local.reshape(-1)
        if o2.shape[0] != self.rows or l2.shape[0] != self.rows or not (o2.is_contiguous() and l2.is_contiguous()):
            raise ValueError("partials must be contiguous [rows, D] / [rows] blocks of this exchange's rows")
        out = torch.empty(o_local.shape, dtype=out_dtype, device=o_local.device)
        lse = torch.empty(lse_local.shape, dtype=torch.float32, device=o_local.device) if with_lse else None
        st = ctypes.c_void_p(torch.cuda.current_stream(o_local.device).cuda_stream)
        rc = self._lib.du_exchange_merge(
            ctypes.c_void_p(o2.data_ptr()), ctypes.c_void_p(l2.data_ptr()), self._ptrs, self.world,
            self.rank, self.rows, self.D, ctypes.c_void_p(out.data_ptr()), _dtype_code(out_dtype),
            ctypes.c_void_p(lse.data_ptr()) if lse is not None else None, st)
        _lib.check(rc, "du_exchange_merge")
        return out, lse

    def close(self):
        """Collective: unmap the peers' buffers and free this rank's (after a barrier, so no
        rank frees a buffer another may still write)."""
        import torch.distributed as dist

        from . import _lib

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.check(self._lib.du_ipc_close_handle(p), "du_ipc_close_handle")
        self._opened = []
        dist.barrier(group=self.group)
        _lib.check(self._lib.du_exchange_buffer_free(self._own), "du_exchange_buffer_free")
        self._own = None


def sharded_decode(
    q_new: torch.Tensor,
    k_shard: torch.Tensor,
    v_shard: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_kv_heads: Optional[int],
    total_len: int,
    kv_pos_offset: int,
    group=None,
    partial_fn: Optional[Callable] = None,
    merge_fn: Optional[Callable] = None,
    exchange: Optional[PeerExchange] = None,
) -> torch.Tensor:
    """Decode over a KV sequence split across the ranks of ``group``.

    Each rank holds keys ``[kv_pos_offset, kv_pos_offset + L_shard)`` of a cache of
    ``total_len`` positions; the query sits at position ``total_len``. Returns the merged
    ``[B, Hq, 1, D]`` output (in q's dtype) on every rank.
    """
    import torch.distributed as dist

    if partial_fn is None:
        from .attention import decode_partial as partial_fn
    if merge_fn is None:
        from .attention import merge_partials as merge_fn
    world = dist.get_world_size(group)
    B, Hq, _, D = q_new.shape
    o, lse = partial_fn(q_new, k_shard, v_shard, cos, sin, num_kv_heads, total_len, kv_pos_offset)
    if exchange is not None:
        out, _ = exchange.merge(o, lse, q_new.dtype)
        return out.reshape(B, Hq, 1, D)
    send = pack_partial(o, lse)
    gathered = torch.empty(world * send.numel(), dtype=send.dtype, device=send.device)
    dist.all_gather_into_tensor(gathered, send, group=group)
    o_all, lse_all = unpack_gathered(gathered, world, (B, Hq), D)
    out, _ = merge_fn(o_all, lse_all, q_new.dtype)
    return out.reshape(B, Hq, 1, D)


def gather_prefill_units(out_s: torch.Tensor, plan: PrefillPlan, world: int, group=None) -> List[torch.Tensor]:
    """Collect every rank's unit outputs (for tests / callers that need the full tensor).
    Not part of the timed path, which is communication-free."""
    import torch.distributed as dist

    pieces = [None] * world
    dist.all_gather_object(pieces, out_s.cpu(), group=group)
    return pieces
