"""Host logic of the multi-GPU path on CPU ranks (gloo, world_size 2).

The sharded long-context decode (KV sequence split across ranks, partials packed into one
buffer, one all-gather, LSE merge) and the communication-free (batch, kv-head) prefill
sharding are run with the oracle as the compute function, and compared with the unsharded
oracle. The GPU kernels behind the same functions are covered by the GPU tests.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from dominusultra_b200 import dist as ddist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_partial(q, k, v, cos, sin, hkv, total_len, off):
    return oracle.decode_partial(q, k, v, cos, sin, hkv, q_pos=total_len, kv_pos_offset=off)


def _oracle_merge(o_all, lse_all, dtype):
    out, lse = oracle.merge_partials(list(o_all), list(lse_all))
    return out.to(dtype), lse


def _oracle_prefill(q, k, v, cos, sin, hkv):
    return oracle.prefill(q, k, v, cos, sin, hkv)


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(99)
        # ---- sharded decode over the KV sequence
        B, Hq, Hkv, L, D = 2, 8, 2, 333, 64
        q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
        cos, sin = oracle.precompute_rope_cos_sin(L + 1, D, torch.bfloat16)
        a, b = ddist.kv_shard(L, world, rank)
        out = ddist.sharded_decode(q, k[:, :, a:b], v[:, :, a:b], cos, sin, Hkv, L, a,
                                   partial_fn=_oracle_partial, merge_fn=_oracle_merge)
        full = oracle.decode(q, k, v, cos, sin, Hkv).to(torch.bfloat16)
        dec_err = (out.float() - full.float()).abs().max().item()

        # ---- communication-free prefill sharding (GQA), outputs gathered only for checking
        B, Hq, Hkv, T, D = 2, 4, 2, 40, 32
        q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
        cos, sin = oracle.precompute_rope_cos_sin(T, D, torch.bfloat16)
        out_s, _, (u0, u1), plan = ddist.sharded_prefill(q, k, v, cos, sin, Hkv, rank, world,
                                                         prefill_fn=_oracle_prefill)
        pieces = ddist.gather_prefill_units(out_s, plan, world)
        full_out = torch.cat([p for p in pieces if p.numel()], 0).reshape(B, Hq, T, D)
        ref, _ = oracle.prefill(q, k, v, cos, sin, Hkv)
        pre_err = (full_out - ref).abs().max().item()
        result_q.put((rank, dec_err, pre_err, (u0, u1)))
    finally:
        dist.destroy_process_group()


def test_sharded_decode_and_prefill_gloo_world2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    for rank, dec_err, pre_err, _ in results:
        assert dec_err <= 2e-2, (rank, dec_err)  # bf16 output rounding only
        assert pre_err <= 1e-6, (rank, pre_err)
    assert results[0][3] == (0, 2) and results[1][3] == (2, 4)


def test_shard_range_covers_exactly():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [ddist.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("B,Hq,Hkv,world,chunks", [
    (2, 32, 32, 8, 1), (2, 32, 8, 8, 1), (2, 32, 1, 8, 4), (2, 32, 1, 2, 1), (4, 32, 8, 8, 1),
    (1, 8, 1, 8, 8),
])
def test_prefill_plan_units(B, Hq, Hkv, world, chunks):
    plan = ddist.plan_prefill(B, Hq, Hkv, world)
    assert plan.chunks == chunks
    assert plan.n_units >= min(world, B * Hq)
    assert plan.heads_per_unit * plan.chunks == Hq // Hkv


def test_mqa_prefill_shards_replicate_kv_head():
    B, Hq, Hkv, T, D = 2, 8, 1, 16, 16
    q = torch.randn(B, Hq, T, D)
    k = torch.randn(B, Hkv, T, D)
    v = torch.randn(B, Hkv, T, D)
    world = 8
    plan = ddist.plan_prefill(B, Hq, Hkv, world)
    assert plan.chunks == 4 and plan.n_units == 8
    seen = []
    for r in range(world):
        qs, ks, vs, (u0, u1) = ddist.prefill_shard_inputs(plan, q, k, v, r, world)
        assert qs.shape == (u1 - u0, 2, T, D) and ks.shape[0] == u1 - u0
        for i, u in enumerate(range(u0, u1)):
            b = plan.unit_kv_index(u) // Hkv
            assert torch.equal(ks[i, 0], k[b, 0])
            seen.append(qs[i])
    assert torch.equal(torch.stack(seen).reshape(B, Hq, T, D), q)


def test_pack_unpack_roundtrip():
    o = torch.randn(2, 3, 8)
    l = torch.randn(2, 3)
    buf = ddist.pack_partial(o, l)
    g = torch.cat([buf, buf * 2])
    oo, ll = ddist.unpack_gathered(g, 2, (2, 3), 8)
    assert torch.equal(oo[0], o) and torch.equal(ll[1], l * 2)
