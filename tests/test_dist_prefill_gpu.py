"""Prefill sharded over (batch, kv-head) units, every rank's shard run in turn on one GPU.

``dist.sharded_prefill`` gives rank r of N a contiguous range of units (one KV head and the
query heads that read it, ``kv_h = h // (Hq / Hkv)`` as in the reference's GQA map) and runs one
prefill on that slab with no communication. Here the ranks of N = 2, 4 and 8 (and an uneven 3)
are emulated one after the other on one GPU: each rank's shard must equal the matching slab of
the unsharded prefill bit for bit (the same kernels on the same rows), and the reassembled
output is checked against the oracle. The Llama-3-8B-shaped layer (B4 H32 Hkv8 S32768 D128,
RoPE base 5e5) is checked on sampled rows (causal row i depends only on keys <= i, so each
sampled row is an exact oracle comparison); the multi-query case (B2 H32 Hkv1 S1024, fewer
units than ranks: each KV group's query heads are split into chunks and the KV head
replicated) against the full oracle.
"""

import pytest
import torch

import oracle
from _helpers import LSE_TOL, OUT_TOL, assert_no_device_timeouts, max_abs
from dominusultra_b200 import dist as ddist
from dominusultra_b200 import dominus_ultra_prefill, precompute_rope_cos_sin

pytestmark = pytest.mark.gpu


def _reassemble(q, k, v, cos, sin, Hkv, world):
    """Run every rank's shard in turn; return the outputs laid out as [units, heads, T, D]."""
    B, Hq, T, D = q.shape
    plan = ddist.plan_prefill(B, Hq, Hkv, world)
    out = torch.empty(plan.n_units, plan.heads_per_unit, T, D, dtype=q.dtype, device=q.device)
    lse = torch.empty(plan.n_units, plan.heads_per_unit, T, dtype=torch.float32, device=q.device)
    covered = 0
    for rank in range(world):
        o_s, l_s, (u0, u1), p = ddist.sharded_prefill(q, k, v, cos, sin, Hkv, rank, world)
        assert p == plan
        if u1 > u0:
            out[u0:u1] = o_s
            lse[u0:u1] = l_s
        covered += u1 - u0
    assert covered == plan.n_units
    return out.reshape(B, Hq, T, D), lse.reshape(B, Hq, T)


def test_sharded_prefill_llama_shape_emulated_ranks(cuda_device):
    B, Hq, Hkv, T, D = 4, 32, 8, 32768, 128
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(2024)
    q = torch.randn(B, Hq, T, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    cos, sin = precompute_rope_cos_sin(T, D, dev, torch.bfloat16, 500000.0)
    full_o, full_l = dominus_ultra_prefill(q, k, v, cos, sin, Hkv)
    for world in (2, 3, 4, 8):
        plan = ddist.plan_prefill(B, Hq, Hkv, world)
        assert plan.chunks == 1 and plan.n_units == B * Hkv
        o, l = _reassemble(q, k, v, cos, sin, Hkv, world)
        torch.cuda.synchronize()
        assert torch.equal(o, full_o) and torch.equal(l, full_l), world
        del o, l
    # One sampled (batch, query head) per rank at eight ranks, against the oracle.
    cpu = {n: t.cpu() for n, t in (("cos", cos), ("sin", sin))}
    gen = torch.Generator().manual_seed(2025)
    rows = sorted(set(list(range(64)) + list(range(T - 64, T)) +
                      torch.randint(0, T, (96,), generator=gen).tolist()))
    plan = ddist.plan_prefill(B, Hq, Hkv, 8)
    for rank in range(8):
        u0, _ = ddist.shard_range(plan.n_units, 8, rank)
        b, kvh = divmod(u0, Hkv)
        h = kvh * (Hq // Hkv) + rank % (Hq // Hkv)
        top = rows[-1] + 1
        qs = q[b:b + 1, h:h + 1].cpu()
        ks, vs = k[b:b + 1, kvh:kvh + 1, :top].cpu(), v[b:b + 1, kvh:kvh + 1, :top].cpu()
        ro, rl = oracle.prefill_rows(qs, ks, vs, cpu["cos"], cpu["sin"], 1, 0, 0, rows)
        assert max_abs(full_o[b, h, rows], ro) <= OUT_TOL, rank
        assert max_abs(full_l[b, h, rows], rl) <= LSE_TOL, rank
    assert torch.isfinite(full_o.float()).all()
    assert_no_device_timeouts()


@pytest.mark.parametrize("Hkv,world", [(1, 2), (1, 8), (8, 3), (8, 8)])
def test_sharded_prefill_gqa_mqa_emulated_ranks(cuda_device, Hkv, world):
    """P3 shapes: B2 H32 S1024 D64 with Hkv 8 (16 units) and Hkv 1 (2 units: query-head chunks
    with the KV head replicated)."""
    B, Hq, T, D = 2, 32, 1024, 64
    g = torch.Generator().manual_seed(77 + Hkv + world)
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", torch.bfloat16)
    dq, dk, dv, dc, ds = (t.cuda() for t in (q, k, v, cos, sin))
    plan = ddist.plan_prefill(B, Hq, Hkv, world)
    if B * Hkv < world:
        assert plan.chunks > 1 and plan.n_units >= world
    o, l = _reassemble(dq, dk, dv, dc, ds, Hkv, world)
    full_o, full_l = dominus_ultra_prefill(dq, dk, dv, dc, ds, Hkv)
    torch.cuda.synchronize()
    assert torch.equal(o, full_o) and torch.equal(l, full_l)
    ro, rl = oracle.prefill(q, k, v, cos, sin, Hkv)
    assert max_abs(o, ro) <= OUT_TOL and max_abs(l, rl) <= LSE_TOL
    assert_no_device_timeouts()
