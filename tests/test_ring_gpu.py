"""Parity of the context-parallel (ring) prefill with the fp32 oracle (GPU).

Gate: out max-abs <= 2e-2, LSE <= 1e-3 on unscaled N(0,1) inputs. Covers the two-segment key
rotation, the block kernel's forms (a query-row window against a ragged key range at
two-segment positions, the causal block, the overwrite and LSE-merge epilogues and rows left
untouched outside the window), a whole ring emulated on one GPU (every rank's schedule run
against the other ranks' buffers) compared with the unsharded prefill, and the NCCL ring on two
GPUs when they are visible.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from _helpers import LSE_TOL, OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominusultra_b200 import precompute_rope_cos_sin, ring

pytestmark = pytest.mark.gpu


def _positions(n, split, off0, off1):
    t = torch.arange(n)
    return torch.where(t < split, off0 + t, off1 + (t - split))


def test_rotate_keys_at_zigzag_positions(cuda_device):
    world, rank, tc, D = 4, 1, 100, 128
    k = randn((1, 2, 2 * tc, D), 3)
    cos, sin = precompute_rope_cos_sin(2 * world * tc, D, "cpu", torch.bfloat16, 5e5)
    out = ring.rotate_keys(k.cuda(), cos.cuda(), sin.cuda(), rank, world)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    pos = _positions(2 * tc, *ring.zigzag_positions(rank, world, tc))
    ref = oracle.apply_rope(k, cos[pos], sin[pos])
    err = (out.float().cpu() - ref).abs()
    assert (err <= 2.0 ** -10 * ref.abs() + 1e-6).all(), err.max().item()


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_block_window_ragged_keys_and_merge(cuda_device, D, dtype):
    B, Hq, Hkv, T, Tkv = 2, 4, 2, 384, 300
    q = randn((B, Hq, T, D), 10, dtype)
    cos, sin = precompute_rope_cos_sin(4096, D, "cpu", dtype, 1e4)
    kpos = 1000 + torch.arange(Tkv)
    k1 = oracle.apply_rope(randn((B, Hkv, Tkv, D), 11, dtype), cos[kpos], sin[kpos]).half()
    v1 = randn((B, Hkv, Tkv, D), 12, dtype)
    k2 = oracle.apply_rope(randn((B, Hkv, Tkv, D), 13, dtype), cos[kpos], sin[kpos]).half()
    v2 = randn((B, Hkv, Tkv, D), 14, dtype)
    qd = q.cuda()
    cd, sd = cos.cuda(), sin.cuda()
    out = torch.full((B, Hq, T, D), 7.0, dtype=dtype, device="cuda")
    lse = torch.full((B, Hq, T), 7.0, device="cuda")
    acc_o = torch.full((B, Hq, T, D), 7.0, device="cuda")
    acc_lse = torch.full((B, Hq, T), 7.0, device="cuda")
    pos = (200, 2000, 50)  # rows < 200 at 2000 + t, rows >= 200 at 50 + (t - 200)
    r0, tq, tk = 130, 200, 250
    blk1 = ring.RingBlock(0, 0, r0, tq, tk, False, 1)
    blk2 = ring.RingBlock(1, 0, r0, tq, Tkv, False, 2)
    ring.prefill_block(qd, k1.cuda(), v1.cuda(), cd, sd, out, lse, acc_o, acc_lse, blk1, pos, Hkv)
    torch.cuda.synchronize()
    o1, l1 = oracle.prefill_block(q, k1, v1, cos, sin, r0, tq, tk, False, *pos, num_kv_heads=Hkv)
    rows = slice(r0, r0 + tq)
    assert max_abs(out[:, :, rows], o1) <= OUT_TOL
    assert max_abs(lse[:, :, rows], l1) <= LSE_TOL
    assert max_abs(acc_o[:, :, rows], o1) <= OUT_TOL and max_abs(acc_lse[:, :, rows], l1) <= LSE_TOL
    for t in (out, lse, acc_o, acc_lse):  # rows outside the window untouched
        assert (t[:, :, :r0].float() == 7.0).all() and (t[:, :, r0 + tq:].float() == 7.0).all()
    ring.prefill_block(qd, k2.cuda(), v2.cuda(), cd, sd, out, lse, acc_o, acc_lse, blk2, pos, Hkv)
    torch.cuda.synchronize()
    o2, l2 = oracle.prefill_block(q, k2, v2, cos, sin, r0, tq, Tkv, False, *pos, num_kv_heads=Hkv)
    om, lm = oracle.merge_partials([o1, o2], [l1, l2])
    assert max_abs(out[:, :, rows], om) <= OUT_TOL and max_abs(lse[:, :, rows], lm) <= LSE_TOL
    assert max_abs(acc_o[:, :, rows], om) <= OUT_TOL
    assert_no_device_timeouts()


def test_causal_block_at_two_segment_positions(cuda_device):
    B, Hq, Hkv, T, D = 1, 8, 2, 512, 128
    dtype = torch.bfloat16
    q = randn((B, Hq, T, D), 20, dtype)
    k = randn((B, Hkv, T, D), 21, dtype)
    v = randn((B, Hkv, T, D), 22, dtype)
    cos, sin = precompute_rope_cos_sin(8192, D, "cpu", dtype, 5e5)
    world, rank = 8, 3
    tc = T // 2
    pos = ring.zigzag_positions(rank, world, tc)
    k_rot = ring.rotate_keys(k.cuda(), cos.cuda(), sin.cuda(), rank, world)
    out = torch.empty((B, Hq, T, D), dtype=dtype, device="cuda")
    lse = torch.empty((B, Hq, T), device="cuda")
    acc_o = torch.empty((B, Hq, T, D), device="cuda")
    acc_lse = torch.empty((B, Hq, T), device="cuda")
    blk = ring.ring_schedule(rank, world, tc)[0]
    assert blk.causal and blk.acc_mode == 1
    ring.prefill_block(q.cuda(), k_rot, v.cuda(), cos.cuda(), sin.cuda(), out, lse, acc_o,
                       acc_lse, blk, pos, Hkv)
    torch.cuda.synchronize()
    o, l = oracle.prefill_block(q, k_rot.cpu(), v, cos, sin, 0, T, T, True, *pos, num_kv_heads=Hkv)
    assert max_abs(out, o) <= OUT_TOL and max_abs(lse, l) <= LSE_TOL
    assert_no_device_timeouts()


@pytest.mark.parametrize("world,tc,D,Hq,Hkv", [(4, 256, 128, 8, 2), (3, 200, 64, 4, 4), (2, 640, 128, 4, 1)])
def test_ring_emulated_on_one_gpu(cuda_device, world, tc, D, Hq, Hkv):
    """Every rank's schedule, run against the other ranks' buffers on one GPU, assembles the
    unsharded causal prefill."""
    B, S = 1, 2 * world * tc
    dtype = torch.bfloat16
    q = randn((B, Hq, S, D), 30, dtype)
    k = randn((B, Hkv, S, D), 31, dtype)
    v = randn((B, Hkv, S, D), 32, dtype)
    cos, sin = precompute_rope_cos_sin(S, D, "cpu", dtype, 5e5)
    cd, sd = cos.cuda(), sin.cuda()
    qs = [ring.zigzag_shard(q, r, world).cuda() for r in range(world)]
    ks = [ring.rotate_keys(ring.zigzag_shard(k, r, world).cuda(), cd, sd, r, world)
          for r in range(world)]
    vs = [ring.zigzag_shard(v, r, world).cuda() for r in range(world)]
    outs, lses = [], []
    for r in range(world):
        out = torch.empty_like(qs[r])
        lse = torch.empty((B, Hq, 2 * tc), device="cuda")
        acc_o = torch.empty((B, Hq, 2 * tc, D), device="cuda")
        acc_lse = torch.empty_like(lse)
        pos = ring.zigzag_positions(r, world, tc)
        for blk in ring.ring_schedule(r, world, tc):
            ring.prefill_block(qs[r], ks[blk.src], vs[blk.src], cd, sd, out, lse, acc_o, acc_lse,
                               blk, pos, Hkv)
        outs.append(out.cpu())
        lses.append(lse.cpu())
    torch.cuda.synchronize()
    ref_o, ref_l = oracle.prefill(q, k, v, cos, sin, Hkv)
    assert max_abs(ring.zigzag_unshard(outs), ref_o) <= OUT_TOL
    assert max_abs(ring.zigzag_unshard(lses), ref_l) <= LSE_TOL
    assert_no_device_timeouts()


def test_ring_emulated_eight_ranks_long_context_sampled_rows(cuda_device):
    """The eight-rank ring of the Llama-3-8B-shaped layer's length (S = 32768, D128, base 5e5,
    four query heads on one KV head), emulated on one GPU, checked on sampled rows of the
    assembled output (each an exact oracle comparison: causal row i depends only on keys <= i)."""
    world, B, Hq, Hkv, S, D = 8, 1, 4, 1, 32768, 128
    tc = S // (2 * world)
    dtype = torch.bfloat16
    q = randn((B, Hq, S, D), 600, dtype)
    k = randn((B, Hkv, S, D), 601, dtype)
    v = randn((B, Hkv, S, D), 602, dtype)
    cos, sin = precompute_rope_cos_sin(S, D, "cpu", dtype, 500000.0)
    cd, sd = cos.cuda(), sin.cuda()
    qs = [ring.zigzag_shard(q, r, world).cuda() for r in range(world)]
    ks = [ring.rotate_keys(ring.zigzag_shard(k, r, world).cuda(), cd, sd, r, world)
          for r in range(world)]
    vs = [ring.zigzag_shard(v, r, world).cuda() for r in range(world)]
    outs, lses = [], []
    acc_o = torch.empty((B, Hq, 2 * tc, D), device="cuda")
    acc_lse = torch.empty((B, Hq, 2 * tc), device="cuda")
    for r in range(world):
        out = torch.empty_like(qs[r])
        lse = torch.empty((B, Hq, 2 * tc), device="cuda")
        pos = ring.zigzag_positions(r, world, tc)
        for blk in ring.ring_schedule(r, world, tc):
            ring.prefill_block(qs[r], ks[blk.src], vs[blk.src], cd, sd, out, lse, acc_o, acc_lse,
                               blk, pos, Hkv)
        outs.append(out.cpu())
        lses.append(lse.cpu())
    torch.cuda.synchronize()
    out, lse = ring.zigzag_unshard(outs), ring.zigzag_unshard(lses)
    g = torch.Generator().manual_seed(603)
    # rows at every chunk boundary of the zigzag layout, plus random ones
    edges = [c * tc + d for c in range(2 * world) for d in (0, tc - 1)]
    rows = sorted(set(edges + torch.randint(0, S, (192,), generator=g).tolist()))
    for h in (0, 3):
        ro, rl = oracle.prefill_rows(q, k, v, cos, sin, Hkv, 0, h, rows)
        assert max_abs(out[0, h, rows], ro) <= OUT_TOL
        assert max_abs(lse[0, h, rows], rl) <= LSE_TOL
    assert torch.isfinite(out.float()).all()
    assert_no_device_timeouts()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q_out):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(5)
        B, Hq, Hkv, S, D = 1, 8, 2, 4096, 128
        q = torch.randn(B, Hq, S, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
        cos, sin = precompute_rope_cos_sin(S, D, "cpu", torch.bfloat16, 5e5)
        dev = torch.device("cuda", rank)
        out, lse = ring.ring_prefill(ring.zigzag_shard(q, rank, world).to(dev),
                                     ring.zigzag_shard(k, rank, world).to(dev),
                                     ring.zigzag_shard(v, rank, world).to(dev),
                                     cos.to(dev), sin.to(dev), Hkv)
        torch.cuda.synchronize()
        ref_o, ref_l = oracle.prefill(q, k, v, cos, sin, Hkv)
        o_err = (out.float().cpu() - ring.zigzag_shard(ref_o, rank, world)).abs().max().item()
        l_err = (lse.cpu() - ring.zigzag_shard(ref_l, rank, world)).abs().max().item()
        q_out.put((rank, o_err, l_err))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ring_prefill_nccl_two_gpus():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, o_err, l_err in results:
        assert o_err <= OUT_TOL and l_err <= LSE_TOL, (rank, o_err, l_err)
