"""Host logic of the context-parallel (ring) prefill on CPU.

The zigzag sharding, the ring schedule (every causal (query, key) pair exactly once, the same
work on every rank at every step) and the ring itself — K/V buffers passed with point-to-point
sends over gloo ranks, blocks LSE-merged into fp32 accumulators — run with the oracle as the
compute function and are compared with the unsharded oracle prefill. The CUDA block kernel
behind the same driver is covered by tests/test_ring_gpu.py.
"""

import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from dominusultra_b200 import _lib
from dominusultra_b200 import ring


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_zigzag_round_trip():
    x = torch.arange(2 * 3 * 24 * 2).reshape(2, 3, 24, 2)
    for world in (1, 2, 3, 4, 6, 12):
        parts = [ring.zigzag_shard(x, r, world) for r in range(world)]
        assert all(p.shape[2] == 24 // world for p in parts)
        assert torch.equal(ring.zigzag_unshard(parts), x)
    with pytest.raises(ValueError, match="divisible"):
        ring.zigzag_shard(x, 0, 5)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_schedule_covers_each_causal_pair_once(world):
    tc = 3
    S = 2 * world * tc
    count = torch.zeros((S, S), dtype=torch.int32)
    per_step_work = {}
    for r in range(world):
        split, off0, off1 = ring.zigzag_positions(r, world, tc)
        qpos = lambda t, o0=off0, o1=off1: o0 + t if t < split else o1 + t - split
        for blk in ring.ring_schedule(r, world, tc):
            _, s0, s1 = ring.zigzag_positions(blk.src, world, tc)
            kpos = lambda j, o0=s0, o1=s1: o0 + j if j < tc else o1 + j - tc
            work = 0
            for t in range(blk.q_row0, blk.q_row0 + blk.tq):
                for j in range(blk.tk):
                    if blk.causal and j > t:
                        continue
                    count[qpos(t), kpos(j)] += 1
                    work += 1
            per_step_work.setdefault(blk.step, set()).add(work)
            assert (blk.acc_mode == 1) == (blk.step == 0)
    assert torch.equal(count, torch.ones((S, S), dtype=torch.int32).tril())
    for step, works in per_step_work.items():
        assert len(works) == 1, (step, works)  # balanced across ranks


def test_c_abi_block_and_segments_reject_bad_arguments():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(0x10000)

    def block(**kw):
        a = dict(q=fake, k=fake, v=fake, cos=fake, sin=fake, out=fake, lse=fake, acc_o=fake,
                 acc_lse=fake, acc_mode=2, B=1, Hq=8, Hkv=8, T=512, Tkv=512, q_row0=0, Tq=512,
                 Tk=256, causal=0, split=256, off0=0, off1=768, D=128, dt=_lib.DU_DTYPE_BF16,
                 sc=0.088, rp=1024)
        a.update(kw)
        return lib.du_prefill_block(*a.values(), null)

    assert block(acc_mode=3) == _lib.DU_ERR_INVALID and "acc_mode" in _lib.last_error()
    assert block(acc_o=null) == _lib.DU_ERR_INVALID and "accumulators" in _lib.last_error()
    assert block(Tk=513) == _lib.DU_ERR_INVALID and "Tk" in _lib.last_error()
    assert block(q_row0=256, Tq=512) == _lib.DU_ERR_INVALID and "q_row0" in _lib.last_error()
    assert block(causal=1) == _lib.DU_ERR_INVALID and "causal" in _lib.last_error()
    assert block(rp=1023) == _lib.DU_ERR_INVALID and "rope" in _lib.last_error()
    assert block(D=256) == _lib.DU_ERR_UNSUPPORTED
    rc = lib.du_rope_segments(fake, fake, fake, fake, 1, 8, 512, 64, _lib.DU_DTYPE_BF16,
                              _lib.DU_DTYPE_F16, 513, 0, 0, 4096, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "pos_split" in _lib.last_error()
    rc = lib.du_rope_segments(fake, fake, fake, fake, 1, 8, 512, 64, _lib.DU_DTYPE_BF16,
                              _lib.DU_DTYPE_F16, 256, 0, 3900, 4096, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "rope" in _lib.last_error()


def _oracle_rotate(k, cos, sin, rank, world):
    split, off0, off1 = ring.zigzag_positions(rank, world, k.shape[2] // 2)
    t = torch.arange(k.shape[2])
    pos = torch.where(t < split, off0 + t, off1 + (t - split))
    return oracle.apply_rope(k, cos[pos], sin[pos])


def _oracle_block(q, k_rot, v, cos, sin, out, lse, acc_o, acc_lse, blk, pos, hkv):
    o, l = oracle.prefill_block(q, k_rot, v, cos, sin, blk.q_row0, blk.tq, blk.tk, blk.causal,
                                *pos, num_kv_heads=hkv)
    r = slice(blk.q_row0, blk.q_row0 + blk.tq)
    if blk.acc_mode == 1:
        acc_o[:, :, r], acc_lse[:, :, r] = o, l
    else:
        acc_o[:, :, r], acc_lse[:, :, r] = oracle.merge_partials(
            [acc_o[:, :, r].clone(), o], [acc_lse[:, :, r].clone(), l])
    out[:, :, r] = acc_o[:, :, r].to(out.dtype)
    lse[:, :, r] = acc_lse[:, :, r]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        B, Hq, Hkv, tc, D = 2, 4, 2, 5, 16
        S = 2 * world * tc
        q = torch.randn(B, Hq, S, D, generator=g)
        k = torch.randn(B, Hkv, S, D, generator=g)
        v = torch.randn(B, Hkv, S, D, generator=g)
        cos, sin = oracle.precompute_rope_cos_sin(S, D, torch.float32)
        out, lse = ring.ring_prefill(ring.zigzag_shard(q, rank, world),
                                     ring.zigzag_shard(k, rank, world),
                                     ring.zigzag_shard(v, rank, world), cos, sin, Hkv,
                                     rotate_fn=_oracle_rotate, block_fn=_oracle_block)
        outs = [None] * world
        lses = [None] * world
        dist.all_gather_object(outs, out)
        dist.all_gather_object(lses, lse)
        ref_o, ref_l = oracle.prefill(q, k, v, cos, sin, Hkv)
        o_err = (ring.zigzag_unshard(outs) - ref_o).abs().max().item()
        l_err = (ring.zigzag_unshard(lses) - ref_l).abs().max().item()
        result_q.put((rank, o_err, l_err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_prefill_gloo(world):
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
    for rank, o_err, l_err in results:
        assert o_err <= 1e-5 and l_err <= 1e-5, (rank, o_err, l_err)
