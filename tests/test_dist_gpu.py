"""Sequence-split decode across 2 GPUs with NCCL (skipped with fewer than 2 GPUs).

Each rank holds a contiguous shard of the KV sequence, runs du_decode_partial at the shard's
absolute positions, the packed partials are exchanged with one all_gather_into_tensor over
NCCL, and every rank merges them with du_merge_partials. The merged output on every rank is
compared with the unsharded fp32 oracle.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out, peer=False):
    import datetime

    import torch.distributed as dist

    import oracle
    from dominusultra_b200 import dist as ddist
    from dominusultra_b200 import precompute_rope_cos_sin

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(321)
        B, Hq, Hkv, L, D = 2, 32, 8, 8192, 128
        q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
        cos, sin = precompute_rope_cos_sin(L + 1, D, "cpu", torch.bfloat16, 500000.0)
        a, b = ddist.kv_shard(L, world, rank)
        dev = torch.device("cuda", rank)
        ex = ddist.PeerExchange(B * Hq, D, device=dev) if peer else None
        ref = oracle.decode(q, k, v, cos, sin, Hkv)
        errs = []
        # Two calls in a row (the peer exchange alternates its slots and flags between calls),
        # the second on rescaled values so a stale slot would show.
        for call in range(2 if peer else 1):
            qs = q if call == 0 else (q * 0.5).to(torch.bfloat16)
            out = ddist.sharded_decode(qs.to(dev), k[:, :, a:b].contiguous().to(dev),
                                       v[:, :, a:b].contiguous().to(dev), cos.to(dev), sin.to(dev),
                                       Hkv, L, a, exchange=ex)
            torch.cuda.synchronize()
            r = ref if call == 0 else oracle.decode(qs, k, v, cos, sin, Hkv)
            errs.append((out.float().cpu() - r).abs().max().item())
        if ex is not None:
            from dominusultra_b200 import _lib
            status = _lib.read_status(reset=True)
            ex.close()
            assert status[0] == 0, status
        q_out.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_decode_two_gpus_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err in res:
        assert err <= 2e-2, (rank, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_decode_two_gpus_peer_exchange():
    """The same sequence-split decode with the partials exchanged and merged over NVLink peer
    memory (PeerExchange, du_exchange_merge) instead of NCCL: two calls in a row on each rank
    match the unsharded oracle, and no bounded wait expires."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, True)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err in res:
        assert err <= 2e-2, (rank, err)
