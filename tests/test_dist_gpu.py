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


def _worker(rank, world, port, q_out):
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
        out = ddist.sharded_decode(q.to(dev), k[:, :, a:b].contiguous().to(dev),
                                   v[:, :, a:b].contiguous().to(dev), cos.to(dev), sin.to(dev),
                                   Hkv, L, a)
        torch.cuda.synchronize()
        ref = oracle.decode(q, k, v, cos, sin, Hkv)
        err = (out.float().cpu() - ref).abs().max().item()
        q_out.put((rank, err))
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
