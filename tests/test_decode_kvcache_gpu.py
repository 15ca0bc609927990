"""Parity of the KV-cache decode step (per-sequence lengths, new token appended) with the fp32
oracle (GPU).

Gate: out max-abs <= 2e-2 on unscaled N(0,1) inputs; the cache update is bit-exact (row s_b of
each sequence holds the new key / value, every other row is untouched). Covers empty, one-token
and full caches, every query-group width the kernel instantiates (1, 2, 4 heads per unit), both
dtypes, lengths far below the capacity, one long sequence beside short ones (a unit spread over
every CTA), CUDA-graph replay with lengths that change between replays, and out-of-range
lengths reported through the device status words.
"""

import pytest
import torch

import oracle
from _helpers import OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominus_ultra import dominus_ultra_decode, dominus_ultra_decode_kvcache, precompute_rope_cos_sin
from dominusultra_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(B, Hq, Hkv, Lmax, D, dtype, seed, base=10000.0):
    q = randn((B, Hq, 1, D), seed, dtype)
    kc = randn((B, Hkv, Lmax, D), seed + 1, dtype)
    vc = randn((B, Hkv, Lmax, D), seed + 2, dtype)
    kn = randn((B, Hkv, 1, D), seed + 3, dtype)
    vn = randn((B, Hkv, 1, D), seed + 4, dtype)
    cos, sin = precompute_rope_cos_sin(Lmax + 1, D, "cpu", dtype, base)
    return q, kc, vc, kn, vn, cos, sin


def _run(B, Hq, Hkv, Lmax, D, dtype, lens, append, seed, base=10000.0):
    q, kc, vc, kn, vn, cos, sin = _inputs(B, Hq, Hkv, Lmax, D, dtype, seed, base)
    kc_d, vc_d = kc.cuda(), vc.cuda()
    seqlens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = dominus_ultra_decode_kvcache(
        q.cuda(), kc_d, vc_d, cos.cuda(), sin.cuda(), seqlens,
        kn.cuda() if append else None, vn.cuda() if append else None, num_kv_heads=Hkv)
    torch.cuda.synchronize()
    assert out.shape == (B, Hq, 1, D) and out.dtype == dtype
    ref, kref, vref = oracle.decode_kvcache(q, kc, vc, cos, sin, lens, kn if append else None,
                                            vn if append else None, num_kv_heads=Hkv)
    assert_no_device_timeouts()
    assert torch.equal(kc_d.cpu(), kref) and torch.equal(vc_d.cpu(), vref), "cache update"
    return max_abs(out, ref), out


CASES = [
    # B, Hq, Hkv, Lmax, D, dtype, lens
    (4, 8, 8, 300, 64, torch.bfloat16, [0, 1, 150, 299]),          # one head per unit
    (3, 8, 4, 513, 64, torch.float16, [512, 64, 65]),              # two heads per unit
    (3, 16, 4, 1000, 128, torch.bfloat16, [999, 3, 640]),          # four heads per unit
    (2, 32, 8, 2048, 128, torch.bfloat16, [2047, 1000]),           # Llama-shaped GQA
    (5, 4, 1, 200, 32, torch.bfloat16, [5, 0, 199, 17, 100]),      # MQA
    (2, 2, 2, 100, 16, torch.float16, [40, 99]),
    (2, 4, 2, 100, 256, torch.bfloat16, [99, 1]),
    (6, 12, 4, 700, 64, torch.bfloat16, [1, 2, 3, 640, 641, 699]),  # ragged around chunks
    (3, 16, 2, 900, 128, torch.bfloat16, [899, 5, 0]),              # group 8, an empty sequence
]


@pytest.mark.parametrize("append", [True, False])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}H{c[1]}K{c[2]}L{c[3]}D{c[4]}")
def test_kvcache_parity(cuda_device, case, append):
    B, Hq, Hkv, Lmax, D, dtype, lens = case
    if append:
        lens = [min(s, Lmax - 1) for s in lens]
    err, _ = _run(B, Hq, Hkv, Lmax, D, dtype, lens, append, seed=len(lens) * 7 + D)
    assert err <= OUT_TOL, err


def test_kvcache_lengths_far_below_capacity(cuda_device):
    """A 16k-position cache holding a few hundred tokens per sequence: only the present chunks
    are streamed and split over the CTAs."""
    err, _ = _run(8, 32, 8, 16384, 128, torch.bfloat16, [300, 5, 1200, 77, 0, 64, 2000, 129],
                  True, seed=91, base=500000.0)
    assert err <= OUT_TOL, err


def test_kvcache_one_long_sequence_spans_every_cta(cuda_device):
    """One unit far longer than the rest: its chunks spread over every CTA of the walk, so the
    merge combines hundreds of fragment slots for its rows."""
    err, _ = _run(3, 1, 1, 60000, 64, torch.bfloat16, [59000, 3, 0], True, seed=17)
    assert err <= OUT_TOL, err


def test_kvcache_uniform_matches_plain_decode(cuda_device):
    """Equal lengths and no append: the same attention as dominus_ultra_decode on the prefix."""
    B, Hq, Hkv, Lmax, D, L = 4, 32, 8, 4096, 128, 3000
    q, kc, vc, _, _, cos, sin = _inputs(B, Hq, Hkv, Lmax, D, torch.bfloat16, 5, 500000.0)
    qd, kd, vd, cd, sd = q.cuda(), kc.cuda(), vc.cuda(), cos.cuda(), sin.cuda()
    seqlens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    a = dominus_ultra_decode_kvcache(qd, kd, vd, cd, sd, seqlens, num_kv_heads=Hkv)
    b = dominus_ultra_decode(qd, kd[:, :, :L].contiguous(), vd[:, :, :L].contiguous(), cd, sd,
                             num_kv_heads=Hkv)
    torch.cuda.synchronize()
    assert_no_device_timeouts()
    assert max_abs(a, b) <= 4e-3


def test_kvcache_cpu_seqlens_and_int64(cuda_device):
    B, Hq, Hkv, Lmax, D = 2, 4, 4, 64, 64
    q, kc, vc, kn, vn, cos, sin = _inputs(B, Hq, Hkv, Lmax, D, torch.bfloat16, 3)
    lens = [10, 63]
    ref, _, _ = oracle.decode_kvcache(q, kc, vc, cos, sin, lens, kn, vn, num_kv_heads=Hkv)
    for sl in (torch.tensor(lens, dtype=torch.int64), torch.tensor(lens, device="cuda")):
        kd, vd = kc.cuda(), vc.cuda()
        out = dominus_ultra_decode_kvcache(q.cuda(), kd, vd, cos.cuda(), sin.cuda(), sl,
                                           kn.cuda(), vn.cuda(), num_kv_heads=Hkv)
        assert max_abs(out, ref) <= OUT_TOL
    with pytest.raises(ValueError, match=r"cache_seqlens\[1\] = 64"):
        dominus_ultra_decode_kvcache(q.cuda(), kc.cuda(), vc.cuda(), cos.cuda(), sin.cuda(),
                                     torch.tensor([0, 64]), kn.cuda(), vn.cuda())


def test_kvcache_generation_loop_in_a_cuda_graph(cuda_device):
    """Capture one step, then replay it as a generation loop: the lengths advance on the device
    between replays and every step matches the oracle (the graph is never re-captured)."""
    B, Hq, Hkv, Lmax, D = 3, 16, 4, 512, 64
    dtype = torch.bfloat16
    q, kc, vc, _, _, cos, sin = _inputs(B, Hq, Hkv, Lmax, D, dtype, 11)
    start = [100, 0, 400]
    kd, vd, cd, sd = kc.cuda(), vc.cuda(), cos.cuda(), sin.cuda()
    qd = q.cuda()
    knd = torch.empty((B, Hkv, 1, D), dtype=dtype, device="cuda")
    vnd = torch.empty_like(knd)
    seqlens = torch.tensor(start, dtype=torch.int32, device="cuda")
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        # warm-up call (allocates the workspace) on a scratch copy of the caches
        dominus_ultra_decode_kvcache(qd, kd.clone(), vd.clone(), cd, sd, seqlens, knd, vnd,
                                     num_kv_heads=Hkv)
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            out = dominus_ultra_decode_kvcache(qd, kd, vd, cd, sd, seqlens, knd, vnd,
                                               num_kv_heads=Hkv)
    kref, vref = kc.clone(), vc.clone()
    lens = list(start)
    for step in range(4):
        kn = randn((B, Hkv, 1, D), 200 + step, dtype)
        vn = randn((B, Hkv, 1, D), 300 + step, dtype)
        with torch.cuda.stream(st):  # inputs change on the replay stream, in order
            knd.copy_(kn)
            vnd.copy_(vn)
            graph.replay()
        st.synchronize()
        ref, kref, vref = oracle.decode_kvcache(q, kref, vref, cos, sin, lens, kn, vn,
                                                num_kv_heads=Hkv)
        assert max_abs(out, ref) <= OUT_TOL, step
        assert torch.equal(kd.cpu(), kref) and torch.equal(vd.cpu(), vref), step
        with torch.cuda.stream(st):
            seqlens += 1
        lens = [s + 1 for s in lens]
    del graph
    assert_no_device_timeouts()


def test_kvcache_out_of_range_lengths_are_reported(cuda_device):
    """Lengths the host cannot see: the kernel turns them into an empty sequence (zero output,
    nothing appended) and reports status code 6; the other sequences are unaffected."""
    B, Hq, Hkv, Lmax, D = 4, 8, 8, 128, 64
    q, kc, vc, kn, vn, cos, sin = _inputs(B, Hq, Hkv, Lmax, D, torch.bfloat16, 23)
    _lib.read_status(reset=True)
    kd, vd = kc.cuda(), vc.cuda()
    seqlens = torch.tensor([5, -3, 128, 127], dtype=torch.int32, device="cuda")
    out = dominus_ultra_decode_kvcache(q.cuda(), kd, vd, cos.cuda(), sin.cuda(), seqlens,
                                       kn.cuda(), vn.cuda(), num_kv_heads=Hkv)
    torch.cuda.synchronize()
    words = _lib.read_status(reset=True)
    assert words[0] == 6 and words[1] in (1, 2), words
    out = out.cpu()
    assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[2]) == 0
    ref, kref, vref = oracle.decode_kvcache(q[[0, 3]], kc[[0, 3]], vc[[0, 3]], cos, sin, [5, 127],
                                            kn[[0, 3]], vn[[0, 3]], num_kv_heads=Hkv)
    assert max_abs(out[[0, 3]], ref) <= OUT_TOL
    assert torch.equal(kd.cpu()[[1, 2]], kc[[1, 2]]) and torch.equal(kd.cpu()[[0, 3]], kref)


def test_kvcache_whole_units_and_split_walk_in_one_graph(cuda_device):
    """128 one-head units: near-uniform lengths take whole units (final rows straight from the
    split kernel, the merge returns at once), a skewed length set on the same shape takes the
    length-balanced split walk. Both are replayed from one captured graph and checked against
    the oracle; the mode word the prep kernel writes (after the chunk offsets and lengths in the
    workspace) shows which path ran."""
    from dominusultra_b200 import attention as A

    B, Hq, Hkv, Lmax, D = 8, 16, 16, 1024, 64
    dtype = torch.bfloat16
    q, kc, vc, _, _, cos, sin = _inputs(B, Hq, Hkv, Lmax, D, dtype, 41)
    kd, vd, cd, sd, qd = kc.cuda(), vc.cuda(), cos.cuda(), sin.cuda(), q.cuda()
    knd = torch.empty((B, Hkv, 1, D), dtype=dtype, device="cuda")
    vnd = torch.empty_like(knd)
    seqlens = torch.zeros(B, dtype=torch.int32, device="cuda")
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        dominus_ultra_decode_kvcache(qd, kd.clone(), vd.clone(), cd, sd, seqlens, knd, vnd,
                                     num_kv_heads=Hkv)
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            out = dominus_ultra_decode_kvcache(qd, kd, vd, cd, sd, seqlens, knd, vnd,
                                               num_kv_heads=Hkv)
    ws = A._WORKSPACES[("decode_kvcache", torch.cuda.current_device(), st.cuda_stream)][0]
    flag_at = 2 * 256  # offsets [B+1] int64 and {len, qpos} [B], each padded to 256 bytes
    kref, vref = kc.clone(), vc.clone()
    cases = [([900, 905, 890, 899, 910, 880, 902, 895], 1),
             ([1000, 3, 5, 0, 7, 2, 1, 4], 0),
             ([700, 702, 698, 705, 699, 701, 703, 700], 1)]
    for step, (lens, whole) in enumerate(cases):
        kn = randn((B, Hkv, 1, D), 500 + step, dtype)
        vn = randn((B, Hkv, 1, D), 600 + step, dtype)
        with torch.cuda.stream(st):
            seqlens.copy_(torch.tensor(lens, dtype=torch.int32))
            knd.copy_(kn)
            vnd.copy_(vn)
            graph.replay()
        st.synchronize()
        mode = int(ws[flag_at:flag_at + 4].view(torch.int32).item())
        assert mode == whole, (step, mode)
        ref, kref, vref = oracle.decode_kvcache(q, kref, vref, cos, sin, lens, kn, vn,
                                                num_kv_heads=Hkv)
        assert max_abs(out, ref) <= OUT_TOL, step
        assert torch.equal(kd.cpu(), kref) and torch.equal(vd.cpu(), vref), step
    del graph
    assert_no_device_timeouts()
