"""Prefill and decode replayed from captured CUDA graphs, and back-to-back calls on one stream
(GPU).

Prefill's attention launch is a programmatic dependent of its key-rotation launch, and
decode's merge a programmatic dependent of its split kernel; in a graph these become
programmatic edges. Each replayed output must equal the eager output bit for bit (same
kernels, same inputs) and match the oracle. Back-to-back prefills with different inputs share
the rotated-key workspace: the next call's rotation must not overwrite it while the previous
attention still reads it.
"""

import pytest
import torch

import oracle
from _helpers import LSE_TOL, OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominusultra_b200 import dominus_ultra_decode, dominus_ultra_prefill, precompute_rope_cos_sin

pytestmark = pytest.mark.gpu


def _capture(fn, st):
    with torch.cuda.stream(st):
        fn()
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            outs = fn()
    return graph, outs


@pytest.mark.parametrize("T,D,Hkv", [(1000, 64, 8), (5000, 64, 4), (700, 128, 2), (200, 64, 2),
                                     (100, 32, 8)])
def test_prefill_graph_replay_matches_eager(cuda_device, T, D, Hkv):
    """One-tile kernel (D64, T <= 4096), two-tile kernel (D64 beyond 4096, D128), and the
    one-launch path of short sequences whose attention kernel rotates its own key tiles
    (T <= 256, D <= 64): back-to-back launches with no rotary launch between them."""
    B, Hq = 1, 8
    dtype = torch.bfloat16
    sets = [tuple(randn(s, 70 + 3 * i + j, dtype).cuda() for j, s in
                  enumerate([(B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)])) for i in range(2)]
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype, 1e4)
    cd, sd = cos.cuda(), sin.cuda()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graph, outs = _capture(lambda: [dominus_ultra_prefill(*s, cd, sd, Hkv) for s in sets], st)
    with torch.cuda.stream(st):
        graph.replay()
        eager = [dominus_ultra_prefill(*s, cd, sd, Hkv) for s in sets]
    st.synchronize()
    for (o, l), (eo, el), s in zip(outs, eager, sets):
        assert torch.equal(o, eo) and torch.equal(l, el)
    ro, rl = oracle.prefill(*(t.cpu() for t in sets[1]), cos, sin, Hkv)
    assert max_abs(outs[1][0], ro) <= OUT_TOL and max_abs(outs[1][1], rl) <= LSE_TOL
    del graph
    assert_no_device_timeouts()


@pytest.mark.parametrize("B,Hq,Hkv,L,D,split", [
    (8, 32, 32, 2048, 64, False),   # CUDA-core kernel, 256 one-head whole units
    (2, 8, 2, 8192, 64, True),      # CUDA-core kernel, four-head units cut into fragments
    (2, 8, 2, 20000, 64, True),
    (37, 16, 4, 600, 128, False),   # tensor-core kernel, 148 four-head whole units
    (2, 32, 8, 3000, 128, True),    # tensor-core kernel, few short units over more CTAs
    (1, 32, 8, 131072, 128, True),
])
def test_decode_graph_replay_matches_eager(cuda_device, B, Hq, Hkv, L, D, split):
    """Whole units and the split walk with its merge, on both decode kernels."""
    from dominusultra_b200 import _lib

    assert (_lib.load().du_decode_workspace_size(B, Hq, Hkv, L, D) > 0) == split, "plan changed"
    dtype = torch.bfloat16
    sets = [tuple(randn(s, 90 + 3 * i + j, dtype).cuda() for j, s in
                  enumerate([(B, Hq, 1, D), (B, Hkv, L, D), (B, Hkv, L, D)])) for i in range(2)]
    cos, sin = precompute_rope_cos_sin(L + 1, D, "cpu", dtype, 1e4)
    cd, sd = cos.cuda(), sin.cuda()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graph, outs = _capture(lambda: [dominus_ultra_decode(*s, cd, sd, Hkv) for s in sets], st)
    with torch.cuda.stream(st):
        graph.replay()
        eager = [dominus_ultra_decode(*s, cd, sd, Hkv) for s in sets]
    st.synchronize()
    for o, eo in zip(outs, eager):
        assert torch.equal(o, eo)
    ref = oracle.decode(*(t.cpu() for t in sets[0]), cos, sin, Hkv)
    assert max_abs(outs[0], ref) <= OUT_TOL
    del graph
    assert_no_device_timeouts()


def test_back_to_back_prefills_share_the_workspace(cuda_device):
    """Several prefills of different inputs issued back to back on one stream, then compared
    with the same prefills each followed by a synchronisation."""
    B, Hq, Hkv, T, D = 2, 16, 16, 2048, 64
    dtype = torch.bfloat16
    sets = [tuple(randn(s, 120 + 3 * i + j, dtype).cuda() for j, s in
                  enumerate([(B, Hq, T, D), (B, Hkv, T, D), (B, Hkv, T, D)])) for i in range(4)]
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype, 1e4)
    cd, sd = cos.cuda(), sin.cuda()
    chained = [dominus_ultra_prefill(*s, cd, sd, Hkv) for s in sets]
    torch.cuda.synchronize()
    for s, (o, l) in zip(sets, chained):
        eo, el = dominus_ultra_prefill(*s, cd, sd, Hkv)
        torch.cuda.synchronize()
        assert torch.equal(o, eo) and torch.equal(l, el)
    assert_no_device_timeouts()


def test_graph_replay_after_the_workspace_grows(cuda_device):
    """A captured prefill and a captured split decode keep writing the workspace they were
    captured with. A larger eager call on the same stream then outgrows that workspace; the old
    buffer must stay alive (not return to the allocator), so that tensors allocated afterwards
    on the stream are not overwritten by the replays, and the replays stay correct."""
    from dominusultra_b200 import _lib

    dtype = torch.bfloat16
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    # small prefill (rotated-key workspace) and small decode on the split walk (partials)
    pB, pH, pHkv, pT, pD = 1, 4, 4, 1000, 64
    pin = tuple(randn(s, 300 + j, dtype) for j, s in
                enumerate([(pB, pH, pT, pD), (pB, pHkv, pT, pD), (pB, pHkv, pT, pD)]))
    pcos, psin = precompute_rope_cos_sin(pT, pD, "cpu", dtype, 1e4)
    dB, dH, dHkv, dL, dD = 2, 8, 2, 20000, 64
    assert _lib.load().du_decode_workspace_size(dB, dH, dHkv, dL, dD) > 0
    din = tuple(randn(s, 310 + j, dtype) for j, s in
                enumerate([(dB, dH, 1, dD), (dB, dHkv, dL, dD), (dB, dHkv, dL, dD)]))
    dcos, dsin = precompute_rope_cos_sin(dL + 1, dD, "cpu", dtype, 1e4)
    pg = [t.cuda() for t in pin] + [pcos.cuda(), psin.cuda()]
    dg = [t.cuda() for t in din] + [dcos.cuda(), dsin.cuda()]
    g_pre, (po, pl) = _capture(lambda: dominus_ultra_prefill(*pg, pHkv), st)
    g_dec, do = _capture(lambda: dominus_ultra_decode(*dg, dHkv), st)

    # Larger eager calls on the same stream: both workspaces grow.
    with torch.cuda.stream(st):
        big_p = [torch.randn(s, device="cuda").to(dtype) for s in
                 ((2, 8, 4096, 64), (2, 8, 4096, 64), (2, 8, 4096, 64))]
        bc, bs = precompute_rope_cos_sin(4096, 64, "cuda", dtype, 1e4)
        dominus_ultra_prefill(*big_p, bc, bs, 8)
        B2, H2, Hkv2, L2, D2 = 8, 32, 8, 16384, 256
        assert (_lib.load().du_decode_workspace_size(B2, H2, Hkv2, L2, D2)
                > _lib.load().du_decode_workspace_size(dB, dH, dHkv, dL, dD))
        big_d = [torch.randn(s, device="cuda").to(dtype) for s in
                 ((B2, H2, 1, D2), (B2, Hkv2, L2, D2), (B2, Hkv2, L2, D2))]
        dc2, ds2 = precompute_rope_cos_sin(L2 + 1, D2, "cuda", dtype, 1e4)
        dominus_ultra_decode(*big_d, dc2, ds2, Hkv2)
        del big_p, big_d
        st.synchronize()
        # Freshly allocated tensors on the stream (with a released workspace they would take
        # its memory).
        sentinels = [torch.full((1 << 20,), 7, dtype=torch.uint8, device="cuda") for _ in range(8)]
        g_pre.replay()
        g_dec.replay()
    st.synchronize()
    for s in sentinels:
        assert bool((s == 7).all()), "a graph replay wrote into memory it no longer owns"
    ro, rl = oracle.prefill(*pin, pcos, psin, pHkv)
    assert max_abs(po, ro) <= OUT_TOL and max_abs(pl, rl) <= LSE_TOL
    rd = oracle.decode(*din, dcos, dsin, dHkv)
    assert max_abs(do, rd) <= OUT_TOL
    del g_pre, g_dec
    assert_no_device_timeouts()
