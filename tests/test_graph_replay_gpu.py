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


@pytest.mark.parametrize("T,D,Hkv", [(1000, 64, 8), (5000, 64, 4), (700, 128, 2)])
def test_prefill_graph_replay_matches_eager(cuda_device, T, D, Hkv):
    """One-tile kernel (D64, T <= 4096) and two-tile kernel (D64 beyond 4096, D128)."""
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


@pytest.mark.parametrize("B,Hq,Hkv,L,D", [(8, 32, 32, 2048, 64), (2, 8, 2, 8192, 64), (2, 32, 8, 3000, 128)])
def test_decode_graph_replay_matches_eager(cuda_device, B, Hq, Hkv, L, D):
    """Whole units (256 one-head units) and the split walk with its merge."""
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
