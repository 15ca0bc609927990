"""Parity of the sm_100a decode kernels (split-KV + merge) with the fp32 oracle (GPU).

Gate: out max-abs <= 2e-2 on unscaled N(0,1) inputs; partial LSEs within 1e-3. Covers the
decode sweep configuration, GQA/MQA, every head_dim, ragged and tiny cache lengths, the
reference's own test cases and golden vectors from the reference's kernel, the shard/merge
path used for the multi-GPU long-context decode, and guard bands around the output.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from _helpers import LSE_TOL, OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominus_ultra import dominus_ultra_decode, precompute_rope_cos_sin
from dominusultra_b200 import _lib, decode_partial, merge_partials

pytestmark = pytest.mark.gpu


def _inputs(B, Hq, Hkv, L, D, dtype, seed, base=10000.0, scale=1.0):
    q = randn((B, Hq, 1, D), seed, dtype, scale)
    k = randn((B, Hkv, L, D), seed + 1, dtype, scale)
    v = randn((B, Hkv, L, D), seed + 2, dtype, scale)
    cos, sin = precompute_rope_cos_sin(L + 1, D, "cpu", dtype, base)
    return q, k, v, cos, sin


def _check(B, Hq, Hkv, L, D, dtype, seed):
    q, k, v, cos, sin = _inputs(B, Hq, Hkv, L, D, dtype, seed)
    out = dominus_ultra_decode(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), num_kv_heads=Hkv)
    torch.cuda.synchronize()
    assert out.shape == (B, Hq, 1, D) and out.dtype == dtype
    ref = oracle.decode(q, k, v, cos, sin, Hkv)
    assert_no_device_timeouts()
    return max_abs(out, ref)


@pytest.mark.parametrize("L", [128, 256, 512, 1024, 2048])
def test_decode_sweep(cuda_device, L):
    """B8 H=Hkv=32 D64, one query at position L."""
    err = _check(8, 32, 32, L, 64, torch.bfloat16, seed=1000 + L)
    assert err <= OUT_TOL, err


CASES = [
    # B, Hq, Hkv, L, D, dtype
    (1, 8, 8, 1, 64, torch.bfloat16),
    (2, 4, 4, 7, 64, torch.float16),
    (2, 32, 8, 128, 64, torch.bfloat16),
    (2, 16, 4, 257, 64, torch.bfloat16),
    (2, 8, 1, 128, 64, torch.bfloat16),
    (1, 32, 1, 1000, 64, torch.float16),
    (2, 6, 2, 300, 64, torch.bfloat16),
    (1, 5, 5, 4097, 64, torch.bfloat16),
    (2, 32, 8, 1500, 128, torch.bfloat16),
    (1, 8, 2, 700, 128, torch.float16),
    (1, 4, 2, 333, 16, torch.bfloat16),
    (1, 4, 4, 999, 32, torch.bfloat16),
    (1, 8, 2, 640, 256, torch.bfloat16),
    (1, 4, 4, 9000, 256, torch.float16),
]


@pytest.mark.parametrize("B,Hq,Hkv,L,D,dtype", CASES)
def test_decode_shapes(cuda_device, B, Hq, Hkv, L, D, dtype):
    err = _check(B, Hq, Hkv, L, D, dtype, seed=2000 + L + D)
    assert err <= OUT_TOL, err


@pytest.mark.parametrize("q_heads,kv_heads", [(32, 8), (16, 4), (8, 1)])
def test_decode_reference_gqa_cases(cuda_device, q_heads, kv_heads):
    """Reference test_dominus.py:291-345 (inputs x0.1, gate 1e-2)."""
    q, k, v, cos, sin = _inputs(2, q_heads, kv_heads, 128, 64, torch.bfloat16, 3000, scale=0.1)
    out = dominus_ultra_decode(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), kv_heads)
    assert max_abs(out, oracle.decode(q, k, v, cos, sin, kv_heads)) < 1e-2


@pytest.mark.parametrize("B,H,L,D", [(1, 8, 64, 64), (4, 32, 256, 128), (2, 16, 128, 64)])
def test_decode_reference_mha_cases(cuda_device, B, H, L, D):
    q, k, v, cos, sin = _inputs(B, H, H, L, D, torch.bfloat16, 3100 + L, scale=0.1)
    out = dominus_ultra_decode(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda())
    assert max_abs(out, oracle.decode(q, k, v, cos, sin, H)) < 1e-2


GOLDEN = np.load(Path(__file__).parent / "golden" / "golden.npz")


@pytest.mark.parametrize("i", range(int(GOLDEN["n_decode"])))
def test_decode_matches_reference_kernel_golden(cuda_device, i):
    B, Hq, Hkv, L, D = (int(x) for x in GOLDEN[f"decode{i}_shape"])
    t = {n: torch.from_numpy(GOLDEN[f"decode{i}_{n}"].copy()) for n in
         ("q", "k", "v", "cos", "sin", "out")}
    out = dominus_ultra_decode(*(t[n].cuda() for n in ("q", "k", "v", "cos", "sin")), Hkv)
    torch.cuda.synchronize()
    assert max_abs(out, t["out"]) <= OUT_TOL


def test_decode_sharded_sequence_merge_matches_full(cuda_device):
    """The long-context path on one GPU: split the KV sequence into 8 shards, compute each
    shard's partial at its absolute positions, merge by LSE, compare with the full oracle."""
    B, Hq, Hkv, L, D = 1, 32, 8, 16384, 128
    dtype = torch.bfloat16
    q, k, v, cos, sin = _inputs(B, Hq, Hkv, L, D, dtype, 4000, base=500000.0)
    qd, kd, vd, cd, sd = q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda()
    R = 8
    step = L // R
    o_parts = torch.empty((R, B, Hq, D), dtype=torch.float32, device="cuda")
    l_parts = torch.empty((R, B, Hq), dtype=torch.float32, device="cuda")
    for r in range(R):
        a, b = r * step, (r + 1) * step
        decode_partial(qd, kd[:, :, a:b].contiguous(), vd[:, :, a:b].contiguous(), cd, sd, Hkv,
                       q_pos=L, kv_pos_offset=a, out=o_parts[r], lse=l_parts[r])
        ref_o, ref_l = oracle.decode_partial(q, k[:, :, a:b], v[:, :, a:b], cos, sin, Hkv,
                                             q_pos=L, kv_pos_offset=a)
        assert max_abs(o_parts[r], ref_o) <= 5e-3
        assert max_abs(l_parts[r], ref_l) <= LSE_TOL
    out, lse = merge_partials(o_parts, l_parts, dtype, with_lse=True)
    ref = oracle.decode(q, k, v, cos, sin, Hkv)[:, :, 0]
    assert max_abs(out, ref) <= OUT_TOL
    assert_no_device_timeouts()


def test_decode_guard_bands_untouched(cuda_device):
    B, Hq, Hkv, L, D = 2, 8, 8, 8192, 64
    dtype = torch.bfloat16
    q, k, v, cos, sin = (t.cuda() for t in _inputs(B, Hq, Hkv, L, D, dtype, 5000))
    lib = _lib.load()
    ws_bytes = lib.du_decode_workspace_size(B, Hq, Hkv, L, D)
    assert ws_bytes > 0  # this shape takes the multi-split path
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")  # zero-filled before first use
    band = 2048
    n = B * Hq * D
    out_buf = torch.full((n + 2 * band,), float("nan"), dtype=dtype, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.du_decode(p(q), p(k), p(v), p(cos), p(sin), ctypes.c_void_p(out_buf[band:].data_ptr()),
                       B, Hq, Hkv, L, D, _lib.DU_DTYPE_BF16, 0.125, L + 1, p(ws), ws_bytes,
                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "du_decode")
    torch.cuda.synchronize()
    assert torch.isnan(out_buf[:band].float()).all() and torch.isnan(out_buf[band + n:].float()).all()
    ref = oracle.decode(q.cpu(), k.cpu(), v.cpu(), cos.cpu(), sin.cpu(), Hkv).reshape(-1)
    assert max_abs(out_buf[band:band + n], ref) <= OUT_TOL
    rc = lib.du_decode(p(q), p(k), p(v), p(cos), p(sin), ctypes.c_void_p(out_buf[band:].data_ptr()),
                       B, Hq, Hkv, L, D, _lib.DU_DTYPE_BF16, 0.125, L + 1, p(ws), ws_bytes - 4,
                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.DU_ERR_WORKSPACE
    assert_no_device_timeouts()


def test_decode_single_token_and_shape(cuda_device):
    """Reference edge cases: cache length 1 (test_dominus.py:410-423), output shape (:347-360)."""
    q, k, v, cos, sin = (t.cuda() for t in _inputs(1, 8, 8, 1, 64, torch.bfloat16, 6000))
    out = dominus_ultra_decode(q, k, v, cos, sin)
    assert out.shape == (1, 8, 1, 64) and torch.isfinite(out.float()).all()
    # with one cached key the output is exactly that key's value row
    assert max_abs(out[:, :, 0], v[:, :, 0]) == 0.0


TC_CASES = [
    # B, Hq, Hkv, L, dtype: groups of 4, 8 and 16 query heads at head_dim 128 (the tcgen05 kernel)
    (2, 8, 2, 1, torch.bfloat16),        # one key: a chunk of 128 rows with 127 masked
    (2, 8, 2, 127, torch.float16),
    (1, 16, 4, 128, torch.bfloat16),     # exactly one chunk
    (1, 16, 4, 129, torch.bfloat16),     # one key into the second chunk
    (40, 32, 8, 300, torch.bfloat16),    # 320 units: several whole units per CTA
    (2, 32, 8, 20000, torch.bfloat16),   # long split walk, fragments across units
    (1, 64, 16, 2500, torch.float16),
    (2, 16, 2, 3000, torch.bfloat16),    # group 8: eight-head units
    (1, 64, 4, 5000, torch.float16),     # group 16: two eight-head units per KV head
    (24, 64, 8, 300, torch.bfloat16),    # 192 eight-head units
    (25, 16, 4, 2048, torch.bfloat16),   # 100 units of 16 chunks: many CTAs reach into a second unit
    (7, 32, 8, 5000, torch.float16),     # ragged last chunk, CTAs cut with unit starts charged
]


@pytest.mark.parametrize("B,Hq,Hkv,L,dtype", TC_CASES)
def test_decode_four_head_units_tensor_core(cuda_device, B, Hq, Hkv, L, dtype):
    D = 128
    q, k, v, cos, sin = _inputs(B, Hq, Hkv, L, D, dtype, seed=L + B, base=500000.0)
    out = dominus_ultra_decode(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), num_kv_heads=Hkv)
    torch.cuda.synchronize()
    ref = oracle.decode(q, k, v, cos, sin, Hkv)
    assert_no_device_timeouts()
    assert max_abs(out, ref) <= OUT_TOL


def test_decode_four_head_partial_outputs(cuda_device):
    """du_decode_partial on a shard at a position offset (fp32 out and LSE, the multi-GPU path)
    through the tensor-core kernel, whole-unit and split plans."""
    for B, L in ((40, 256), (2, 9000)):
        Hq, Hkv, D, off = 32, 8, 128, 777
        q, k, v, _, _ = _inputs(B, Hq, Hkv, L, D, torch.bfloat16, seed=5 + B)
        cos, sin = precompute_rope_cos_sin(off + L + 1, D, "cpu", torch.bfloat16, 500000.0)
        o, lse = decode_partial(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), Hkv,
                                off + L, off)
        torch.cuda.synchronize()
        ro, rl = oracle.decode_partial(q, k, v, cos, sin, Hkv, q_pos=off + L, kv_pos_offset=off)
        assert_no_device_timeouts()
        assert max_abs(o, ro) <= OUT_TOL and max_abs(lse, rl) <= LSE_TOL


@pytest.mark.parametrize("B,Hq,Hkv,L,D", [(4, 32, 8, 16384, 128), (1, 64, 8, 20000, 128),
                                          (2, 32, 8, 3000, 128), (25, 16, 4, 2048, 128),
                                          (4, 64, 8, 16384, 128)])
def test_decode_split_merge_in_kernel_leaves_counters_zero(cuda_device, B, Hq, Hkv, L, D):
    """The tensor-core decode merges a unit's partials inside the split kernel: the CTA that
    takes the unit's last ticket merges. Two calls in a row on one zero-filled workspace match
    the oracle, and both leave the ticket counters (the first 16 KB) zero."""
    lib = _lib.load()
    ws_bytes = lib.du_decode_workspace_size(B, Hq, Hkv, L, D)
    assert ws_bytes > 16384
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        q, k, v, cos, sin = _inputs(B, Hq, Hkv, L, D, torch.bfloat16, 6000 + 10 * call)
        out = torch.full((B, Hq, D), float("nan"), dtype=torch.bfloat16, device="cuda")
        dq, dk, dv, dc, ds = (t.cuda() for t in (q, k, v, cos, sin))
        rc = lib.du_decode(p(dq), p(dk), p(dv), p(dc), p(ds), p(out), B, Hq, Hkv, L, D,
                           _lib.DU_DTYPE_BF16, D ** -0.5, L + 1, p(ws), ws_bytes, st)
        _lib.check(rc, "du_decode")
        torch.cuda.synchronize()
        assert int(ws[:16384].count_nonzero().item()) == 0, call
        assert max_abs(out, oracle.decode(q, k, v, cos, sin, Hkv).squeeze(2)) <= OUT_TOL
    assert_no_device_timeouts()
