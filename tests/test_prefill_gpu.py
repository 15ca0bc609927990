"""Parity of the sm_100a prefill kernel with the fp32 oracle (GPU).

Gates (from the build's contract): out max-abs <= 2e-2 (bf16/fp16 outputs), LSE max-abs <=
1e-3 (fp32), on unscaled N(0,1) inputs with seeded generators. Shapes cover every head_dim the
reference accepts, GQA/MQA, ragged T (not multiples of the 128-row tile), the benchmark
configurations, and the reference's own test-suite cases.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from _helpers import LSE_TOL, OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominus_ultra import dominus_ultra_prefill, precompute_rope_cos_sin
from dominusultra_b200 import _lib

pytestmark = pytest.mark.gpu


def _run_case(B, Hq, Hkv, T, D, dtype, seed, base=10000.0, heads=None, device="cuda"):
    q = randn((B, Hq, T, D), seed, dtype)
    k = randn((B, Hkv, T, D), seed + 1, dtype)
    v = randn((B, Hkv, T, D), seed + 2, dtype)
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype, base)
    out, lse = dominus_ultra_prefill(
        q.to(device), k.to(device), v.to(device), cos.to(device), sin.to(device), num_kv_heads=Hkv
    )
    torch.cuda.synchronize()
    ref_out, ref_lse = oracle.prefill(q, k, v, cos, sin, Hkv, heads=heads)
    out, lse = out.cpu(), lse.cpu()
    if heads is not None:
        idx = list(heads)
        o_err = max(max_abs(out[b, h], ref_out[b, h]) for b, h in idx)
        l_err = max(max_abs(lse[b, h], ref_lse[b, h]) for b, h in idx)
        assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()
    else:
        o_err = max_abs(out, ref_out)
        l_err = max_abs(lse, ref_lse)
    assert out.dtype == dtype and lse.dtype == torch.float32
    assert_no_device_timeouts()
    return o_err, l_err


SMALL = [
    # B, Hq, Hkv, T, D, dtype. Head_dim <= 64 with T <= 256 takes the one-launch path whose
    # attention kernel rotates its own key tiles (T below one 128-row key tile included).
    (1, 2, 2, 128, 64, torch.bfloat16),
    (1, 8, 2, 64, 64, torch.bfloat16),
    (1, 2, 2, 1, 64, torch.bfloat16),
    (1, 2, 2, 8, 64, torch.bfloat16),
    (1, 2, 1, 17, 64, torch.float16),
    (2, 4, 2, 100, 64, torch.bfloat16),
    (1, 2, 2, 129, 64, torch.bfloat16),
    (1, 4, 1, 257, 64, torch.float16),
    (2, 2, 2, 300, 128, torch.bfloat16),
    (1, 4, 4, 256, 128, torch.float16),
    (1, 2, 2, 200, 32, torch.bfloat16),
    # the longest sequences whose key tiles the attention kernel rotates itself (two tiles)
    (1, 4, 2, 256, 64, torch.float16),
    (1, 2, 2, 255, 32, torch.bfloat16),
    (1, 2, 2, 150, 16, torch.bfloat16),
    (1, 2, 1, 333, 256, torch.bfloat16),
    (1, 2, 2, 128, 256, torch.float16),
    (1, 8, 2, 1000, 64, torch.bfloat16),
]


@pytest.mark.parametrize("B,Hq,Hkv,T,D,dtype", SMALL)
def test_prefill_small_shapes(cuda_device, B, Hq, Hkv, T, D, dtype):
    o_err, l_err = _run_case(B, Hq, Hkv, T, D, dtype, seed=11 + T + D)
    assert o_err <= OUT_TOL, o_err
    assert l_err <= LSE_TOL, l_err


def _sample_heads(B, Hq, n, seed):
    g = torch.Generator().manual_seed(seed)
    pairs = [(b, h) for b in range(B) for h in range(Hq)]
    idx = torch.randperm(len(pairs), generator=g)[:n].tolist()
    return [pairs[i] for i in sorted(idx)]


def test_prefill_cpu_reference_config(cuda_device):
    """B1 H=Hkv=8 S512 D64: the configuration the reference's CPU path runs on."""
    o_err, l_err = _run_case(1, 8, 8, 512, 64, torch.bfloat16, seed=100)
    assert o_err <= OUT_TOL and l_err <= LSE_TOL, (o_err, l_err)


@pytest.mark.parametrize("S", [128, 256, 512, 1024, 2048])
def test_prefill_mha_sweep(cuda_device, S):
    """B2 H=Hkv=32 D64 causal sweep (heads sampled for the oracle at the larger S)."""
    heads = None if S <= 256 else _sample_heads(2, 32, 8, S)
    o_err, l_err = _run_case(2, 32, 32, S, 64, torch.bfloat16, seed=200 + S, heads=heads)
    assert o_err <= OUT_TOL and l_err <= LSE_TOL, (o_err, l_err)


@pytest.mark.parametrize("Hkv", [8, 1])
def test_prefill_gqa_mqa(cuda_device, Hkv):
    """B2 H32 Hkv in {8, 1} S1024 D64."""
    heads = _sample_heads(2, 32, 8, 300 + Hkv)
    o_err, l_err = _run_case(2, 32, Hkv, 1024, 64, torch.bfloat16, seed=300 + Hkv, heads=heads)
    assert o_err <= OUT_TOL and l_err <= LSE_TOL, (o_err, l_err)


def test_prefill_llama_shape_long_context_sampled_rows(cuda_device):
    """One (batch, kv-head) unit of the Llama-3-8B-shaped layer (4 query heads sharing a KV
    head, D128, RoPE base 5e5) at S=32768, checked on sampled rows: causal row i depends only
    on keys <= i, so each sampled row is an exact oracle comparison."""
    B, Hq, Hkv, T, D = 1, 4, 1, 32768, 128
    dtype = torch.bfloat16
    q = randn((B, Hq, T, D), 500, dtype)
    k = randn((B, Hkv, T, D), 501, dtype)
    v = randn((B, Hkv, T, D), 502, dtype)
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype, 500000.0)
    out, lse = dominus_ultra_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), Hkv)
    torch.cuda.synchronize()
    out, lse = out.cpu(), lse.cpu()
    g = torch.Generator().manual_seed(503)
    rows = sorted(set(list(range(128)) + list(range(T - 128, T)) +
                      torch.randint(0, T, (256,), generator=g).tolist()))
    for h in (0, 3):
        ro, rl = oracle.prefill_rows(q, k, v, cos, sin, Hkv, 0, h, rows)
        assert max_abs(out[0, h, rows], ro) <= OUT_TOL
        assert max_abs(lse[0, h, rows], rl) <= LSE_TOL
    assert torch.isfinite(out.float()).all()
    assert_no_device_timeouts()


@pytest.mark.parametrize("T,D", [(4096, 64), (4097, 64), (6000, 64), (5000, 32)])
def test_prefill_both_kernels_around_the_length_switch(cuda_device, T, D):
    """Head_dim <= 64 runs one query tile per CTA up to T = 4096 and two tiles per CTA beyond;
    both sides of the switch, ragged lengths included, against the oracle on sampled rows."""
    B, Hq, Hkv = 1, 4, 2
    dtype = torch.bfloat16
    q = randn((B, Hq, T, D), 510 + T, dtype)
    k = randn((B, Hkv, T, D), 511 + T, dtype)
    v = randn((B, Hkv, T, D), 512 + T, dtype)
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype)
    out, lse = dominus_ultra_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), Hkv)
    torch.cuda.synchronize()
    out, lse = out.cpu(), lse.cpu()
    g = torch.Generator().manual_seed(513 + T)
    rows = sorted(set(list(range(64)) + list(range(T - 200, T)) +
                      torch.randint(0, T, (128,), generator=g).tolist()))
    for h in (0, 3):
        ro, rl = oracle.prefill_rows(q, k, v, cos, sin, Hkv, 0, h, rows)
        assert max_abs(out[0, h, rows], ro) <= OUT_TOL
        assert max_abs(lse[0, h, rows], rl) <= LSE_TOL
    assert_no_device_timeouts()


GOLDEN = np.load(Path(__file__).parent / "golden" / "golden.npz")


@pytest.mark.parametrize("i", range(int(GOLDEN["n_prefill"])))
def test_prefill_matches_reference_kernel_golden(cuda_device, i):
    """fp16 cases computed by the reference's own Triton kernel (CPU interpreter)."""
    B, Hq, Hkv, T, D = (int(x) for x in GOLDEN[f"prefill{i}_shape"])
    t = {n: torch.from_numpy(GOLDEN[f"prefill{i}_{n}"].copy()) for n in
         ("q", "k", "v", "cos", "sin", "out", "lse")}
    out, lse = dominus_ultra_prefill(*(t[n].cuda() for n in ("q", "k", "v", "cos", "sin")), Hkv)
    torch.cuda.synchronize()
    assert max_abs(out, t["out"]) <= OUT_TOL
    assert max_abs(lse, t["lse"]) <= 2e-3


@pytest.mark.parametrize("B,H,T,D", [(1, 8, 64, 64), (2, 16, 256, 128), (4, 32, 512, 64),
                                     (1, 32, 512, 128), (2, 8, 128, 64)])
def test_prefill_reference_suite_cases(cuda_device, B, H, T, D):
    """Cases from the reference's MHA sweep (inputs scaled by 0.1, gate 1e-2 as there)."""
    dtype = torch.bfloat16
    q = randn((B, H, T, D), 40 + T, dtype, 0.1)
    k = randn((B, H, T, D), 41 + T, dtype, 0.1)
    v = randn((B, H, T, D), 42 + T, dtype, 0.1)
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype)
    out, _ = dominus_ultra_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), H)
    ref, _ = oracle.prefill(q, k, v, cos, sin, H)
    assert max_abs(out, ref) < 1e-2


@pytest.mark.parametrize("q_heads,kv_heads", [(32, 8), (32, 4), (16, 4), (8, 1)])
def test_prefill_reference_gqa_cases(cuda_device, q_heads, kv_heads):
    dtype = torch.bfloat16
    B, T, D = 2, 128, 64
    q = randn((B, q_heads, T, D), 60, dtype, 0.1)
    k = randn((B, kv_heads, T, D), 61, dtype, 0.1)
    v = randn((B, kv_heads, T, D), 62, dtype, 0.1)
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", dtype)
    out, _ = dominus_ultra_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), kv_heads)
    ref, _ = oracle.prefill(q, k, v, cos, sin, kv_heads)
    assert max_abs(out, ref) < 1e-2


def test_prefill_guard_bands_untouched(cuda_device):
    """Outputs written through the C ABI into buffers with NaN guard bands on both sides:
    the bands must stay NaN (no out-of-bounds stores), the interior must be finite."""
    B, Hq, Hkv, T, D = 1, 3, 1, 200, 64
    dtype = torch.bfloat16
    q = randn((B, Hq, T, D), 70, dtype).cuda()
    k = randn((B, Hkv, T, D), 71, dtype).cuda()
    v = randn((B, Hkv, T, D), 72, dtype).cuda()
    cos, sin = precompute_rope_cos_sin(T, D, "cuda", dtype)
    band = 4096
    n_out = B * Hq * T * D
    n_lse = B * Hq * T
    out_buf = torch.full((n_out + 2 * band,), float("nan"), dtype=dtype, device="cuda")
    lse_buf = torch.full((n_lse + 2 * band,), float("nan"), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    ws = torch.empty(lib.du_prefill_workspace_size(B, Hq, Hkv, T, D), dtype=torch.uint8, device="cuda")
    rc = lib.du_prefill(p(q), p(k), p(v), p(cos), p(sin), ctypes.c_void_p(out_buf[band:].data_ptr()),
                        ctypes.c_void_p(lse_buf[band:].data_ptr()), B, Hq, Hkv, T, D,
                        _lib.DU_DTYPE_BF16, 1.0 / 8.0, T, p(ws), ws.numel(),
                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "du_prefill")
    torch.cuda.synchronize()
    assert torch.isnan(out_buf[:band].float()).all() and torch.isnan(out_buf[band + n_out:].float()).all()
    assert torch.isnan(lse_buf[:band]).all() and torch.isnan(lse_buf[band + n_lse:]).all()
    assert torch.isfinite(out_buf[band:band + n_out].float()).all()
    assert torch.isfinite(lse_buf[band:band + n_lse]).all()
    assert_no_device_timeouts()


def test_prefill_shapes_dtypes_and_stability(cuda_device):
    """Output shape/dtype contract and NaN/Inf freedom at unscaled inputs
    (reference test_dominus.py:194-228 and :425-438)."""
    for dtype in (torch.bfloat16, torch.float16):
        B, H, T, D = 2, 8, 128, 64
        q, k, v = (randn((B, H, T, D), s, dtype).cuda() for s in (80, 81, 82))
        cos, sin = precompute_rope_cos_sin(T, D, "cuda", dtype)
        out, lse = dominus_ultra_prefill(q, k, v, cos, sin)
        assert out.shape == (B, H, T, D) and out.dtype == dtype
        assert lse.shape == (B, H, T) and lse.dtype == torch.float32
        assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()


def test_prefill_longer_tables_accepted(cuda_device):
    """Tables longer than T are allowed (dominus_ultra.py:88): rows 0..T-1 are used."""
    B, H, T, D = 1, 2, 77, 64
    dtype = torch.bfloat16
    q, k, v = (randn((B, H, T, D), s, dtype) for s in (90, 91, 92))
    cos, sin = precompute_rope_cos_sin(1000, D, "cpu", dtype)
    out, lse = dominus_ultra_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda())
    ref_o, ref_l = oracle.prefill(q, k, v, cos, sin, H)
    assert max_abs(out, ref_o) <= OUT_TOL and max_abs(lse, ref_l) <= LSE_TOL
