"""du_decode_noalloc: decode for callers that cannot allocate device memory.

Some callers of this library cannot allocate device memory: a host that binds the C ABI from
another runtime with no CUDA allocator of its own, or a serving loop that must not call
cudaMalloc once it is running. For them ``du_decode_noalloc`` keeps the split-KV partials in
a fixed scratch array inside the library instead of a caller-provided workspace; the caller
still passes the inputs and the output.

These tests call it through the C ABI and compare it with ``du_decode`` (which takes a
workspace) on two calls in a row, within the parity tolerance of the other tests, and check
that a size needing more than the fixed scratch is refused. The file is named to be collected
last, and it passes alone in a fresh process as well as after the other tests.
"""

import ctypes

import pytest
import torch

from _helpers import OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominusultra_b200 import _lib, precompute_rope_cos_sin

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(B, Hq, Hkv, L, D, seed, dtype=torch.bfloat16):
    q = randn((B, Hq, D), seed, dtype).cuda()
    k = randn((B, Hkv, L, D), seed + 1, dtype).cuda()
    v = randn((B, Hkv, L, D), seed + 2, dtype).cuda()
    cos, sin = precompute_rope_cos_sin(L + 1, D, "cuda", dtype)
    return q, k, v, cos, sin


def _decode_with_workspace(lib, q, k, v, cos, sin, B, Hq, Hkv, L, D, code):
    out = torch.empty((B, Hq, D), dtype=q.dtype, device="cuda")
    nbytes = lib.du_decode_workspace_size(B, Hq, Hkv, L, D)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda") if nbytes else None
    rc = lib.du_decode(_p(q), _p(k), _p(v), _p(cos), _p(sin), _p(out), B, Hq, Hkv, L, D, code,
                       D ** -0.5, L + 1, _p(ws), nbytes, _stream())
    _lib.check(rc, "du_decode")
    return out, nbytes


def test_noalloc_decode_matches_workspace_decode_twice(cuda_device):
    lib = _lib.load()
    cases = [
        # B, Hq, Hkv, L, D, dtype: both take the multi-split path (non-zero scratch)
        (2, 8, 8, 8192, 64, torch.bfloat16, _lib.DU_DTYPE_BF16),
        (1, 32, 8, 40000, 128, torch.float16, _lib.DU_DTYPE_F16),
    ]
    for i, (B, Hq, Hkv, L, D, dtype, code) in enumerate(cases):
        q, k, v, cos, sin = _inputs(B, Hq, Hkv, L, D, 700 + 10 * i, dtype)
        ref, nbytes = _decode_with_workspace(lib, q, k, v, cos, sin, B, Hq, Hkv, L, D, code)
        assert 0 < nbytes <= _lib.DU_NOALLOC_SCRATCH_BYTES
        out = torch.full((B, Hq, D), float("nan"), dtype=dtype, device="cuda")
        rc = lib.du_decode_noalloc(_p(q), _p(k), _p(v), _p(cos), _p(sin), _p(out),
                                   B, Hq, Hkv, L, D, code, D ** -0.5, L + 1, _stream())
        _lib.check(rc, "du_decode_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert max_abs(out, ref) <= OUT_TOL
    assert_no_device_timeouts()


def test_noalloc_scratch_covers_every_planned_split(cuda_device):
    """A unit is spread over at most a bounded number of CTAs, so the partials of any shape fit
    the fixed scratch (the refusal with DU_ERR_WORKSPACE stays as a guard)."""
    lib = _lib.load()
    worst = 0
    for D in (64, 128, 256):
        for B, Hq, Hkv in ((1, 8, 8), (1, 32, 8), (4, 32, 8), (8, 32, 32), (2, 64, 16), (1, 128, 32)):
            for L in (1000, 4096, 131072):
                worst = max(worst, lib.du_decode_workspace_size(B, Hq, Hkv, L, D))
    assert 0 < worst <= _lib.DU_NOALLOC_SCRATCH_BYTES
