"""du_decode_noalloc: decode for callers that cannot allocate device memory.

Some callers of this library cannot allocate device memory: a host that binds the C ABI from
another runtime with no CUDA allocator of its own, or a serving loop that must not call
cudaMalloc once it is running. For them ``du_decode_noalloc`` keeps the split-KV partials in
a fixed scratch array inside the library instead of a caller-provided workspace; the caller
still passes the inputs and the output.

These tests call it through the C ABI:

* two calls in a row on one stream, with different inputs and outputs and no synchronisation
  between them, each checked against the CPU oracle and against ``du_decode`` (which takes a
  workspace) within the parity tolerance of the other tests;
* a size whose partials need more than the fixed scratch is refused with DU_ERR_WORKSPACE
  before anything is launched (its output buffer stays untouched);
* the sizes the header promises to fit do fit.

The file is named to be collected last, and it passes alone in a fresh process as well as
after the other tests.
"""

import ctypes

import pytest
import torch

import oracle
from _helpers import OUT_TOL, assert_no_device_timeouts, max_abs, randn
from dominusultra_b200 import _lib, precompute_rope_cos_sin

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(B, Hq, Hkv, L, D, seed, dtype=torch.bfloat16):
    """CPU inputs (for the oracle) and their device copies."""
    q = randn((B, Hq, 1, D), seed, dtype)
    k = randn((B, Hkv, L, D), seed + 1, dtype)
    v = randn((B, Hkv, L, D), seed + 2, dtype)
    cos, sin = precompute_rope_cos_sin(L + 1, D, "cpu", dtype)
    host = (q, k, v, cos, sin)
    return host, tuple(t.cuda() for t in host)


def _decode_with_workspace(lib, dev_inputs, B, Hq, Hkv, L, D, code):
    q, k, v, cos, sin = dev_inputs
    out = torch.empty((B, Hq, D), dtype=q.dtype, device="cuda")
    nbytes = lib.du_decode_workspace_size(B, Hq, Hkv, L, D)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda") if nbytes else None
    rc = lib.du_decode(_p(q), _p(k), _p(v), _p(cos), _p(sin), _p(out), B, Hq, Hkv, L, D, code,
                       D ** -0.5, L + 1, _p(ws), nbytes, _stream())
    _lib.check(rc, "du_decode")
    return out, nbytes


def _noalloc(lib, dev_inputs, out, B, Hq, Hkv, L, D, code):
    q, k, v, cos, sin = dev_inputs
    return lib.du_decode_noalloc(_p(q), _p(k), _p(v), _p(cos), _p(sin), _p(out),
                                 B, Hq, Hkv, L, D, code, D ** -0.5, L + 1, _stream())


@pytest.mark.parametrize("B,Hq,Hkv,L,D,dtype", [
    # both take the split walk, so the partials go through the scratch array
    (2, 8, 2, 20000, 64, torch.bfloat16),   # CUDA-core kernel
    (1, 32, 8, 40000, 128, torch.float16),  # tensor-core kernel
])
def test_noalloc_decode_two_calls_in_a_row(cuda_device, B, Hq, Hkv, L, D, dtype):
    lib = _lib.load()
    code = _lib.DU_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DU_DTYPE_F16
    assert 0 < lib.du_decode_workspace_size(B, Hq, Hkv, L, D) <= _lib.DU_NOALLOC_SCRATCH_BYTES
    host_a, dev_a = _inputs(B, Hq, Hkv, L, D, 700, dtype)
    host_b, dev_b = _inputs(B, Hq, Hkv, L, D, 750, dtype)
    out_a = torch.full((B, Hq, D), float("nan"), dtype=dtype, device="cuda")
    out_b = torch.full((B, Hq, D), float("nan"), dtype=dtype, device="cuda")
    torch.cuda.synchronize()
    # Two calls back to back on one stream share the scratch array; stream order keeps the
    # second call's split kernel behind the first call's merge.
    _lib.check(_noalloc(lib, dev_a, out_a, B, Hq, Hkv, L, D, code), "du_decode_noalloc (1)")
    _lib.check(_noalloc(lib, dev_b, out_b, B, Hq, Hkv, L, D, code), "du_decode_noalloc (2)")
    torch.cuda.synchronize()
    ref_a, _ = _decode_with_workspace(lib, dev_a, B, Hq, Hkv, L, D, code)
    ref_b, _ = _decode_with_workspace(lib, dev_b, B, Hq, Hkv, L, D, code)
    torch.cuda.synchronize()
    for out, ref, host in ((out_a, ref_a, host_a), (out_b, ref_b, host_b)):
        assert torch.isfinite(out.float()).all()
        assert max_abs(out, ref) <= OUT_TOL
        assert max_abs(out, oracle.decode(*host, Hkv).squeeze(2)) <= OUT_TOL
    assert_no_device_timeouts()


def test_noalloc_refuses_sizes_beyond_the_scratch(cuda_device):
    """Partials of B 64 x Hq 32 rows at head_dim 256 need more than 4 MiB: refused with
    DU_ERR_WORKSPACE before any launch (real buffers are passed all the same)."""
    lib = _lib.load()
    B, Hq, Hkv, L, D = 64, 32, 8, 8192, 256
    need = lib.du_decode_workspace_size(B, Hq, Hkv, L, D)
    assert need > _lib.DU_NOALLOC_SCRATCH_BYTES
    dtype = torch.bfloat16
    q = torch.zeros((B, Hq, D), dtype=dtype, device="cuda")
    k = torch.zeros((B, Hkv, L, D), dtype=dtype, device="cuda")
    v = torch.zeros((B, Hkv, L, D), dtype=dtype, device="cuda")
    cos, sin = precompute_rope_cos_sin(L + 1, D, "cuda", dtype)
    out = torch.full((B, Hq, D), 3.0, dtype=dtype, device="cuda")
    torch.cuda.synchronize()
    rc = _noalloc(lib, (q, k, v, cos, sin), out, B, Hq, Hkv, L, D, _lib.DU_DTYPE_BF16)
    assert rc == _lib.DU_ERR_WORKSPACE
    msg = _lib.last_error()
    assert str(need) in msg and str(_lib.DU_NOALLOC_SCRATCH_BYTES) in msg
    torch.cuda.synchronize()
    assert bool((out == 3.0).all()), "a refused call must not launch"
    del k, v
    assert_no_device_timeouts()


def test_noalloc_scratch_covers_the_documented_sizes(cuda_device):
    """Every shape with head_dim <= 128, B <= 16 and Hq <= 128 fits the fixed scratch."""
    lib = _lib.load()
    worst = 0
    for D in (16, 32, 64, 128):
        for B in (1, 2, 4, 8, 16):
            for Hq in (1, 2, 4, 8, 16, 32, 64, 128):
                for Hkv in (h for h in (1, 2, 4, 8, 16, 32, 64, 128) if h <= Hq and Hq % h == 0):
                    for L in (1000, 4096, 16384, 131072, 1 << 20):
                        worst = max(worst, lib.du_decode_workspace_size(B, Hq, Hkv, L, D))
    assert 0 < worst <= _lib.DU_NOALLOC_SCRATCH_BYTES
