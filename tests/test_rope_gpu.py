"""Standalone RoPE kernel (du_rope) against the fp32 oracle on the GPU.

One rounding on output: |ours - oracle| stays within one unit in the last place of the output
dtype (the reference's own check allows 2e-2 for bf16 and 6e-3 for fp16, rope.py:297).
"""

import ctypes

import pytest
import torch

import rope
from dominusultra_b200 import _lib
import oracle

from _helpers import assert_no_device_timeouts, randn

pytestmark = pytest.mark.gpu

ULP = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}


def _check(actual, expected, dtype):
    expected = expected.float()
    err = (actual.float().cpu() - expected).abs()
    bound = ULP[dtype] * expected.abs() + 1e-6
    assert (err <= bound).all(), f"max err {err.max().item():.3g}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [16, 32, 64, 128, 256])
def test_apply_rope_matches_oracle(cuda_device, dtype, D):
    B, H, T = 2, 3, 77
    q = randn((B, H, T, D), 10 + D, dtype)
    k = randn((B, H, T, D), 20 + D, dtype)
    cos, sin = rope.make_half_split_pos_emb(T, D, "cpu", dtype)
    out_q, out_k = rope.apply_rope(q.cuda(), k.cuda())
    torch.cuda.synchronize()
    assert out_q.dtype == dtype and out_q.shape == q.shape
    _check(out_q, oracle.apply_rope(q, cos, sin), dtype)
    _check(out_k, oracle.apply_rope(k, cos, sin), dtype)
    gq, gk = rope.apply_rope_backward(q.cuda(), k.cuda())
    torch.cuda.synchronize()
    _check(gq, oracle.apply_rope_backward(q, cos, sin), dtype)
    _check(gk, oracle.apply_rope_backward(k, cos, sin), dtype)
    assert_no_device_timeouts()


def test_forward_backward_round_trip_and_out_buffers(cuda_device):
    dtype = torch.float16
    q = randn((1, 4, 300, 64), 31, dtype).cuda()
    k = randn((1, 4, 300, 64), 32, dtype).cuda()
    oq, ok = torch.empty_like(q), torch.empty_like(k)
    rq, rk = rope.apply_rope(q, k, base=5e5, out_q=oq, out_k=ok)
    assert rq.data_ptr() == oq.data_ptr() and rk.data_ptr() == ok.data_ptr()
    bq, bk = rope.apply_rope_backward(rq, rk, base=5e5)
    torch.cuda.synchronize()
    # R^T R = I up to two fp16 roundings of values of size ~4
    assert (bq - q).abs().max().item() < 1e-2 and (bk - k).abs().max().item() < 1e-2
    with pytest.raises(ValueError, match="first output"):
        rope.apply_rope(q, k, out_q=torch.empty_like(q, dtype=torch.bfloat16))


def test_c_abi_position_offset_and_fp16_output(cuda_device):
    """du_rope at a position offset into a longer table, bf16 in -> fp16 out (the rotated-key
    operand of the prefill), in place of the reference's per-position loads."""
    B, H, T, D, off = 1, 2, 50, 128, 1000
    dtype = torch.bfloat16
    x = randn((B, H, T, D), 41, dtype)
    cos, sin = rope.make_half_split_pos_emb(off + T + 7, D, "cpu", dtype, base=5e5)
    out = torch.empty((B, H, T, D), dtype=torch.float16, device="cuda")
    xc, cc, sc = x.cuda(), cos.cuda(), sin.cuda()
    lib = _lib.load()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.du_rope(p(xc), p(cc), p(sc), p(out), B, H, T, D, _lib.DU_DTYPE_BF16, _lib.DU_DTYPE_F16,
                     off, cos.shape[0], 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "du_rope")
    torch.cuda.synchronize()
    _check(out, oracle.apply_rope(x, cos[off:off + T], sin[off:off + T]), torch.float16)
    # in place: out aliases x
    rc = lib.du_rope(p(xc), p(cc), p(sc), p(xc), B, H, T, D, _lib.DU_DTYPE_BF16, _lib.DU_DTYPE_BF16,
                     off, cos.shape[0], 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "du_rope")
    torch.cuda.synchronize()
    _check(xc, oracle.apply_rope(x, cos[off:off + T], sin[off:off + T]), dtype)
