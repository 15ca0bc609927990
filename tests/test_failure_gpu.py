"""Failure detection on the GPU without a fault, a trap or a hang.

Every wait in the kernels is bounded; when one runs out the kernel records an error in the
library's status words and returns, and the host reads it with du_read_status. Here a
self-test kernel waits on an mbarrier that nothing ever arrives at, with a 20 ms limit: the
test checks the recorded status and that the CUDA context still runs the real kernels
correctly afterwards.
"""

import ctypes

import pytest
import torch

import oracle
from _helpers import LSE_TOL, OUT_TOL, max_abs, randn
from dominusultra_b200 import _lib, dominus_ultra_prefill, precompute_rope_cos_sin

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda_device):
    lib = _lib.load()
    _lib.read_status(reset=True)
    rc = lib.du_selftest_wait_timeout(20000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "du_selftest_wait_timeout")
    torch.cuda.synchronize()
    words = _lib.read_status(reset=True)
    assert words[0] == _lib.DU_ERR_TIMEOUT and words[1] == 200, words
    assert _lib.read_status(reset=True)[0] == 0  # reset took effect

    # the context is intact: a normal prefill still matches the oracle
    B, H, T, D = 1, 2, 300, 64
    q, k, v = (randn((B, H, T, D), s, torch.bfloat16) for s in (1, 2, 3))
    cos, sin = precompute_rope_cos_sin(T, D, "cpu", torch.bfloat16)
    out, lse = dominus_ultra_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda())
    ref_o, ref_l = oracle.prefill(q, k, v, cos, sin, H)
    assert max_abs(out, ref_o) <= OUT_TOL and max_abs(lse, ref_l) <= LSE_TOL
    assert _lib.read_status(reset=True)[0] == 0


def test_selftest_rejects_bad_limits(cuda_device):
    lib = _lib.load()
    assert lib.du_selftest_wait_timeout(0, None) == _lib.DU_ERR_INVALID
    assert lib.du_selftest_wait_timeout(2000000, None) == _lib.DU_ERR_INVALID
