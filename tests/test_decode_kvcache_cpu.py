"""CPU checks of the KV-cache decode step: wrapper validation, C-ABI argument checks, and the
oracle's restatement against the plain decode oracle (no GPU needed)."""

from __future__ import annotations

import ctypes

import pytest
import torch

import oracle
from dominusultra_b200 import _lib, dominus_ultra_decode_kvcache, precompute_rope_cos_sin
from tests._helpers import randn


def _cpu(shape, dtype=torch.bfloat16):
    return torch.zeros(shape, dtype=dtype)


class TestKvcacheValidation:
    def test_rank(self):
        with pytest.raises(ValueError, match="rank-4"):
            dominus_ultra_decode_kvcache(_cpu((1, 2, 64)), _cpu((1, 2, 8, 64)), _cpu((1, 2, 8, 64)),
                                         None, None, torch.zeros(1, dtype=torch.int32))

    def test_new_kv_pairing(self):
        q, k = _cpu((1, 2, 1, 64)), _cpu((1, 2, 8, 64))
        with pytest.raises(ValueError, match="given together"):
            dominus_ultra_decode_kvcache(q, k, k, None, None, torch.zeros(1, dtype=torch.int32),
                                         k_new=_cpu((1, 2, 1, 64)))

    def test_new_kv_shape(self):
        q, k = _cpu((1, 2, 1, 64)), _cpu((1, 2, 8, 64))
        with pytest.raises(ValueError, match="k_new and v_new must have shape"):
            dominus_ultra_decode_kvcache(q, k, k, None, None, torch.zeros(1, dtype=torch.int32),
                                         k_new=_cpu((1, 2, 2, 64)), v_new=_cpu((1, 2, 2, 64)))

    def test_seqlens_shape_and_dtype(self):
        q, k = _cpu((2, 2, 1, 64)), _cpu((2, 2, 8, 64))
        with pytest.raises(ValueError, match=r"shape \[batch\]"):
            dominus_ultra_decode_kvcache(q, k, k, None, None, torch.zeros(3, dtype=torch.int32))
        with pytest.raises(ValueError, match="int32 or int64"):
            dominus_ultra_decode_kvcache(q, k, k, None, None, torch.zeros(2))

    def test_cache_shape(self):
        q = _cpu((1, 4, 1, 64))
        with pytest.raises(ValueError, match="matching GQA cache shapes"):
            dominus_ultra_decode_kvcache(q, _cpu((1, 2, 8, 64)), _cpu((1, 2, 9, 64)), None, None,
                                         torch.zeros(1, dtype=torch.int32), num_kv_heads=2)

    def test_cpu_tensors_rejected(self):
        q, k = _cpu((1, 2, 1, 64)), _cpu((1, 2, 8, 64))
        cos, sin = precompute_rope_cos_sin(9, 64, "cpu", torch.bfloat16)
        with pytest.raises(ValueError, match="require CUDA tensors"):
            dominus_ultra_decode_kvcache(q, k, k, cos, sin, torch.zeros(1, dtype=torch.int32))


def test_c_abi_kvcache_rejects_bad_arguments():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(0x10000)
    args = lambda **kw: dict(dict(q=fake, kn=null, vn=null, kc=fake, vc=fake, sl=fake, cos=fake,
                                  sin=fake, out=fake, B=2, Hq=8, Hkv=8, L=128, D=64,
                                  dt=_lib.DU_DTYPE_BF16, sc=0.125, rp=129, ws=fake,
                                  wsb=1 << 30), **kw)
    call = lambda a: lib.du_decode_kvcache(*a.values(), null)
    assert call(args(kn=fake)) == _lib.DU_ERR_INVALID and "together" in _lib.last_error()
    assert call(args(sl=ctypes.c_void_p(0x10002))) == _lib.DU_ERR_INVALID
    assert "4-byte" in _lib.last_error()
    assert call(args(B=0)) == _lib.DU_ERR_INVALID and "positive" in _lib.last_error()
    assert call(args(D=48)) == _lib.DU_ERR_UNSUPPORTED
    assert call(args(wsb=16)) == _lib.DU_ERR_WORKSPACE
    assert call(args(ws=ctypes.c_void_p(0x10010))) == _lib.DU_ERR_WORKSPACE
    assert call(args(sc=0.0)) == _lib.DU_ERR_INVALID


def test_kvcache_workspace_size_covers_fragment_slots():
    lib = _lib.load()
    small = lib.du_decode_kvcache_workspace_size(1, 8, 8, 128, 64)
    large = lib.du_decode_kvcache_workspace_size(64, 32, 8, 128, 128)
    assert 0 < small < large
    # offsets [B+1] int64, {len, qpos} [B], and (units + grid) * GT slots of D + 1 floats
    assert large >= 64 * 32 * 129 * 4
    assert lib.du_decode_kvcache_workspace_size(0, 8, 8, 128, 64) == 0


@pytest.mark.parametrize("append", [False, True])
def test_oracle_kvcache_matches_prefix_decode(append):
    """Each sequence of the KV-cache step is the reference decode of its own prefix."""
    B, H, Hkv, Lmax, D = 3, 4, 2, 40, 32
    q = randn((B, H, 1, D), 1)
    kc, vc = randn((B, Hkv, Lmax, D), 2), randn((B, Hkv, Lmax, D), 3)
    kn, vn = randn((B, Hkv, 1, D), 4), randn((B, Hkv, 1, D), 5)
    cos, sin = oracle.precompute_rope_cos_sin(Lmax + 1, D, torch.bfloat16)
    lens = [7, 0, Lmax - 1]
    out, kc2, vc2 = oracle.decode_kvcache(q, kc, vc, cos, sin, lens,
                                          kn if append else None, vn if append else None,
                                          num_kv_heads=Hkv)
    for b, s in enumerate(lens):
        if append:
            assert torch.equal(kc2[b, :, s], kn[b, :, 0]) and torch.equal(vc2[b, :, s], vn[b, :, 0])
            keep = [j for j in range(Lmax) if j != s]
            assert torch.equal(kc2[b, :, keep], kc[b, :, keep])
        else:
            assert torch.equal(kc2, kc) and torch.equal(vc2, vc)
        n = s + (1 if append else 0)
        if n == 0:
            assert torch.count_nonzero(out[b]) == 0
            continue
        # q at position s: for the no-append case this is exactly oracle.decode over the prefix
        ref, _ = oracle.decode_partial(q[b:b + 1], kc2[b:b + 1, :, :n], vc2[b:b + 1, :, :n], cos,
                                       sin, num_kv_heads=Hkv, q_pos=s)
        assert torch.allclose(out[b, :, 0], ref[0], atol=1e-6)
        if not append:
            full = oracle.decode(q[b:b + 1], kc[b:b + 1, :, :s], vc[b:b + 1, :, :s], cos, sin,
                                 num_kv_heads=Hkv)
            assert torch.allclose(out[b:b + 1], full, atol=1e-5)
