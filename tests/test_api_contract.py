"""Host-side contract of the drop-in API and the C ABI (runs without a GPU).

* the reference's CPU contract tests (``test_dominus.py:53-89``), run against this package;
* the reference's validation order and messages (``dominus_ultra.py:451-470``, ``:537-556``),
  including the rejection of CPU tensors (there is no CPU path);
* the shared library loads and exports every entry point ``include/dominus_ultra_b200.h``
  declares, and its argument validation rejects bad calls before any CUDA work.
"""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import dominus_ultra
from dominusultra_b200 import _lib
from rope import make_half_split_pos_emb

ROOT = Path(__file__).resolve().parent.parent
from dominus_ultra import (  # noqa: E402
    dominus_ultra_decode,
    dominus_ultra_prefill,
    precompute_rope_cos_sin,
)


class TestRoPECPUContract:
    def test_precompute_shape_and_origin(self):
        cos, sin = precompute_rope_cos_sin(17, 64, "cpu", torch.float32)
        assert cos.shape == (17, 32)
        assert sin.shape == (17, 32)
        assert torch.equal(cos[0], torch.ones(32))
        assert torch.equal(sin[0], torch.zeros(32))

    def test_precompute_matches_direct_frequency_formula(self):
        positions, dim, base = 7, 32, 10000.0
        cos, sin = precompute_rope_cos_sin(positions, dim, "cpu", base=base)
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        expected = torch.arange(positions, dtype=torch.float32)[:, None] * inv_freq[None, :]
        assert torch.allclose(cos, expected.cos())
        assert torch.allclose(sin, expected.sin())

    def test_standalone_and_fused_rope_tables_match(self):
        fused_cos, fused_sin = precompute_rope_cos_sin(19, 64, "cpu")
        rope_cos, rope_sin = make_half_split_pos_emb(19, 64, "cpu")
        assert torch.equal(fused_cos, rope_cos)
        assert torch.equal(fused_sin, rope_sin)

    @pytest.mark.parametrize(
        "max_seq_len,dim,base",
        [(0, 64, 10000.0), (8, 0, 10000.0), (8, 63, 10000.0), (8, 64, 0.0)],
    )
    def test_precompute_rejects_invalid_configuration(self, max_seq_len, dim, base):
        with pytest.raises(ValueError):
            precompute_rope_cos_sin(max_seq_len, dim, "cpu", base=base)


def _cpu(shape, dtype=torch.bfloat16):
    return torch.zeros(shape, dtype=dtype)


class TestPrefillValidation:
    def test_rank(self):
        with pytest.raises(ValueError, match="rank-4"):
            dominus_ultra_prefill(_cpu((2, 8, 64)), _cpu((2, 8, 64)), _cpu((2, 8, 64)), None, None)

    def test_positive(self):
        z = _cpu((0, 8, 16, 64))
        with pytest.raises(ValueError, match="must be positive"):
            dominus_ultra_prefill(z, z, z, None, None)

    def test_divisible(self):
        q = _cpu((1, 8, 16, 64))
        k = _cpu((1, 3, 16, 64))
        with pytest.raises(ValueError, match="divisible"):
            dominus_ultra_prefill(q, k, k, None, None, num_kv_heads=3)

    def test_kv_shape(self):
        q = _cpu((1, 8, 16, 64))
        k = _cpu((1, 2, 15, 64))
        with pytest.raises(ValueError, match="k and v must have shape"):
            dominus_ultra_prefill(q, k, k, None, None, num_kv_heads=2)

    def test_head_dim(self):
        q = _cpu((1, 2, 16, 48))
        with pytest.raises(ValueError, match="power of two"):
            dominus_ultra_prefill(q, q, q, None, None)

    def test_cpu_tensors_rejected(self):
        q = _cpu((1, 2, 16, 64))
        cos, sin = precompute_rope_cos_sin(16, 64, "cpu", torch.bfloat16)
        with pytest.raises(ValueError, match="require CUDA tensors"):
            dominus_ultra_prefill(q, q, q, cos, sin)

    def test_dtype_checked_after_device(self):
        q = _cpu((1, 2, 16, 64), torch.float32)
        with pytest.raises(ValueError, match="require CUDA tensors"):
            dominus_ultra_prefill(q, q, q, None, None)


class TestDecodeValidation:
    def test_one_position(self):
        q = _cpu((1, 2, 2, 64))
        k = _cpu((1, 2, 8, 64))
        with pytest.raises(ValueError, match="exactly one sequence position"):
            dominus_ultra_decode(q, k, k, None, None)

    def test_cache_shape(self):
        q = _cpu((1, 4, 1, 64))
        k = _cpu((1, 2, 8, 64))
        v = _cpu((1, 2, 9, 64))
        with pytest.raises(ValueError, match="matching GQA cache shapes"):
            dominus_ultra_decode(q, k, v, None, None, num_kv_heads=2)

    def test_shape_checked_before_head_count(self):
        # As in the reference, the cache-shape check fires before the head-count check.
        q = _cpu((1, 4, 1, 64))
        k = _cpu((1, 2, 8, 64))
        with pytest.raises(ValueError, match="matching GQA cache shapes"):
            dominus_ultra_decode(q, k, k, None, None, num_kv_heads=4)

    def test_cpu_tensors_rejected(self):
        q = _cpu((1, 2, 1, 64))
        k = _cpu((1, 2, 8, 64))
        cos, sin = precompute_rope_cos_sin(9, 64, "cpu", torch.bfloat16)
        with pytest.raises(ValueError, match="require CUDA tensors"):
            dominus_ultra_decode(q, k, k, cos, sin)


def _declared_functions():
    header = (ROOT / "include" / "dominus_ultra_b200.h").read_text()
    body = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    return sorted(set(re.findall(r"\b(du_[a-z_0-9]+)\s*\(", body)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_functions()
    assert len(declared) >= 8
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures must mirror the header"
    assert lib.du_version() >= 100


def test_c_abi_rejects_bad_arguments_before_launch():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(0x10000)
    rc = lib.du_prefill(fake, fake, fake, fake, fake, fake, fake, 0, 8, 8, 128, 64,
                        _lib.DU_DTYPE_BF16, 0.125, 128, null, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "positive" in _lib.last_error()
    rc = lib.du_prefill(fake, fake, fake, fake, fake, fake, fake, 1, 8, 3, 128, 64,
                        _lib.DU_DTYPE_BF16, 0.125, 128, null, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "divisible" in _lib.last_error()
    rc = lib.du_prefill(fake, fake, fake, fake, fake, fake, fake, 1, 8, 8, 128, 48,
                        _lib.DU_DTYPE_BF16, 0.125, 128, null, 0, null)
    assert rc == _lib.DU_ERR_UNSUPPORTED
    rc = lib.du_prefill(fake, fake, fake, fake, fake, fake, fake, 1, 8, 8, 128, 64,
                        _lib.DU_DTYPE_BF16, 0.125, 127, null, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "rope" in _lib.last_error()
    rc = lib.du_prefill(ctypes.c_void_p(0x10008), fake, fake, fake, fake, fake, fake, 1, 8, 8,
                        128, 64, _lib.DU_DTYPE_BF16, 0.125, 128, null, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "aligned" in _lib.last_error()
    rc = lib.du_decode(fake, fake, fake, fake, fake, fake, 1, 8, 8, 128, 64,
                       _lib.DU_DTYPE_F16, 0.125, 128, null, 0, null)
    assert rc == _lib.DU_ERR_INVALID and "positions" in _lib.last_error()
    rc = lib.du_merge_partials(fake, fake, 0, 4, 64, 0, 0, 0, 0, fake, _lib.DU_DTYPE_F32, null, null)
    assert rc == _lib.DU_ERR_INVALID
    # The no-allocation decode refuses sizes beyond its fixed scratch before any CUDA call
    # (sizes planned for 148 SMs, the B200's count and the fallback without a device).
    need = lib.du_decode_workspace_size(64, 32, 8, 8192, 256)
    assert need > _lib.DU_NOALLOC_SCRATCH_BYTES
    rc = lib.du_decode_noalloc(fake, fake, fake, fake, fake, fake, 64, 32, 8, 8192, 256,
                               _lib.DU_DTYPE_BF16, 0.0625, 8193, null)
    assert rc == _lib.DU_ERR_WORKSPACE and str(need) in _lib.last_error()


def test_exchange_merge_rejects_bad_arguments_before_launch():
    """The peer-memory exchange validates world, rank, sizes and its buffers before any CUDA
    call (the kernel itself needs every rank of the call; it runs in the 2-GPU tests)."""
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(0x10000)
    bufs = (ctypes.c_void_p * 2)(0x20000, 0x30000)
    assert lib.du_exchange_buffer_bytes(9, 128, 128) == 0
    assert lib.du_exchange_buffer_bytes(2, 128, 6) == 0
    assert lib.du_exchange_buffer_bytes(2, 128, 128) == 256 + 2 * 2 * 128 * 129 * 8
    rc = lib.du_exchange_merge(fake, fake, bufs, 9, 0, 128, 128, fake, _lib.DU_DTYPE_BF16, null, null)
    assert rc == _lib.DU_ERR_UNSUPPORTED
    rc = lib.du_exchange_merge(fake, fake, bufs, 2, 2, 128, 128, fake, _lib.DU_DTYPE_BF16, null, null)
    assert rc == _lib.DU_ERR_INVALID and "rank" in _lib.last_error()
    rc = lib.du_exchange_merge(fake, fake, bufs, 2, 0, 128, 130, fake, _lib.DU_DTYPE_BF16, null, null)
    assert rc == _lib.DU_ERR_INVALID
    bad = (ctypes.c_void_p * 2)(0x20000, 0x30010)  # not 256-byte aligned
    rc = lib.du_exchange_merge(fake, fake, bad, 2, 0, 128, 128, fake, _lib.DU_DTYPE_BF16, null, null)
    assert rc == _lib.DU_ERR_INVALID and "aligned" in _lib.last_error()
    rc = lib.du_exchange_merge(fake, fake, bufs, 2, 0, 128, 128, fake, 7, null, null)
    assert rc == _lib.DU_ERR_INVALID and "out_dtype" in _lib.last_error()


def test_workspace_size_is_consistent():
    lib = _lib.load()
    assert lib.du_decode_workspace_size(8, 32, 32, 128, 64) == 0  # one split per row
    big = lib.du_decode_workspace_size(4, 32, 8, 16384, 128)
    assert big > 0 and big % 4 == 0
    assert lib.du_decode_workspace_size(0, 32, 8, 128, 64) == 0


def test_dropin_module_surface():
    """Everything the reference's test file imports (test_dominus.py:16-21) is importable from
    the same module names."""
    for name in ("precompute_rope_cos_sin", "dominus_ultra_prefill", "dominus_ultra_decode"):
        assert callable(getattr(dominus_ultra, name))
    assert callable(dominus_ultra._main)
    import rope

    assert callable(rope.make_half_split_pos_emb)
