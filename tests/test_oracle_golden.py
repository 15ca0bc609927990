"""Pin the CPU oracle (and the RoPE tables) to golden vectors made by the reference itself.

``tests/golden/golden.npz`` was produced by ``tests/golden/make_golden.py`` from the reference's
own ``precompute_rope_cos_sin`` / ``rope.make_half_split_pos_emb`` (bit-exact targets) and its
Triton ``prefill_kernel`` / ``decode_kernel`` run under Triton's CPU interpreter in fp16. The
reference kernels rotate and cast P in fp16, the oracle works in fp32, so the pin is a
tolerance: out within 4e-3 and LSE within 2e-3 (observed: <= 1.3e-3 and <= 8.1e-4).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import rope
from dominusultra_b200 import precompute_rope_cos_sin

GOLDEN = np.load(Path(__file__).parent / "golden" / "golden.npz")
OUT_TOL = 4e-3
LSE_TOL = 2e-3


def _t(name: str, dtype=None) -> torch.Tensor:
    a = GOLDEN[name]
    if a.dtype == np.uint16:
        return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


def _table_dtype(i):
    return getattr(torch, str(GOLDEN[f"table{i}_dtype"]))


@pytest.mark.parametrize("i", range(int(GOLDEN["n_tables"])))
def test_product_tables_bit_exact(i):
    n, d, base = GOLDEN[f"table{i}_meta"]
    dtype = _table_dtype(i)
    cos, sin = precompute_rope_cos_sin(int(n), int(d), "cpu", dtype, float(base))
    assert torch.equal(cos, _t(f"table{i}_cos").to(dtype))
    assert torch.equal(sin, _t(f"table{i}_sin").to(dtype))
    rc, rs = rope.make_half_split_pos_emb(int(n), int(d), "cpu", dtype, float(base))
    assert torch.equal(rc, _t(f"table{i}_rope_cos").to(dtype))
    assert torch.equal(rs, _t(f"table{i}_rope_sin").to(dtype))


@pytest.mark.parametrize("i", range(int(GOLDEN["n_tables"])))
def test_oracle_tables_bit_exact(i):
    n, d, base = GOLDEN[f"table{i}_meta"]
    dtype = _table_dtype(i)
    cos, sin = oracle.precompute_rope_cos_sin(int(n), int(d), dtype, float(base))
    assert torch.equal(cos, _t(f"table{i}_cos").to(dtype))
    assert torch.equal(sin, _t(f"table{i}_sin").to(dtype))


@pytest.mark.parametrize("i", range(int(GOLDEN["n_prefill"])))
def test_oracle_prefill_matches_reference_kernel(i):
    B, Hq, Hkv, T, D = (int(x) for x in GOLDEN[f"prefill{i}_shape"])
    q, k, v, c, s = (_t(f"prefill{i}_{n}") for n in ("q", "k", "v", "cos", "sin"))
    out, lse = oracle.prefill(q, k, v, c, s, Hkv)
    assert (out - _t(f"prefill{i}_out").float()).abs().max().item() <= OUT_TOL
    assert (lse - _t(f"prefill{i}_lse")).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("i", range(int(GOLDEN["n_decode"])))
def test_oracle_decode_matches_reference_kernel(i):
    B, Hq, Hkv, L, D = (int(x) for x in GOLDEN[f"decode{i}_shape"])
    q, k, v, c, s = (_t(f"decode{i}_{n}") for n in ("q", "k", "v", "cos", "sin"))
    out = oracle.decode(q, k, v, c, s, Hkv)
    assert (out - _t(f"decode{i}_out").float()).abs().max().item() <= OUT_TOL
    part, _ = oracle.decode_partial(q, k, v, c, s, Hkv)
    assert (part - out[:, :, 0]).abs().max().item() <= 1e-5


def test_pin_detects_a_planted_rope_mistake(monkeypatch):
    """A wrong rotation sign in the oracle must fail the pin (the pin has teeth)."""
    i = 0
    B, Hq, Hkv, T, D = (int(x) for x in GOLDEN[f"prefill{i}_shape"])
    q, k, v, c, s = (_t(f"prefill{i}_{n}") for n in ("q", "k", "v", "cos", "sin"))

    def wrong_rope(x, cos, sin):
        x = x.float()
        h = x.shape[-1] // 2
        x1, x2 = x[..., :h], x[..., h:]
        return torch.cat([x1 * cos.float() + x2 * sin.float(), x2 * cos.float() - x1 * sin.float()], -1)

    monkeypatch.setattr(oracle.oracle, "apply_rope", wrong_rope)
    out, lse = oracle.oracle.prefill(q, k, v, c, s, Hkv)
    err = max(
        (out - _t(f"prefill{i}_out").float()).abs().max().item(),
        (lse - _t(f"prefill{i}_lse")).abs().max().item(),
    )
    assert err > 10 * OUT_TOL


def test_merge_identity_matches_full_decode():
    """Splitting the cache and merging partials reproduces the unsplit oracle."""
    g = torch.Generator().manual_seed(7)
    B, Hq, Hkv, L, D = 2, 4, 2, 301, 64
    q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16)
    cos, sin = oracle.precompute_rope_cos_sin(L + 1, D, torch.bfloat16)
    full = oracle.decode(q, k, v, cos, sin, Hkv)[:, :, 0]
    cuts = [0, 100, 101, 250, L]
    parts = [
        oracle.decode_partial(q, k[:, :, a:b], v[:, :, a:b], cos, sin, Hkv, q_pos=L, kv_pos_offset=a)
        for a, b in zip(cuts[:-1], cuts[1:])
    ]
    merged, _ = oracle.merge_partials([p[0] for p in parts], [p[1] for p in parts])
    assert (merged - full).abs().max().item() <= 1e-5
