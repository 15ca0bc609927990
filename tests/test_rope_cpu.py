"""Standalone RoPE: host-side contract and the oracle (no GPU).

Mirrors the reference's rope checks (``rope.py:96-121`` validation, ``:239-246`` torch
reference): the oracle's forward/backward pair is an exact transpose, the tables match the
reference builder, and the drop-in raises the reference's messages before any launch.
"""

import pytest
import torch

import rope
import oracle


def test_backward_is_the_transpose_of_forward():
    torch.manual_seed(0)
    x = torch.randn(2, 3, 37, 64, dtype=torch.float64)
    cos, sin = rope.make_half_split_pos_emb(37, 64, "cpu", torch.float64)
    y = oracle.apply_rope(x, cos, sin).double()
    back = oracle.apply_rope_backward(y, cos, sin).double()
    assert (back - x).abs().max().item() < 1e-5  # fp32 arithmetic inside the oracle
    # <R x, y> == <x, R^T y> for random x, y
    z = torch.randn_like(x)
    lhs = (oracle.apply_rope(x, cos, sin).double() * z).sum()
    rhs = (x * oracle.apply_rope_backward(z, cos, sin).double()).sum()
    assert abs(lhs.item() - rhs.item()) < 1e-3


def test_oracle_matches_reference_formula():
    """The reference's own torch restatement (rope.py:239-246), evaluated here in fp32."""
    torch.manual_seed(1)
    x = torch.randn(1, 2, 9, 32)
    cos, sin = rope.make_half_split_pos_emb(9, 32, "cpu", torch.float32)
    half = 16
    low, high = x[..., :half], x[..., half:]
    fwd = torch.cat((low * cos - high * sin, high * cos + low * sin), dim=-1)
    bwd = torch.cat((low * cos + high * sin, high * cos - low * sin), dim=-1)
    assert torch.equal(oracle.apply_rope(x, cos, sin), fwd)
    assert torch.equal(oracle.apply_rope_backward(x, cos, sin), bwd)


def test_tables_match_attention_tables():
    from dominusultra_b200 import precompute_rope_cos_sin

    c1, s1 = rope.make_half_split_pos_emb(100, 64, "cpu", torch.bfloat16)
    c2, s2 = precompute_rope_cos_sin(100, 64, "cpu", torch.bfloat16)
    assert torch.equal(c1, c2) and torch.equal(s1, s2)
    inter = rope.make_interleaved_pos_emb(10, 16, "cpu", torch.float32)
    c, s = rope.make_half_split_pos_emb(10, 16, "cpu", torch.float32)
    assert torch.equal(inter[:, 0::2], c) and torch.equal(inter[:, 1::2], s)


@pytest.mark.parametrize(
    "args,msg",
    [
        ((torch.zeros(2, 3, 4), torch.zeros(2, 3, 4)), "same rank-4"),
        ((torch.zeros(1, 2, 3, 64), torch.zeros(1, 2, 4, 64)), "same rank-4"),
        ((torch.zeros(1, 2, 3, 64), torch.zeros(1, 2, 3, 64)), "require CUDA"),
    ],
)
def test_validation_messages(args, msg):
    with pytest.raises(ValueError, match=msg):
        rope.apply_rope(*args)
    with pytest.raises(ValueError, match=msg):
        rope.apply_rope_backward(*args)


def test_table_arguments_validated():
    with pytest.raises(ValueError, match="seq_len"):
        rope.make_half_split_pos_emb(0, 64, "cpu")
    with pytest.raises(ValueError, match="even"):
        rope.make_half_split_pos_emb(4, 63, "cpu")
    with pytest.raises(ValueError, match="positive"):
        rope.make_half_split_pos_emb(4, 64, "cpu", base=0.0)
