# dominus_ultra.py
"""
Dominus Ultra -- causal attention with fused RoPE + GQA, B200-native (sm_100a).

Drop-in replacement for the reference's single-file module of the same name: it exports the
same three functions with the same signatures, argument meaning and errors, and keeps the
``python dominus_ultra.py --self-test`` entry point. The kernels are hand-written sm_100a CUDA
(tcgen05 tensor cores + TMEM + TMA for prefill, split-KV streaming for decode) in
``dominusultra_b200/csrc``, reached through the C ABI in ``include/dominus_ultra_b200.h``.
"""

from dominusultra_b200.attention import (  # noqa: F401
    _validate_attention_tensors,
    _validate_head_dim,
    _validate_rope_tables,
    dominus_ultra_decode,
    dominus_ultra_decode_kvcache,
    dominus_ultra_prefill,
    precompute_rope_cos_sin,
)

__all__ = ["precompute_rope_cos_sin", "dominus_ultra_prefill", "dominus_ultra_decode"]


def _main() -> int:
    """Small correctness self-test (reference behaviour: ``dominus_ultra.py:586-645``)."""
    import argparse

    import torch

    parser = argparse.ArgumentParser(
        prog="dominus_ultra",
        description=(
            "B200 sm_100a attention kernels (prefill/decode) with RoPE helpers. "
            "This module requires a CUDA B200 GPU to execute kernels."
        ),
    )
    parser.add_argument(
        "--self-test",
        action="store_true",
        help="Run a small correctness test (requires CUDA).",
    )
    args = parser.parse_args()

    if not args.self_test:
        parser.print_help()
        return 0

    if not torch.cuda.is_available():
        raise SystemExit("--self-test requires CUDA (torch.cuda.is_available() is false)")

    torch.manual_seed(42)
    device = "cuda"
    dtype = torch.bfloat16
    B, Hq, Hk, T, D = 1, 8, 8, 128, 64

    q = torch.randn(B, Hq, T, D, device=device, dtype=dtype) * 0.1
    k = torch.randn(B, Hk, T, D, device=device, dtype=dtype) * 0.1
    v = torch.randn(B, Hk, T, D, device=device, dtype=dtype) * 0.1
    cos, sin = precompute_rope_cos_sin(T, D, device, dtype)
    out, _lse = dominus_ultra_prefill(q, k, v, cos, sin, Hk)

    def apply_rope(x, cos, sin):
        x1 = x[..., : D // 2]
        x2 = x[..., D // 2 :]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    q_ref = apply_rope(q.to(torch.float32), cos, sin)
    k_ref = apply_rope(k.to(torch.float32), cos, sin)
    out_ref = torch.nn.functional.scaled_dot_product_attention(
        q_ref, k_ref, v.to(torch.float32), is_causal=True
    )
    diff = (out.to(torch.float32) - out_ref).abs().max().item()
    passed = torch.allclose(out.to(torch.float32), out_ref, atol=2.0e-2, rtol=2.0e-2)
    print(f"Max abs diff vs torch.sdpa (manual RoPE): {diff:.6f}")
    print(f"Correctness gate: {'PASS' if passed else 'FAIL'}")
    return 0 if passed else 1


if __name__ == "__main__":
    raise SystemExit(_main())
