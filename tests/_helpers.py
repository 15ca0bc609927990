"""Shared helpers for the GPU parity tests: seeded inputs and the gates."""

from __future__ import annotations

import torch

from dominusultra_b200 import _lib

OUT_TOL = 2e-2  # max-abs on outputs (bf16/fp16) vs the fp32 oracle
LSE_TOL = 1e-3  # max-abs on the fp32 natural-log LSE vs the fp32 oracle


def randn(shape, seed: int, dtype=torch.bfloat16, scale: float = 1.0) -> torch.Tensor:
    """Seeded N(0, 1) values drawn in fp32 on the CPU, then cast (inputs are identical
    for the kernel and the oracle)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g, dtype=torch.float32)
    if scale != 1.0:
        x = x * scale
    return x.to(dtype)


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


def assert_no_device_timeouts() -> None:
    words = _lib.read_status(reset=True)
    assert words[0] == 0, f"device-side bounded wait expired: status words {words}"
