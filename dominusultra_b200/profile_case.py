"""Run a few launches of one kernel on one configuration (for ncu captures).

    python -m dominusultra_b200.profile_case prefill --B 8 --H 32 --Hkv 32 --S 2048 --D 64
    python -m dominusultra_b200.profile_case decode  --B 8 --H 32 --Hkv 32 --L 2048 --D 64

Inputs are seeded N(0,1) bf16 on the device; `--iters` launches follow one warm-up launch.
Sizes should keep the inputs above the 126 MB L2 so DRAM counters are meaningful.
"""

from __future__ import annotations

import argparse

import torch

from . import dominus_ultra_decode, dominus_ultra_prefill, precompute_rope_cos_sin


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["prefill", "decode"])
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--H", type=int, default=32)
    ap.add_argument("--Hkv", type=int, default=32)
    ap.add_argument("--S", type=int, default=2048)
    ap.add_argument("--L", type=int, default=2048)
    ap.add_argument("--D", type=int, default=64)
    ap.add_argument("--base", type=float, default=10000.0)
    ap.add_argument("--iters", type=int, default=2)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    dt = torch.bfloat16
    if a.kernel == "prefill":
        q = torch.randn(a.B, a.H, a.S, a.D, generator=g, device=dev).to(dt)
        k = torch.randn(a.B, a.Hkv, a.S, a.D, generator=g, device=dev).to(dt)
        v = torch.randn(a.B, a.Hkv, a.S, a.D, generator=g, device=dev).to(dt)
        cos, sin = precompute_rope_cos_sin(a.S, a.D, dev, dt, a.base)
        for _ in range(1 + a.iters):
            dominus_ultra_prefill(q, k, v, cos, sin, a.Hkv)
    else:
        q = torch.randn(a.B, a.H, 1, a.D, generator=g, device=dev).to(dt)
        k = torch.randn(a.B, a.Hkv, a.L, a.D, generator=g, device=dev).to(dt)
        v = torch.randn(a.B, a.Hkv, a.L, a.D, generator=g, device=dev).to(dt)
        cos, sin = precompute_rope_cos_sin(a.L + 1, a.D, dev, dt, a.base)
        for _ in range(1 + a.iters):
            dominus_ultra_decode(q, k, v, cos, sin, a.Hkv)
    torch.cuda.synchronize()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
