"""Generate golden vectors from the reference implementation itself.

Run in a container that has the reference checkout (read-only) and Triton installed:

    python tests/golden/make_golden.py --reference /path/to/DominusUltra

It writes ``tests/golden/golden.npz`` with:

* RoPE tables from the reference's own ``precompute_rope_cos_sin`` (``dominus_ultra.py:25-58``)
  and ``rope.make_half_split_pos_emb`` (``rope.py:124-148``), run on CPU: these are the exact
  bits the product's table function must reproduce.
* Prefill and decode cases computed by the reference's Triton ``prefill_kernel``
  (``dominus_ultra.py:119-285``) and ``decode_kernel`` (``dominus_ultra.py:288-413``) under
  Triton's CPU interpreter (``TRITON_INTERPRET=1``), with seeded fp16 inputs. The interpreter
  cannot run the bf16 variants (it has no bf16 builder), so fp16 is the pinned dtype; bf16
  behaviour is pinned through the oracle, which these vectors pin.

The autotuner needs a GPU driver, so the kernels are launched through their undecorated JIT
function with one of the reference's own tile configs (``dominus_ultra.py:61-67``).
bf16 tensors are stored as their uint16 bit patterns.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent

# (B, Hq, Hkv, T, D): prefill cases, fp16. Includes GQA/MQA, T below/above and not a
# multiple of the tile, and every head_dim the reference accepts.
PREFILL_CASES = [
    (1, 2, 2, 64, 64),
    (1, 4, 2, 37, 64),
    (2, 4, 1, 100, 32),
    (1, 2, 1, 130, 128),
    (1, 2, 2, 17, 16),
    (1, 2, 2, 8, 64),
    (1, 2, 1, 1, 64),
    # both sides of the product's switch between its one-tile (T <= 4096) and two-tile prefill
    # kernels at head_dim 64, and head_dim 256
    (1, 1, 1, 4096, 64),
    (1, 1, 1, 4097, 64),
    (1, 2, 1, 100, 256),
]
# (B, Hq, Hkv, L, D): decode cases (one query at position L), fp16.
DECODE_CASES = [
    (2, 4, 4, 64, 64),
    (1, 8, 2, 257, 64),
    (2, 4, 1, 37, 128),
    (1, 2, 2, 1, 64),
    (1, 4, 2, 200, 32),
    (1, 2, 1, 19, 16),
    (1, 2, 1, 150, 256),
]
# (positions, dim, dtype name, base): RoPE table cases.
TABLE_CASES = [
    (17, 64, "float32", 10000.0),
    (19, 64, "float32", 10000.0),
    (7, 32, "float32", 10000.0),
    (129, 64, "bfloat16", 10000.0),
    (129, 128, "float16", 10000.0),
    (100, 128, "bfloat16", 500000.0),
    (64, 16, "bfloat16", 10000.0),
]


def _np(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True,
                        help="directory holding the reference module (dominus_ultra.py, rope.py)")
    parser.add_argument("--out", default=str(HERE / "golden.npz"))
    args = parser.parse_args()
    sys.path.insert(0, args.reference)

    import torch
    import triton  # type: ignore[import-untyped]

    import dominus_ultra as ref  # the reference module
    import rope as ref_rope  # the reference standalone RoPE module

    store = {}
    for i, (n, d, dt, base) in enumerate(TABLE_CASES):
        dtype = getattr(torch, dt)
        cos, sin = ref.precompute_rope_cos_sin(n, d, "cpu", dtype, base)
        store[f"table{i}_cos"] = _np(cos)
        store[f"table{i}_sin"] = _np(sin)
        rc, rs = ref_rope.make_half_split_pos_emb(n, d, "cpu", dtype, base)
        store[f"table{i}_rope_cos"] = _np(rc)
        store[f"table{i}_rope_sin"] = _np(rs)
        store[f"table{i}_meta"] = np.array([n, d, base], dtype=np.float64)
        store[f"table{i}_dtype"] = np.array(dt)

    dtype = torch.float16
    for i, (B, Hq, Hkv, T, D) in enumerate(PREFILL_CASES):
        g = torch.Generator().manual_seed(1000 + i)
        q = torch.randn(B, Hq, T, D, generator=g).to(dtype)
        k = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
        v = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
        cos, sin = ref.precompute_rope_cos_sin(T, D, "cpu", dtype)
        out = torch.empty_like(q)
        lse = torch.empty((B, Hq, T), dtype=torch.float32)
        bm = bn = 64
        ref.prefill_kernel.fn[(triton.cdiv(T, bm), B * Hq)](
            q, k, v, cos, sin, out, lse,
            *q.stride(), *k.stride(), *v.stride(), *out.stride(), *lse.stride(),
            B=B, H=Hq, KvH=Hkv, T=T, D=D, scale=1.0 / (D**0.5), BLOCK_M=bm, BLOCK_N=bn,
        )
        for name, t in (("q", q), ("k", k), ("v", v), ("cos", cos), ("sin", sin),
                        ("out", out), ("lse", lse)):
            store[f"prefill{i}_{name}"] = _np(t)
        store[f"prefill{i}_shape"] = np.array([B, Hq, Hkv, T, D])

    for i, (B, Hq, Hkv, L, D) in enumerate(DECODE_CASES):
        g = torch.Generator().manual_seed(2000 + i)
        q = torch.randn(B, Hq, 1, D, generator=g).to(dtype)
        kc = torch.randn(B, Hkv, L, D, generator=g).to(dtype)
        vc = torch.randn(B, Hkv, L, D, generator=g).to(dtype)
        cos, sin = ref.precompute_rope_cos_sin(L + 1, D, "cpu", dtype)
        out = torch.empty((B, Hq, D), dtype=dtype)
        qs = q.squeeze(2)
        ref.decode_kernel[(B * Hq,)](
            qs, kc, vc, cos, sin, out,
            *qs.stride(), *kc.stride(), *vc.stride(), *out.stride(),
            B=B, H=Hq, KvH=Hkv, past_T=L, D=D, scale=1.0 / (D**0.5),
        )
        for name, t in (("q", q), ("k", kc), ("v", vc), ("cos", cos), ("sin", sin),
                        ("out", out.unsqueeze(2))):
            store[f"decode{i}_{name}"] = _np(t)
        store[f"decode{i}_shape"] = np.array([B, Hq, Hkv, L, D])

    store["n_tables"] = np.array(len(TABLE_CASES))
    store["n_prefill"] = np.array(len(PREFILL_CASES))
    store["n_decode"] = np.array(len(DECODE_CASES))
    np.savez_compressed(args.out, **store)
    print(f"wrote {args.out} ({Path(args.out).stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
