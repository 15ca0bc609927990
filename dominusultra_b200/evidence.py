"""Correctness-gated GPU evidence in the reference's ``dominus-ultra-evidence-v1`` format.

The reference publishes GPU results as a JSON report (``gpu_evidence.py:35``, ``:506-523``):
``{"schema_version", "payload_sha256", "payload"}`` where the payload holds the verdict, suite,
dtypes, warm-up / iteration counts, seed, environment metadata and one result per (case,
dtype), and the SHA-256 is taken over the canonical JSON of the payload (sorted keys, compact
separators, ASCII). This module produces the same schema from this build's kernels so that
results line up with the reference's protocol (``docs/EVIDENCE_PROTOCOL.md``): the same case
labels (``mode:B:Hq:Hkv:T:D``), the same input scaling (N(0,1) x 0.1), the same fp32 SDPA
correctness reference and tolerances, and PyTorch SDPA with RoPE applied outside the timed
region as the timing baseline.

    python -m dominusultra_b200.evidence --suite quick --output-dir evidence_results
"""

from __future__ import annotations

import argparse
import gc
import hashlib
import json
import os
import platform
import shlex
import statistics
import subprocess
import sys
from dataclasses import asdict, dataclass
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, Callable, Dict, List, Sequence, Tuple

import torch
import torch.nn.functional as F

SCHEMA_VERSION = "dominus-ultra-evidence-v1"
REPOSITORY = "https://github.com/MiMindMendinc/DominusUltra"


@dataclass(frozen=True)
class EvidenceCase:
    mode: str
    batch_size: int
    num_heads: int
    num_kv_heads: int
    context_length: int
    head_dim: int

    @property
    def label(self) -> str:
        return (f"{self.mode}:B{self.batch_size}:Hq{self.num_heads}:Hkv{self.num_kv_heads}:"
                f"T{self.context_length}:D{self.head_dim}")


# The reference's suites (gpu_evidence.py:55-70): same shapes, same order.
QUICK_CASES: Tuple[EvidenceCase, ...] = tuple(
    EvidenceCase(*c) for c in (
        ("prefill", 1, 8, 8, 128, 64), ("prefill", 1, 8, 2, 257, 64),
        ("decode", 2, 8, 8, 128, 64), ("decode", 2, 8, 2, 257, 64),
    ))
FULL_CASES: Tuple[EvidenceCase, ...] = QUICK_CASES + tuple(
    EvidenceCase(*c) for c in (
        ("prefill", 1, 16, 16, 512, 64), ("prefill", 1, 16, 4, 1024, 64),
        ("prefill", 1, 8, 2, 512, 128), ("decode", 4, 16, 16, 512, 64),
        ("decode", 4, 16, 4, 1024, 64), ("decode", 2, 8, 2, 512, 128),
    ))


def tolerances(dtype_name: str) -> Dict[str, float]:
    """The reference protocol's pass thresholds (gpu_evidence.py:185-188)."""
    if dtype_name == "bfloat16":
        return {"atol": 2.0e-2, "rtol": 2.0e-2, "lse_atol": 5.0e-2}
    return {"atol": 6.0e-3, "rtol": 6.0e-3, "lse_atol": 2.0e-2}


def latency_stats(samples_ms: List[float]) -> Dict[str, Any]:
    ordered = sorted(samples_ms)
    p95 = ordered[min(len(ordered) - 1, max(0, int(0.95 * len(ordered)) - 1))]
    return {"samples_ms": samples_ms, "mean_ms": statistics.mean(samples_ms),
            "median_ms": statistics.median(samples_ms), "p95_ms": p95,
            "std_ms": statistics.pstdev(samples_ms), "min_ms": ordered[0], "max_ms": ordered[-1]}


def error_metrics(actual: torch.Tensor, expected: torch.Tensor) -> Dict[str, float]:
    delta = actual.float() - expected.float()
    return {"max_abs": delta.abs().max().item(), "mean_abs": delta.abs().mean().item(),
            "rmse": delta.square().mean().sqrt().item()}


def canonical_sha256(payload: Dict[str, Any]) -> str:
    """SHA-256 of the payload's canonical JSON (sorted keys, compact, ASCII)."""
    blob = json.dumps(payload, sort_keys=True, separators=(",", ":"), ensure_ascii=True)
    return hashlib.sha256(blob.encode("utf-8")).hexdigest()


def make_report(payload: Dict[str, Any]) -> Dict[str, Any]:
    return {"schema_version": SCHEMA_VERSION, "payload_sha256": canonical_sha256(payload),
            "payload": payload}


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    return torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1)


def _events(fn: Callable[[], Any], warmup: int, iterations: int) -> Dict[str, Any]:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    pairs = []
    for _ in range(iterations):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        pairs.append((a, b))
    torch.cuda.synchronize()
    return latency_stats([a.elapsed_time(b) for a, b in pairs])


def _case_result(case: EvidenceCase, dtype_name: str, warmup: int, iterations: int) -> Dict[str, Any]:
    from . import dominus_ultra_decode, dominus_ultra_prefill, precompute_rope_cos_sin

    dtype = torch.bfloat16 if dtype_name == "bfloat16" else torch.float16
    tol = tolerances(dtype_name)
    B, Hq, Hkv, T, D = (case.batch_size, case.num_heads, case.num_kv_heads, case.context_length,
                        case.head_dim)
    group = Hq // Hkv
    prefill = case.mode == "prefill"
    q = torch.randn(B, Hq, T if prefill else 1, D, device="cuda", dtype=dtype) * 0.1
    k = torch.randn(B, Hkv, T, D, device="cuda", dtype=dtype) * 0.1
    v = torch.randn(B, Hkv, T, D, device="cuda", dtype=dtype) * 0.1
    cos, sin = precompute_rope_cos_sin(T if prefill else T + 1, D, "cuda", dtype)
    ke, ve = k.repeat_interleave(group, dim=1), v.repeat_interleave(group, dim=1)
    qc, qs = (cos, sin) if prefill else (cos[T:T + 1], sin[T:T + 1])
    kc, ks = (cos, sin) if prefill else (cos[:T], sin[:T])
    q_ref = _rope(q.float(), qc.float(), qs.float())
    k_ref = _rope(ke.float(), kc.float(), ks.float())
    out_ref = F.scaled_dot_product_attention(q_ref, k_ref, ve.float(), is_causal=prefill)
    correctness: Dict[str, Any] = {"tolerances": tol}
    if prefill:
        out, lse = dominus_ultra_prefill(q, k, v, cos, sin, num_kv_heads=Hkv)
        scores = torch.matmul(q_ref, k_ref.transpose(-2, -1)) / (D ** 0.5)
        mask = torch.ones((T, T), device="cuda", dtype=torch.bool).triu(1)
        lse_ref = torch.logsumexp(scores.masked_fill(mask, -float("inf")), dim=-1)
        correctness["lse_pass"] = torch.allclose(lse, lse_ref, atol=tol["lse_atol"], rtol=tol["rtol"])
        correctness["lse_error"] = error_metrics(lse, lse_ref)
    else:
        out = dominus_ultra_decode(q, k, v, cos, sin, num_kv_heads=Hkv)
    correctness["output_pass"] = torch.allclose(out.float(), out_ref, atol=tol["atol"], rtol=tol["rtol"])
    correctness["output_error"] = error_metrics(out, out_ref)
    passed = correctness["output_pass"] and correctness.get("lse_pass", True)

    q_t, k_t = _rope(q, qc, qs), _rope(ke, kc, ks)  # RoPE outside the baseline's timed region
    if prefill:
        kernel = _events(lambda: dominus_ultra_prefill(q, k, v, cos, sin, num_kv_heads=Hkv), warmup, iterations)
    else:
        kernel = _events(lambda: dominus_ultra_decode(q, k, v, cos, sin, num_kv_heads=Hkv), warmup, iterations)
    base = _events(lambda: F.scaled_dot_product_attention(q_t, k_t, ve, is_causal=prefill), warmup, iterations)
    positions = B * T if prefill else B
    return {
        "case": asdict(case), "label": case.label, "dtype": dtype_name,
        "status": "pass" if passed else "fail",
        "correctness": correctness,
        "timing_method": "CUDA events; compile/autotune excluded by warmup",
        "baseline": "PyTorch SDPA with RoPE precomputed outside the timed region",
        "kernel": kernel, "baseline_timing": base,
        "speedup_median": base["median_ms"] / kernel["median_ms"],
        "kernel_token_positions_per_second": positions / (kernel["median_ms"] / 1000.0),
        "baseline_token_positions_per_second": positions / (base["median_ms"] / 1000.0),
        "peak_memory_allocated_bytes": torch.cuda.max_memory_allocated(),
    }


def run_case(case: EvidenceCase, dtype_name: str, warmup: int, iterations: int, seed: int) -> Dict[str, Any]:
    gc.collect()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    torch.manual_seed(seed)
    torch.cuda.manual_seed_all(seed)
    try:
        return _case_result(case, dtype_name, warmup, iterations)
    except Exception as error:  # recorded as evidence, like a failed tolerance
        return {"case": asdict(case), "label": case.label, "dtype": dtype_name, "status": "error",
                "error_type": type(error).__name__, "error": str(error)[:4000]}


def _cmd(args: Sequence[str]) -> str:
    try:
        r = subprocess.run(args, check=False, capture_output=True, text=True, timeout=10)
    except (OSError, subprocess.TimeoutExpired):
        return "unavailable"
    return (r.stdout.strip() or r.stderr.strip()) or "unavailable"


def environment(command: str) -> Dict[str, Any]:
    root = Path(__file__).resolve().parent.parent
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    status = _cmd(("git", "-C", str(root), "status", "--porcelain"))
    sources = [root / "dominus_ultra.py", root / "include" / "dominus_ultra_b200.h",
               *sorted((root / "dominusultra_b200" / "csrc").glob("*"))]
    return {
        "generated_at": datetime.now(timezone.utc).isoformat(),
        "repository": REPOSITORY,
        "implementation": "dominusultra_b200 (sm_100a CUDA behind a C ABI)",
        "command": command,
        "python": platform.python_version(),
        "python_implementation": platform.python_implementation(),
        "platform": platform.platform(),
        "torch": torch.__version__,
        "torch_git_version": getattr(torch.version, "git_version", "unknown"),
        "cuda_runtime": torch.version.cuda,
        "cudnn": torch.backends.cudnn.version(),
        "device_index": torch.cuda.current_device(),
        "device_name": props.name,
        "compute_capability": f"{props.major}.{props.minor}",
        "total_memory_bytes": props.total_memory,
        "multiprocessor_count": props.multi_processor_count,
        "bf16_supported": torch.cuda.is_bf16_supported(),
        "nvidia_smi": _cmd(("nvidia-smi", "--query-gpu=index,name,driver_version,memory.total",
                            "--format=csv,noheader,nounits")),
        "tracked_environment": {k: os.environ[k] for k in ("CUDA_VISIBLE_DEVICES",) if k in os.environ},
        "git": {"commit": _cmd(("git", "-C", str(root), "rev-parse", "HEAD")),
                "branch": _cmd(("git", "-C", str(root), "branch", "--show-current")),
                "dirty": status not in ("", "unavailable")},
        "source_sha256": {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest()
                          for p in sources if p.is_file()},
    }


def markdown(report: Dict[str, Any]) -> str:
    p = report["payload"]
    env = p["environment"]
    lines = [
        "# DominusUltra GPU evidence", "",
        f"- Schema: `{report['schema_version']}`",
        f"- Payload SHA-256: `{report['payload_sha256']}`",
        f"- Verdict: **{p['verdict'].upper()}**",
        f"- Device: {env['device_name']} (sm_{env['compute_capability'].replace('.', '')}), "
        f"{env['multiprocessor_count']} SMs",
        f"- Implementation: {env['implementation']}; commit `{env['git']['commit']}`",
        "", "| case | dtype | status | kernel median ms | SDPA median ms | speedup |",
        "|---|---|---|---|---|---|",
    ]
    for r in p["results"]:
        if r["status"] == "error":
            lines.append(f"| `{r['label']}` | {r['dtype']} | ERROR | — | — | — |")
            continue
        lines.append(f"| `{r['label']}` | {r['dtype']} | {r['status'].upper()} | "
                     f"{r['kernel']['median_ms']:.4f} | {r['baseline_timing']['median_ms']:.4f} | "
                     f"{r['speedup_median']:.3f}x |")
    lines += ["", "Throughput here is token positions per isolated call, not end-to-end generation "
              "speed; raw samples and error metrics are in the JSON file.", ""]
    return "\n".join(lines)


def write_report(output_dir: Path, payload: Dict[str, Any]) -> Tuple[Path, Path, str]:
    report = make_report(payload)
    stamp = datetime.now(timezone.utc).strftime("%Y%m%dT%H%M%SZ")
    output_dir.mkdir(parents=True, exist_ok=True)
    json_path = output_dir / f"dominus-ultra-evidence-{stamp}.json"
    md_path = output_dir / f"dominus-ultra-evidence-{stamp}.md"
    json_path.write_text(json.dumps(report, indent=2) + "\n", encoding="utf-8")
    md_path.write_text(markdown(report), encoding="utf-8")
    return json_path, md_path, report["payload_sha256"]


def main(argv: Sequence[str] = ()) -> int:
    ap = argparse.ArgumentParser(description="Correctness-gated GPU evidence (dominus-ultra-evidence-v1)")
    ap.add_argument("--suite", choices=("quick", "full"), default="quick")
    ap.add_argument("--dtype", choices=("auto", "float16", "bfloat16", "both"), default="auto")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--iterations", type=int, default=50)
    ap.add_argument("--seed", type=int, default=20260811)
    ap.add_argument("--output-dir", type=Path, default=Path("evidence_results"))
    args = ap.parse_args(list(argv) or None)
    if args.warmup < 1 or args.iterations < 2:
        print("--warmup must be >= 1 and --iterations must be >= 2", file=sys.stderr)
        return 2
    if not torch.cuda.is_available():
        print("CUDA is required; torch.cuda.is_available() returned false", file=sys.stderr)
        return 2
    dtypes = {"auto": ("bfloat16",), "both": ("float16", "bfloat16")}.get(args.dtype, (args.dtype,))
    cases = QUICK_CASES if args.suite == "quick" else FULL_CASES
    results: List[Dict[str, Any]] = []
    for di, dt in enumerate(dtypes):
        for ci, case in enumerate(cases):
            results.append(run_case(case, dt, args.warmup, args.iterations, args.seed + di * 10_000 + ci))
            print(f"[{len(results)}/{len(cases) * len(dtypes)}] {case.label} {dt} -> "
                  f"{results[-1]['status'].upper()}")
    payload = {
        "verdict": "pass" if all(r["status"] == "pass" for r in results) else "fail",
        "suite": args.suite, "dtypes": list(dtypes), "warmup": args.warmup,
        "iterations": args.iterations, "seed": args.seed,
        "environment": environment(shlex.join((sys.executable, "-m", "dominusultra_b200.evidence", *(argv or sys.argv[1:])))),
        "results": results,
    }
    json_path, md_path, sha = write_report(args.output_dir, payload)
    print(f"Verdict: {payload['verdict'].upper()}\nPayload SHA-256: {sha}\nJSON: {json_path}\nMarkdown: {md_path}")
    return 0 if payload["verdict"] == "pass" else 1


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1:]))
