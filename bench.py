"""Benchmark of the fused-RoPE causal attention hot path on B200.

One JSON line on rank 0. Headline: causal bf16 prefill TFLOP/s on the MHA sweep's largest
configuration (B=2, H=Hkv=32, S=2048, D=64, RoPE base 1e4); a step is one
``dominus_ultra_prefill`` call over one batch. A secondary ``decode`` object reports the decode
sweep's largest configuration (B=8, H=Hkv=32, cache L=2048, D=64) in KV-cache HBM GB/s.

* ``value``: device time (CUDA events, max over ranks) with inputs resident in HBM. Each step
  reads a different one of several input sets whose total exceeds the 126 MB L2, so every step
  streams from HBM (``config.l2``).
* ``e2e``: the same metric through the public API with pinned host buffers: host->device copy
  of q/k/v, the call, and a device->host read of out/lse inside the timed region.
* ``roofline``: algorithmic FLOPs (4*B*H*D*S(S+1)/2) per launch over the kernel's mean launch
  time, against the measured dense bf16 peak (``MEASURED_PEAKS.json``).
* ``cpu_baseline``: the fp32 torch reference path (RoPE then SDPA, the reference's oracle) on
  the host cores, rank 0 only.
* Multi-GPU (torchrun): weak scaling; every rank runs the per-GPU workload on its own
  (batch, kv-head) units with no communication, time = max over ranks.
* ``prefill_p5``: the Llama-3-8B-shaped prefill (B4 H32 Hkv8 S32768 D128) as one fixed job whose
  32 (batch, kv-head) units are split over the ranks (strong scaling, no communication), with
  its roofline against the sustained dense bf16 peak. ``decode_p5_shard``: the 16384-key shard
  each rank streams in the long-context decode at eight GPUs, against the HBM peak.
  ``decode_long``: that decode itself, the KV sequence split over the ranks, one NCCL
  all-gather and the LSE merge per step (strong scaling).

``--impl reference`` times the reference's CPU path (the oracle port) on the same config.
``--sweep`` prints one line per reference benchmark configuration instead (prefill P1-P3, the
decode sweep P4), each graph-timed over ``--steps`` calls on rotating input sets.
``--profile-case prefill|decode NAME=VALUE ...`` runs ``--steps`` calls of one configuration
and nothing else (the command the ncu summaries under profiles/ were taken with).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

PREFILL = dict(B=2, H=32, Hkv=32, S=2048, D=64, base=10000.0)
DECODE = dict(B=8, H=32, Hkv=32, L=2048, D=64, base=10000.0)
# Long-context Llama-3-8B-shaped decode: the KV sequence is split across the ranks.
DECODE_LONG = dict(B=4, H=32, Hkv=8, L=131072, D=128, base=500000.0)

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum, bytes) of the dominant
# kernel from the ncu captures summarised under profiles/ (prefill: prefill_fa1_kernel at the
# bench shape; decode: decode_kernel at the bench shape).
NCU_TRAFFIC = {"prefill": 50646784 + 14848, "decode": 134576128 + 5068032}


def headline_workload(cfg=None):
    """The headline configuration's name, identical in both arms of the bench."""
    c = cfg or PREFILL
    return (f"prefill B{c['B']} H{c['H']} Hkv{c['Hkv']} S{c['S']} D{c['D']} causal RoPE base 1e4 "
            "(per GPU)")


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def prefill_flops(B, H, S, D):
    return 4.0 * B * H * D * S * (S + 1) / 2.0


def decode_bytes(B, H, Hkv, L, D):
    return 2.0 * B * Hkv * L * D * 2 + 2.0 * B * H * D * 2 + 2.0 * (L + 1) * (D // 2) * 2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks
            self._nv = None

    _REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
        "sw_power_cap": 0x4,
    }

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        for name, bit in self._REASONS.items():
            if mask & bit:
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def start(self):
        if self._nv is None:
            return
        self._sample()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self):
        if self._nv is None:
            return None
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
        try:
            self._sample()
        except Exception:
            pass
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return dist, dist.get_rank(), world, local
    return None, 0, 1, 0


def barrier(dist):
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_prefill_sets(cfg, n_sets, seed, device, dtype=torch.bfloat16):
    from dominusultra_b200 import precompute_rope_cos_sin

    B, H, Hkv, S, D = cfg["B"], cfg["H"], cfg["Hkv"], cfg["S"], cfg["D"]
    g = torch.Generator(device=device).manual_seed(seed)
    sets = []
    for _ in range(n_sets):
        q = torch.randn(B, H, S, D, generator=g, device=device, dtype=torch.float32).to(dtype)
        k = torch.randn(B, Hkv, S, D, generator=g, device=device, dtype=torch.float32).to(dtype)
        v = torch.randn(B, Hkv, S, D, generator=g, device=device, dtype=torch.float32).to(dtype)
        sets.append((q, k, v))
    cos, sin = precompute_rope_cos_sin(S, D, device, dtype, cfg["base"])
    return sets, cos, sin


def time_region(fn, steps, stream):
    """Events around exactly `steps` calls of fn(i) on `stream`; returns total ms."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        fn(i)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def graph_time(fn, steps, stream):
    """Device time of exactly `steps` calls fn(i), launched as one CUDA graph replay (so host
    launch overhead is not in the number); returns total ms. `stream` is a side stream (graphs
    are not captured on the default stream); fn runs untimed on it once first so that nothing
    is allocated during the capture."""
    with torch.cuda.stream(stream):
        fn(0)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(steps):
            fn(i)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay launches on the current stream
        g.replay()
        stream.synchronize()
        start.record(stream)
        g.replay()
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end)
    del g
    return ms


def time_launches(fn, steps, stream):
    """Mean per-launch time: an event pair around each call."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        evs[i][0].record(stream)
        fn(i)
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in evs)


def rope_bytes(cfg):
    """Key-rotation pass traffic: read K (16-bit), write fp16 R(K), read the table rows."""
    B, Hkv, S, D = cfg["B"], cfg["Hkv"], cfg["S"], cfg["D"]
    return 2.0 * B * Hkv * S * D * 2 + 2.0 * S * (D // 2) * 2


def rope_pass_ms(sets, cos, sin, cfg, steps, stream):
    """Device ms of the prefill's key-rotation launch alone (du_rope, bf16 -> fp16, the same
    sizes and the same workspace as inside du_prefill)."""
    import ctypes

    from dominusultra_b200 import _lib
    from dominusultra_b200.attention import _cached_workspace

    lib = _lib.load()
    B, H, Hkv, S, D = cfg["B"], cfg["H"], cfg["Hkv"], cfg["S"], cfg["D"]
    ws, _ = _cached_workspace("prefill", int(lib.du_prefill_workspace_size(B, H, Hkv, S, D)),
                              cos.device, stream.cuda_stream)

    def one(i):
        k = sets[i % len(sets)][1]
        rc = lib.du_rope(ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(cos.data_ptr()),
                         ctypes.c_void_p(sin.data_ptr()), ctypes.c_void_p(ws), B, Hkv, S, D,
                         _lib.DU_DTYPE_BF16, _lib.DU_DTYPE_F16, 0, cos.shape[0], 0,
                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        _lib.check(rc, "du_rope")

    return graph_time(one, steps, stream) / steps


def cpu_prefill_baseline(cfg, reps=3):
    """fp32 torch reference path on the host cores (RoPE then SDPA per head block)."""
    import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    B, H, Hkv, S, D = cfg["B"], cfg["H"], cfg["Hkv"], cfg["S"], cfg["D"]
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    cos, sin = oracle.precompute_rope_cos_sin(S, D, torch.bfloat16, cfg["base"])

    def run():
        qr = oracle.apply_rope(q, cos, sin)
        kr = oracle.apply_rope(k, cos, sin).repeat_interleave(H // Hkv, dim=1)
        return torch.nn.functional.scaled_dot_product_attention(
            qr, kr, v.float().repeat_interleave(H // Hkv, dim=1), is_causal=True)

    run()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return prefill_flops(B, H, S, D) / t / 1e12, t, torch.get_num_threads()


def run_reference(args):
    """--impl reference: the reference's CPU path (fp32 torch RoPE + SDPA) on the host cores."""
    dist_rank = int(os.environ.get("RANK", "0"))
    if dist_rank != 0:
        return 0
    cfg = PREFILL
    tf, t, cores = cpu_prefill_baseline(cfg, reps=1)
    times = []
    for _ in range(args.warmup):
        cpu_prefill_baseline(cfg, reps=1)
    for _ in range(args.steps):
        _, ts, _ = cpu_prefill_baseline(cfg, reps=1)
        times.append(ts)
    ms = 1000.0 * statistics.mean(times)
    flops = prefill_flops(cfg["B"], cfg["H"], cfg["S"], cfg["D"])
    value = flops / (ms / 1000.0) / 1e12
    line = {
        "impl": "reference",
        "metric": "causal prefill TFLOP/s per B200 (decode KV-cache HBM GB/s in 'decode')",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": headline_workload(cfg),
                   "impl_path": "fp32 torch RoPE then scaled_dot_product_attention on CPU"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "cpu_model": cpu_model(),
                         "kind": "port",
                         "sample": "full workload per step (one prefill of the config)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_decode(rank, device, stream, steps, warmup, peaks):
    from dominusultra_b200 import dominus_ultra_decode, precompute_rope_cos_sin

    c = DECODE
    B, H, Hkv, L, D = c["B"], c["H"], c["Hkv"], c["L"], c["D"]
    per_set = 2 * B * Hkv * L * D * 2
    n_sets = max(2, math.ceil(2 * L2_BYTES / per_set))
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    sets = []
    for _ in range(n_sets):
        q = torch.randn(B, H, 1, D, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(B, Hkv, L, D, generator=g, device=device).to(torch.bfloat16)
        sets.append((q, k, v))
    cos, sin = precompute_rope_cos_sin(L + 1, D, device, torch.bfloat16, c["base"])

    def step(i):
        q, k, v = sets[i % n_sets]
        dominus_ultra_decode(q, k, v, cos, sin, Hkv)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device)
    ms_total = graph_time(step, steps, side)
    nbytes = decode_bytes(B, H, Hkv, L, D)
    gbs = nbytes / (ms_total / steps / 1000.0) / 1e9
    achieved = gbs  # the step is the split kernel plus the small merge (its share: profiles)
    from dominusultra_b200 import _lib

    splits_ws = int(_lib.load().du_decode_workspace_size(B, H, Hkv, L, D))
    return {
        "metric": "decode KV-cache HBM GB/s per B200",
        "value": gbs, "unit": "GB/s", "ms_per_step": ms_total / steps,
        "config": {"workload": f"decode B{B} H{H} Hkv{Hkv} L{L} D{D} bf16 RoPE base 1e4",
                   "l2": f"{n_sets} rotating input sets of {per_set / 1e6:.0f} MB (> L2)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": NCU_TRAFFIC["decode"],
                     "algorithmic_bytes": nbytes,
                     "launches_per_step": 2 if splits_ws > 0 else 1},
    }


def bench_decode_long(dist, rank, world, device, stream, steps, warmup, peaks):
    """Sequence-split decode: rank r holds keys [r L/N, (r+1) L/N) at their absolute positions;
    per step: partial kernel(s) on the shard, one packed all-gather over NCCL, LSE merge."""
    from dominusultra_b200 import dist as ddist
    from dominusultra_b200 import decode_partial, merge_partials, precompute_rope_cos_sin

    c = DECODE_LONG
    B, H, Hkv, L, D = c["B"], c["H"], c["Hkv"], c["L"], c["D"]
    a, b = ddist.kv_shard(L, world, rank)
    Ls = b - a
    g = torch.Generator(device=device).manual_seed(4000 + rank)
    q = torch.randn(B, H, 1, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(B, Hkv, Ls, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(B, Hkv, Ls, D, generator=g, device=device).to(torch.bfloat16)
    cos, sin = precompute_rope_cos_sin(L + 1, D, device, torch.bfloat16, c["base"])
    rows = B * H
    send = torch.empty(rows * (D + 1), dtype=torch.float32, device=device)
    gathered = torch.empty(world * send.numel(), dtype=torch.float32, device=device)
    o_view = send[: rows * D].view(B, H, D)
    l_view = send[rows * D:].view(B, H)

    def step_nccl(_i):
        decode_partial(q, k, v, cos, sin, Hkv, q_pos=L, kv_pos_offset=a, out=o_view, lse=l_view)
        if dist is not None:
            dist.all_gather_into_tensor(gathered, send)
            o_all, l_all = ddist.unpack_gathered(gathered, world, (B, H), D)
        else:
            o_all, l_all = o_view.unsqueeze(0), l_view.unsqueeze(0)
        merge_partials(o_all, l_all, torch.bfloat16)

    # With several ranks the partials are exchanged and merged over NVLink peer memory in one
    # kernel (PeerExchange); the NCCL all-gather + merge form is timed beside it. Every rank
    # takes the same path: if any rank cannot map the others' buffers, all use NCCL.
    ex = None
    if dist is not None and world > 1:
        try:
            ex = ddist.PeerExchange(rows, D, device=device)
            ok = 1
        except (RuntimeError, ValueError):  # no CUDA IPC here, or more ranks than it supports
            ok = 0
        flag = torch.tensor([ok], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0:
            if ex is not None:
                ex.close()  # collective: two barriers, matched below on the ranks that failed
            else:
                dist.barrier()
                dist.barrier()
            ex = None

    def step_peer(_i):
        decode_partial(q, k, v, cos, sin, Hkv, q_pos=L, kv_pos_offset=a, out=o_view, lse=l_view)
        ex.merge(o_view, l_view, torch.bfloat16)

    step = step_peer if ex is not None else step_nccl
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    if ex is not None:
        # A bounded wait that expired during the warm-up (status code 5 on any rank) means the
        # peer exchange does not work here: every rank falls back to NCCL before timing.
        from dominusultra_b200 import _lib as _dlib

        bad = torch.tensor([1 if _dlib.read_status(reset=True)[0] != 0 else 0], device=device)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        if int(bad.item()):
            ex.close()
            ex = None
            step = step_nccl
            for i in range(warmup):
                step(i)
            torch.cuda.synchronize()
    barrier(dist)
    # Eagerly launched, the host path of a step (Python wrappers and the collective, ~75 us with
    # NCCL) exceeds the device time of a rank's shard at eight GPUs; a generation loop replays the
    # step as a CUDA graph, and so does the timed region here (the eager figure is reported too).
    eager_ms = max_over_ranks(dist, time_region(step, steps, stream) / steps, device)
    barrier(dist)
    side = torch.cuda.Stream(device)
    ms = max_over_ranks(dist, graph_time(step, steps, side) / steps, device)
    nccl_ms = None
    if ex is not None:
        for i in range(warmup):
            step_nccl(i)
        torch.cuda.synchronize()
        barrier(dist)
        nccl_ms = max_over_ranks(dist, graph_time(step_nccl, steps, side) / steps, device)
        barrier(dist)
        ex.close()
    exchange = ("partials exchanged and merged over NVLink peer memory in one kernel "
                "(du_exchange_merge)") if ex is not None else "one NCCL all-gather + merge per step"
    total_bytes = decode_bytes(B, H, Hkv, L, D)
    return {
        "metric": "long-context decode KV-cache GB/s (whole job)",
        "value": total_bytes / (ms / 1000.0) / 1e9, "unit": "GB/s", "ms_per_step": ms,
        "timing": "CUDA graph of the steps (partial kernel, exchange, merge), replayed between "
                  "events; max over ranks",
        "eager_ms_per_step": eager_ms,
        "nccl_allgather_ms_per_step": nccl_ms,
        "scaling": "strong",
        "config": {"workload": f"decode B{B} H{H} Hkv{Hkv} L{L} D{D} bf16 RoPE base 5e5, "
                               f"KV sequence split over {world} GPU(s), {exchange}",
                   "kv_bytes_per_gpu": total_bytes / world},
        "per_gpu_hbm_frac": (total_bytes / world) / (ms / 1000.0) / 1e9 / peaks["hbm_gbs"],
    }


# The Llama-3-8B-shaped layer's prefill: 32 (batch, kv-head) units, split over the ranks.
PREFILL_P5 = dict(B=4, H=32, Hkv=8, S=32768, D=128, base=500000.0)
# What one rank streams in the long-context decode at eight GPUs: a 16384-key shard.
DECODE_P5_SHARD = dict(B=4, H=32, Hkv=8, L=16384, D=128, base=500000.0, total=131072)


def bench_prefill_p5(dist, rank, world, device, stream, steps, warmup, peaks, peak_kind):
    """The fixed Llama-3-8B-shaped prefill job (B4 H32 Hkv8 S32768 D128, 35.2 TFLOP) split over
    the ranks by ``dist.sharded_prefill``: each rank computes its contiguous range of (batch,
    kv-head) units with no communication. Strong scaling: the job is the same at every N. Every
    rank builds the same full inputs (one seed) and takes its slab; time = max over ranks."""
    from dominusultra_b200 import dist as ddist
    from dominusultra_b200 import precompute_rope_cos_sin

    c = PREFILL_P5
    B, H, Hkv, S, D = c["B"], c["H"], c["Hkv"], c["S"], c["D"]
    g = torch.Generator(device=device).manual_seed(5500)
    q = torch.randn(B, H, S, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g, device=device).to(torch.bfloat16)
    cos, sin = precompute_rope_cos_sin(S, D, device, torch.bfloat16, c["base"])
    plan = ddist.plan_prefill(B, H, Hkv, world)
    u0, u1 = ddist.shard_range(plan.n_units, world, rank)
    busiest = -(-plan.n_units // world)  # units of the most loaded rank

    def step(_i):
        ddist.sharded_prefill(q, k, v, cos, sin, Hkv, rank, world)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(dist)
    ms = time_region(step, steps, stream) / steps
    ms = max_over_ranks(dist, ms, device)
    flops = prefill_flops(B, H, S, D)
    per_gpu = flops * busiest / plan.n_units
    achieved = per_gpu / (ms / 1000.0) / 1e12
    peak = peaks["bf16_tflops_sustained"]
    return {
        "metric": "causal prefill TFLOP/s (whole job)",
        "value": flops / (ms / 1000.0) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
        "ms_per_step": ms, "steps": steps, "scaling": "strong",
        "config": {"workload": f"prefill B{B} H{H} Hkv{Hkv} S{S} D{D} causal RoPE base 5e5, "
                               f"{plan.n_units} (batch, kv-head) units sharded over {world} GPU(s) "
                               "by dist.sharded_prefill, no communication",
                   "units_this_rank": [u0, u1], "units_busiest_rank": busiest,
                   "l2": "inputs 1.6 GB (> L2)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None,
                     "peak_kind": f"{peak_kind} bf16 dense (sustained)",
                     "kernel": "prefill_fa_kernel<128> (step: key rotation + attention)",
                     "algorithmic_flops_per_gpu": per_gpu},
    }


def bench_decode_p5_shard(dist, rank, world, device, steps, warmup, peaks, peak_kind):
    """One rank's share of the long-context decode at eight GPUs: decode_partial over a
    16384-key shard (the last one: keys at positions 114688..131071, query at 131072) of
    B4 H32 Hkv8 D128, graph-timed over two rotating input sets (268 MB each, > L2). Every rank
    runs the same shard (weak scaling); time = max over ranks."""
    from dominusultra_b200 import decode_partial, precompute_rope_cos_sin

    c = DECODE_P5_SHARD
    B, H, Hkv, L, D, total = c["B"], c["H"], c["Hkv"], c["L"], c["D"], c["total"]
    off = total - L
    g = torch.Generator(device=device).manual_seed(6000 + rank)
    sets = [tuple(torch.randn(*shape, generator=g, device=device).to(torch.bfloat16)
                  for shape in ((B, H, 1, D), (B, Hkv, L, D), (B, Hkv, L, D))) for _ in range(2)]
    cos, sin = precompute_rope_cos_sin(total + 1, D, device, torch.bfloat16, c["base"])
    o = torch.empty(B, H, D, dtype=torch.float32, device=device)
    lse = torch.empty(B, H, dtype=torch.float32, device=device)

    def step(i):
        qq, kk, vv = sets[i % 2]
        decode_partial(qq, kk, vv, cos, sin, Hkv, q_pos=total, kv_pos_offset=off, out=o, lse=lse)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(dist)
    side = torch.cuda.Stream(device)
    ms = max_over_ranks(dist, graph_time(step, steps, side) / steps, device)
    nbytes = decode_bytes(B, H, Hkv, L, D)
    gbs = nbytes / (ms / 1000.0) / 1e9
    from dominusultra_b200 import _lib

    split = int(_lib.load().du_decode_workspace_size(B, H, Hkv, L, D)) > 0
    return {
        "metric": "decode KV-cache HBM GB/s per B200 (one rank's shard)",
        "value": gbs, "unit": "GB/s", "ms_per_step": ms, "n_gpus": world, "scaling": "weak",
        "config": {"workload": f"decode_partial B{B} H{H} Hkv{Hkv} L{L} D{D} bf16 RoPE base 5e5, "
                               f"keys at positions {off}..{total - 1}, query at {total}",
                   "l2": "2 rotating input sets of 268 MB (> L2)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": None,
                     "peak_kind": f"{peak_kind} copy bandwidth",
                     "kernel": "decode_tc_kernel<128, bf16, 4>" + (" + merge_kernel" if split else ""),
                     "algorithmic_bytes": nbytes},
    }


def profile_case(args):
    """--profile-case: a few launches of one kernel on one configuration, for ncu captures
    (one warm-up launch, then --steps launches). Inputs are seeded N(0,1) bf16 on the device;
    keep them above the 126 MB L2 so that DRAM counters mean something."""
    from dominusultra_b200 import dominus_ultra_decode, dominus_ultra_prefill, precompute_rope_cos_sin

    kind, sizes = args.profile_case[0], dict(kv.split("=") for kv in args.profile_case[1:])
    B, H, Hkv, D = (int(sizes.get(n, d)) for n, d in (("B", 8), ("H", 32), ("Hkv", 32), ("D", 64)))
    base = float(sizes.get("base", 10000.0))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    dt = torch.bfloat16
    if kind == "prefill":
        S = int(sizes.get("S", 2048))
        q = torch.randn(B, H, S, D, generator=g, device=dev).to(dt)
        k = torch.randn(B, Hkv, S, D, generator=g, device=dev).to(dt)
        v = torch.randn(B, Hkv, S, D, generator=g, device=dev).to(dt)
        cos, sin = precompute_rope_cos_sin(S, D, dev, dt, base)
        for _ in range(1 + args.steps):
            dominus_ultra_prefill(q, k, v, cos, sin, Hkv)
    elif kind == "decode":
        L = int(sizes.get("L", 2048))
        q = torch.randn(B, H, 1, D, generator=g, device=dev).to(dt)
        k = torch.randn(B, Hkv, L, D, generator=g, device=dev).to(dt)
        v = torch.randn(B, Hkv, L, D, generator=g, device=dev).to(dt)
        cos, sin = precompute_rope_cos_sin(L + 1, D, dev, dt, base)
        for _ in range(1 + args.steps):
            dominus_ultra_decode(q, k, v, cos, sin, Hkv)
    else:
        raise SystemExit("--profile-case takes prefill or decode, then NAME=VALUE sizes")
    torch.cuda.synchronize()
    return 0


def reference_gpu_baseline(device, steps, warmup):
    """The reference's own Triton kernels (installed unmodified in baseline/_ref) on this GPU,
    on the headline prefill and decode configurations; compile and autotune excluded by
    warm-up. Reported beside the CPU baseline; 'unavailable' with the reason if they cannot
    run here."""
    import importlib.util

    path = ROOT / "baseline" / "_ref" / "dominus_ultra.py"
    if not path.exists():
        return {"unavailable": "reference not installed in baseline/_ref"}
    try:
        spec = importlib.util.spec_from_file_location("dominus_ultra_reference", path)
        ref = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ref)
        from dominusultra_b200 import precompute_rope_cos_sin

        res = {"impl": "reference Triton kernels from baseline/_ref (unmodified)"}
        c = PREFILL
        B, H, Hkv, S, D = c["B"], c["H"], c["Hkv"], c["S"], c["D"]
        g = torch.Generator(device=device).manual_seed(99)
        q = torch.randn(B, H, S, D, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(B, Hkv, S, D, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(B, Hkv, S, D, generator=g, device=device).to(torch.bfloat16)
        cos, sin = precompute_rope_cos_sin(S, D, device, torch.bfloat16, c["base"])
        stream = torch.cuda.current_stream(device)
        fn = lambda i: ref.dominus_ultra_prefill(q, k, v, cos, sin, Hkv)  # noqa: E731
        for i in range(max(warmup, 3)):
            fn(i)
        torch.cuda.synchronize()
        ms = time_region(fn, steps, stream) / steps
        res["prefill"] = {"value": prefill_flops(B, H, S, D) / (ms / 1000.0) / 1e12,
                          "unit": "TFLOP/s", "ms_per_step": ms}
        c = DECODE
        B, H, Hkv, L, D = c["B"], c["H"], c["Hkv"], c["L"], c["D"]
        q = torch.randn(B, H, 1, D, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(B, Hkv, L, D, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(B, Hkv, L, D, generator=g, device=device).to(torch.bfloat16)
        cos, sin = precompute_rope_cos_sin(L + 1, D, device, torch.bfloat16, c["base"])
        fn = lambda i: ref.dominus_ultra_decode(q, k, v, cos, sin, Hkv)  # noqa: E731
        for i in range(max(warmup, 3)):
            fn(i)
        torch.cuda.synchronize()
        ms = time_region(fn, steps, stream) / steps
        res["decode"] = {"value": decode_bytes(B, H, Hkv, L, D) / (ms / 1000.0) / 1e9,
                         "unit": "GB/s", "ms_per_step": ms,
                         "note": "no L2 flush between steps (KV is 134 MB, just above L2)"}
        return res
    except Exception as e:  # the reference's kernels failing here is reported, not fatal
        return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}


RING = dict(B=4, H=32, Hkv=8, S=32768, D=128, base=500000.0)


def bench_ring(dist, rank, world, device, stream, steps, warmup, peaks, peak_kind, seq):
    """Context-parallel prefill of the Llama-3-8B-shaped layer: the sequence zigzag-sharded over
    the ranks (chunks r and 2N-1-r), K/V passed around the ring with NCCL point-to-point,
    overlapped with the block kernels. Strong scaling: the whole sequence is fixed."""
    from dominusultra_b200 import precompute_rope_cos_sin, ring

    c = dict(RING, S=seq or RING["S"])
    B, H, Hkv, S, D = c["B"], c["H"], c["Hkv"], c["S"], c["D"]
    tc = S // (2 * world)
    g = torch.Generator(device=device).manual_seed(5000 + rank)
    q = torch.randn(B, H, 2 * tc, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(B, Hkv, 2 * tc, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(B, Hkv, 2 * tc, D, generator=g, device=device).to(torch.bfloat16)
    cos, sin = precompute_rope_cos_sin(S, D, device, torch.bfloat16, c["base"])

    def step(_i):
        ring.ring_prefill(q, k, v, cos, sin, Hkv)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(dist)
    ms = time_region(step, steps, stream) / steps
    ms = max_over_ranks(dist, ms, device)
    flops = prefill_flops(B, H, S, D)
    tflops = flops / (ms / 1000.0) / 1e12
    return {
        "metric": "context-parallel causal prefill TFLOP/s (whole job)", "value": tflops,
        "unit": "TFLOP/s", "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
        "data": "synthetic N(0,1) bf16, seeded per rank",
        "config": {"workload": f"prefill B{B} H{H} Hkv{Hkv} S{S} D{D} causal RoPE base 5e5, "
                               f"sequence zigzag-sharded over {world} GPU(s), ring of NCCL "
                               "point-to-point K/V transfers"},
        "per_gpu_frac_of_peak": tflops / world / peaks["bf16_tflops_sustained"],
        "peak_kind": f"{peak_kind} bf16 dense (sustained)",
    }


# The reference's benchmark configurations (benchmark.py sweeps): P1 its CPU-runnable case, P2
# the MHA prefill sweep, P3 grouped- and multi-query prefill, P4 the decode sweep.
SWEEP_PREFILL = ([("P1", dict(B=1, H=8, Hkv=8, S=512, D=64))]
                 + [("P2", dict(B=2, H=32, Hkv=32, S=s, D=64)) for s in (128, 256, 512, 1024, 2048)]
                 + [("P3", dict(B=2, H=32, Hkv=h, S=1024, D=64)) for h in (8, 1)])
SWEEP_DECODE = [("P4", dict(B=8, H=32, Hkv=32, L=n, D=64)) for n in (128, 256, 512, 1024, 2048)]


def bench_sweep(dist, rank, world, device, steps, warmup, peaks, peak_kind):
    """One line per configuration: graph-timed device time of `steps` calls through the public
    API, each call on a different input set (sets together > 2x L2), max over ranks."""
    from dominusultra_b200 import dominus_ultra_decode, precompute_rope_cos_sin
    from dominusultra_b200 import dominus_ultra_prefill

    side = torch.cuda.Stream(device)
    lines = []
    for tag, c in SWEEP_PREFILL + SWEEP_DECODE:
        c = dict(c, base=10000.0)
        B, H, Hkv, D = c["B"], c["H"], c["Hkv"], c["D"]
        prefill = "S" in c
        n = c["S"] if prefill else c["L"]
        per_set = (B * H * n * D + 2 * B * Hkv * n * D) * 2 if prefill else 2 * B * Hkv * n * D * 2
        n_sets = max(2, math.ceil(2 * L2_BYTES / per_set))
        g = torch.Generator(device=device).manual_seed(77 + rank)
        qn = n if prefill else 1
        sets = [tuple(torch.randn(*shape, generator=g, device=device).to(torch.bfloat16)
                      for shape in ((B, H, qn, D), (B, Hkv, n, D), (B, Hkv, n, D)))
                for _ in range(n_sets)]
        cos, sin = precompute_rope_cos_sin(n if prefill else n + 1, D, device, torch.bfloat16, c["base"])
        fn = dominus_ultra_prefill if prefill else dominus_ultra_decode

        def step(i, sets=sets, cos=cos, sin=sin, fn=fn, Hkv=Hkv):
            q, k, v = sets[i % len(sets)]
            fn(q, k, v, cos, sin, Hkv)

        for i in range(warmup):
            step(i)
        torch.cuda.synchronize()
        barrier(dist)
        ms = max_over_ranks(dist, graph_time(step, steps, side), device) / steps
        if prefill:
            work, unit, peak = prefill_flops(B, H, n, D) * world / 1e12, "TFLOP/s", peaks["bf16_tflops"]
            metric, shape = "causal prefill TFLOP/s", f"prefill B{B} H{H} Hkv{Hkv} S{n} D{D}"
        else:
            work, unit, peak = decode_bytes(B, H, Hkv, n, D) * world / 1e9, "GB/s", peaks["hbm_gbs"]
            metric, shape = "decode KV-cache HBM GB/s", f"decode B{B} H{H} Hkv{Hkv} L{n} D{D}"
        value = work / (ms / 1000.0)
        lines.append({"metric": metric, "value": value, "unit": unit, "n_gpus": world,
                      "us_per_call": ms * 1000.0, "frac_of_peak": value / world / peak,
                      "peak": f"{peak} {unit} per GPU ({peak_kind})", "scaling": "weak",
                      "config": {"workload": f"{tag} {shape} bf16 RoPE base 1e4",
                                 "l2": f"{n_sets} rotating input sets of {per_set / 1e6:.1f} MB"}})
        del sets
    return lines


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-long-decode", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true")
    ap.add_argument("--ring", action="store_true",
                    help="only the context-parallel (ring) prefill of the Llama-3-8B-shaped layer")
    ap.add_argument("--ring-seq", type=int, default=0, help="sequence length of --ring")
    ap.add_argument("--sweep", action="store_true",
                    help="only the reference's benchmark configurations, one line each")
    ap.add_argument("--no-p5", action="store_true",
                    help="skip the Llama-3-8B-shaped prefill split and decode shard objects")
    ap.add_argument("--profile-case", nargs="+", metavar="ARG",
                    help="prefill|decode [B=.. H=.. Hkv=.. S=.. L=.. D=.. base=..]: run --steps "
                         "launches of that call only (for ncu captures)")
    args = ap.parse_args()
    if args.profile_case:
        return profile_case(args)
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        return run_reference(args)

    from dominusultra_b200 import _lib, dominus_ultra_prefill

    dist, rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    peaks, peak_kind = load_peaks()
    _lib.load()
    if args.ring:
        line = bench_ring(dist, rank, world, device, stream, args.steps, args.warmup, peaks,
                          peak_kind, args.ring_seq)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0
    if args.sweep:
        for line in bench_sweep(dist, rank, world, device, args.steps, args.warmup, peaks, peak_kind):
            if rank == 0:
                print(json.dumps(line), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0

    cfg = PREFILL
    B, H, Hkv, S, D = cfg["B"], cfg["H"], cfg["Hkv"], cfg["S"], cfg["D"]
    per_set = (B * H * S * D + 2 * B * Hkv * S * D) * 2
    n_sets = max(2, math.ceil(2 * L2_BYTES / per_set))
    sets, cos, sin = make_prefill_sets(cfg, n_sets, 1234 + rank, device)

    def step(i):
        q, k, v = sets[i % n_sets]
        dominus_ultra_prefill(q, k, v, cos, sin, Hkv)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    side = torch.cuda.Stream(device)  # graphs are captured on a side stream
    sampler = ClockSampler(device.index)
    barrier(dist)
    torch.cuda.synchronize()
    sampler.start()
    ms_total = graph_time(step, args.steps, side)
    torch.cuda.synchronize()
    barrier(dist)
    clocks = sampler.stop()
    ms_total = max_over_ranks(dist, ms_total, device)
    ms_step = ms_total / args.steps
    flops = prefill_flops(B, H, S, D)
    value = world * flops / (ms_step / 1000.0) / 1e12

    # The dominant kernel: a step is the key-rotation launch plus the attention launch, and the
    # attention launch starts (as a programmatic dependent) while the rotation runs, so events
    # cannot separate them. The step time bounds the attention launch's duration from above:
    # achieved = algorithmic FLOPs / step time is a lower bound on the kernel's rate. The
    # rotation pass is timed on its own for reference.
    rope_ms = rope_pass_ms(sets, cos, sin, cfg, args.steps, side)
    attn_ms = ms_step
    achieved = flops / (attn_ms / 1000.0) / 1e12

    # End to end through the public API with pinned host buffers.
    host_sets = [tuple(t.cpu().pin_memory() for t in s) for s in sets[:2]]
    q0, k0, v0 = sets[0]
    out_h = torch.empty(q0.shape, dtype=q0.dtype).pin_memory()
    lse_h = torch.empty((B, H, S), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        qh, kh, vh = host_sets[i % 2]
        q = qh.to(device, non_blocking=True)
        k = kh.to(device, non_blocking=True)
        v = vh.to(device, non_blocking=True)
        out, lse = dominus_ultra_prefill(q, k, v, cos, sin, Hkv)
        out_h.copy_(out, non_blocking=True)
        lse_h.copy_(lse, non_blocking=True)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(dist)
    e2e_serial_ms = time_region(e2e_step, args.steps, stream) / args.steps
    e2e_serial_ms = max_over_ranks(dist, e2e_serial_ms, device)

    # The same steps with the copies on their own streams, double-buffered: step i+1's inputs
    # cross PCIe while step i computes and step i-1's outputs come back (host-to-device and
    # device-to-host copies run on separate copy engines). Every step still copies its own
    # inputs in and its own outputs out inside the timed region.
    h2d_st, d2h_st = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dev_in = [tuple(torch.empty(t.shape, dtype=t.dtype, device=device) for t in host_sets[0])
              for _ in range(2)]
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_pipelined(n):
        first = torch.cuda.Event(enable_timing=True)
        last = torch.cuda.Event(enable_timing=True)
        first.record(stream)
        h2d_st.wait_event(first)
        d2h_st.wait_event(first)
        for i in range(n):
            slot = i % 2
            with torch.cuda.stream(h2d_st):
                if i >= 2:
                    h2d_st.wait_event(comp_done[slot])  # step i-2 has finished reading the slot
                for dst, src in zip(dev_in[slot], host_sets[i % 2]):
                    dst.copy_(src, non_blocking=True)
                h2d_done[slot].record(h2d_st)
            stream.wait_event(h2d_done[slot])
            q, k, v = dev_in[slot]
            out, lse = dominus_ultra_prefill(q, k, v, cos, sin, Hkv)
            comp_done[slot].record(stream)
            with torch.cuda.stream(d2h_st):
                d2h_st.wait_event(comp_done[slot])
                out_h.copy_(out, non_blocking=True)
                lse_h.copy_(lse, non_blocking=True)
            out.record_stream(d2h_st)
            lse.record_stream(d2h_st)
        last.record(d2h_st)
        last.synchronize()
        return first.elapsed_time(last)

    e2e_pipelined(2)
    torch.cuda.synchronize()
    barrier(dist)
    e2e_ms = e2e_pipelined(args.steps) / args.steps
    e2e_ms = max_over_ranks(dist, e2e_ms, device)
    h2d = sum(t.numel() * t.element_size() for t in host_sets[0])
    d2h = out_h.numel() * out_h.element_size() + lse_h.numel() * 4

    decode = None
    if not args.no_decode:
        decode = bench_decode(rank, device, stream, args.steps, args.warmup, peaks)
        if dist is not None:
            dms = max_over_ranks(dist, decode["ms_per_step"], device)
            decode["ms_per_step"] = dms
            decode["value"] = world * decode_bytes(DECODE["B"], DECODE["H"], DECODE["Hkv"],
                                                   DECODE["L"], DECODE["D"]) / (dms / 1000.0) / 1e9

    decode_long = None
    if not args.no_long_decode:
        decode_long = bench_decode_long(dist, rank, world, device, stream, args.steps, args.warmup, peaks)

    prefill_p5 = decode_p5_shard = None
    if not args.no_p5:
        # The decode shard first: the long dense prefill that follows runs at the power cap.
        decode_p5_shard = bench_decode_p5_shard(dist, rank, world, device, args.steps,
                                                args.warmup, peaks, peak_kind)
        prefill_p5 = bench_prefill_p5(dist, rank, world, device, stream, args.steps, args.warmup,
                                      peaks, peak_kind)

    status = _lib.read_status(reset=True)
    line = None
    if rank == 0:
        peak = peaks["bf16_tflops"]
        line = {
            "metric": "causal prefill TFLOP/s per B200 (decode KV-cache HBM GB/s in 'decode')",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic N(0,1) bf16, seeded per rank; RoPE tables from precompute_rope_cos_sin",
            "config": {
                "workload": headline_workload(cfg),
                "parallelism": f"(batch, kv-head) units sharded over {world} GPU(s), no communication",
                "l2": f"{n_sets} rotating input sets of {per_set / 1e6:.0f} MB (> L2)",
            },
            "roofline": {
                "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": NCU_TRAFFIC["prefill"],
                "peak_kind": f"{peak_kind} bf16 dense (burst)",
                "kernel": "prefill_fa1_kernel", "kernel_ms": attn_ms,
                "kernel_ms_is": "the step time (rotation overlapped with the attention launch): "
                                "an upper bound on the attention launch",
                "algorithmic_flops": flops,
                "rope_pass": {"kernel": "rope_kernel (keys, bf16 -> fp16)", "ms": rope_ms,
                              "gbs": rope_bytes(cfg) / (rope_ms / 1000.0) / 1e9},
            },
            "e2e": {"value": world * flops / (e2e_ms / 1000.0) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "copies": "pinned host buffers; H2D and D2H on their own streams, double-buffered "
                              "across steps",
                    "serial_ms_per_step": e2e_serial_ms},
            "gpu_launches": 2 * args.steps,  # per step: key rotation + attention
            "clocks": clocks,
            "device_status": status,
        }
        if decode is not None:
            line["decode"] = decode
        if decode_long is not None:
            line["decode_long"] = decode_long
        if prefill_p5 is not None:
            line["prefill_p5"] = prefill_p5
        if decode_p5_shard is not None:
            line["decode_p5_shard"] = decode_p5_shard
        if not args.no_reference_gpu:
            line["reference_gpu"] = reference_gpu_baseline(device, min(args.steps, 20), args.warmup)
        if not args.no_cpu_baseline:
            tf, t, cores = cpu_prefill_baseline(cfg)
            line["cpu_baseline"] = {
                "value": tf, "unit": "TFLOP/s", "cores": cores, "cpu_model": cpu_model(), "kind": "port",
                "sample": f"full workload (one prefill of the config), median of 3, {t * 1000:.0f} ms each",
            }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
