"""TriBench's latency measurement without Triton.

TriBench times a kernel pack's entry point with ``triton.testing.do_bench`` (its default timer
backend, tribench/bench.py:25-39, called from run_benchmark at :163 with warmup 200 ms and
rep 2000 ms, cli.py:47-48) and summarises the raw latencies (bench.py:165-198,
eval_metrics.py:16-25, metrics.py:6-17). ``do_bench`` below restates that published procedure
in plain PyTorch so the sm_100a path can be measured exactly as ``tribench run`` would measure
it, with no Triton on the box:

  * one call to settle, then five calls with an L2 flush (zeroing a 256 MB buffer) each, timed
    together with CUDA events, give the per-call estimate;
  * warm-up calls = max(1, warmup_ms / estimate), timed calls = max(1, rep_ms / estimate);
  * every timed call is preceded by the L2 flush and bracketed by its own pair of events.

``summarize`` computes TriBench's BenchResult latency fields and throughputs from them.
"""
from __future__ import annotations

import math

import torch

L2_FLUSH_BYTES = 256 * 1024 * 1024


def do_bench(fn, warmup_ms: float = 200.0, rep_ms: float = 2000.0, device=None) -> list[float]:
    """All per-call latencies (ms) of ``fn`` on the current CUDA stream."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    fn()
    torch.cuda.synchronize(dev)
    cache = torch.empty(L2_FLUSH_BYTES, dtype=torch.int8, device=dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(5):
        cache.zero_()
        fn()
    end.record()
    torch.cuda.synchronize(dev)
    estimate_ms = max(start.elapsed_time(end) / 5, 1e-6)
    n_warmup = max(1, int(warmup_ms / estimate_ms))
    n_repeat = max(1, int(rep_ms / estimate_ms))
    for _ in range(n_warmup):
        fn()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_repeat)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_repeat)]
    for i in range(n_repeat):
        cache.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize(dev)
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def _percentile(sorted_vals: list[float], q: float) -> float:
    """Linear-interpolation percentile (numpy's default method)."""
    if not sorted_vals:
        raise ValueError("no latencies")
    pos = (len(sorted_vals) - 1) * q / 100.0
    lo = math.floor(pos)
    hi = min(lo + 1, len(sorted_vals) - 1)
    return sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (pos - lo)


def summarize(latencies_ms: list[float], flops: float | None = None, nbytes: float | None = None) -> dict:
    """TriBench's latency statistics (BenchResult fields) of one measurement."""
    s = sorted(float(x) for x in latencies_ms)
    n = len(s)
    mean = sum(s) / n
    std = math.sqrt(sum((x - mean) ** 2 for x in s) / n)  # population std, as numpy.std
    p50 = _percentile(s, 50)
    p99 = _percentile(s, 99)
    out = {
        "latency_ms_p50": p50, "latency_ms_p90": _percentile(s, 90), "latency_ms_p95": _percentile(s, 95),
        "latency_ms_p99": p99, "latency_ms_min": s[0], "latency_ms_max": s[-1], "latency_ms_mean": mean,
        "latency_ms_std": std, "tail_ratio_p99_p50": p99 / p50 if p50 > 0 else None,
        "jitter_cv": std / mean if mean > 0 else None, "reps": n,
    }
    if flops:
        out["tflops"] = flops / (p50 * 1e-3) / 1e12 if p50 > 0 else 0.0
    if nbytes:
        out["gbps"] = nbytes / (p50 * 1e-3) / 1e9 if p50 > 0 else 0.0
    return out
