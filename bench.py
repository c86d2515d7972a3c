#!/usr/bin/env python
"""Benchmark of the sage_attn path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload h8k|c2|c3|c4|c5] [--impl ours|reference]

A step is one pass of the path over one batch: the pre-pass (K smoothing + INT8 Q/K
quantisation, + FP8 V for c4) followed by the fused attention kernel, on inputs already
resident in HBM. The default workload is "h8k" — B=2, H=32, S=8192, D=128, fp16, non-causal,
smoothed K, fp16 P.V — the S=8K D=128 configuration the headline metric is quoted on.

Multi-GPU (torchrun, one process per GPU): the (batch x head) grid is partitioned across the
ranks and a step ends when the whole output is assembled on rank 0 — the north star's only
collective, the final output gather. Rank 0's output buffer is mapped into every rank (CUDA
IPC, NVLink peer access). By default (--gather copy) each rank computes its heads in 8 waves
that alternate over two compute streams (consecutive waves overlap, so no SM idles at a wave's
end) and copies every finished wave into the mapping with the copy engine while the next waves
compute; --gather peer lets the attention epilogues store straight into the mapping (SM stores
into another GPU's memory reach only ~170 GB/s at the destination); --gather nccl sends each
finished wave to rank 0 point to point while computing the next. The default
workloads scale weakly (the global batch at N ranks is N times the 1-GPU batch, so N=1 is the
1-GPU line exactly, with no gather); the sharded long-context workload "c5" (B=16, H=64, S=32K,
causal) scales strongly (its fixed 1024-head grid is split). value = total ops of all ranks /
max-over-ranks device time, gather included.

Rooflines divide by the tcgen05 rates measured on this hardware (profiles/tensor_peaks.json,
made by `python -m tribench_b200.peaks`): ops per SM clock x SMs x the SM clock the timed
region ran at (the max clock when the run held it).

At N=1 the line also carries the reference's own Triton kernel (run_sage_attn /
run_flash_attn from the installed TriBench in baseline/_ref) timed with CUDA events on the
same device-resident inputs, and the default step with one Q scale per token (blkq=1).

--workload fa_s4k_d64 | fa_s8k_d64 benchmarks the flash_attn pack (fp16 QK^T and P.V, no
quantisation; its meta.json cases) through sage_flash_attn_fwd, one launch per step.

--impl reference times the reference's own algorithm on the host CPU (the reference.py `ref`
PyTorch path, restated per (batch, head) slice in oracle.ref_attention_torch), one sampled
head per step, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

from tribench_b200 import shard, timing  # noqa: E402

METRIC = "sage_attn TOPS (S=8K, D=128) vs INT8 tensor peak"
UNIT = "TOPS"
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="h8k",
                    choices=["h8k", "c2", "c3", "c4", "c5", "s4k_d64", "s8k_d64", "fa_s4k_d64", "fa_s8k_d64"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-chunks", type=int, default=16, help="head chunks of the host pipeline (e2e)")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", default="copy", choices=["copy", "peer", "nccl"],
                    help="N > 1: output gather into rank 0's IPC-mapped buffer by copy-engine copies of each "
                         "finished wave, waves on two overlapping compute streams (copy); by peer stores from "
                         "the attention epilogue (peer); or NCCL point to point per finished wave (nccl)")
    ap.add_argument("--waves", type=int, default=None,
                    help="head waves per rank (default 1; with --gather copy: 8; with --gather nccl: 8 for c5, "
                         "4 otherwise)")
    ap.add_argument("--no-triton-reference", action="store_true",
                    help="skip timing the reference's Triton kernel (baseline/_ref) at N=1")
    ap.add_argument("--no-blkq1", action="store_true", help="skip the per-token (blkq=1) side measurement")
    ap.add_argument("--no-tribench-timing", action="store_true",
                    help="skip the drop-in run() measured with TriBench's do_bench procedure")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def workload_case(name: str, world: int) -> dict:
    import tribench_b200 as tb

    case = dict(tb.CONFIGS[name]) if name in tb.CONFIGS else dict(tb.flash_attn.FLASH_CONFIGS[name], pv="16bit")
    case["name"] = name
    case["batch_size_per_rank"] = case["batch_size"]
    if name == "c5":
        # the sharded long-context config: the fixed (B x H) grid is split across ranks
        case["shard"] = "strong"
    else:
        case["batch_size"] = case["batch_size"] * world
        case["shard"] = "weak"
    return case


def read_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"bf16_burst": p.get("bf16_tflops"), "bf16_sustained": p.get("bf16_tflops_sustained"),
                "hbm": p.get("hbm_gbs"), "source": "measured"}
    return {"bf16_burst": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


def read_tensor_peaks() -> dict | None:
    """Per-SM-clock tcgen05 rates and the sustained (power-capped) rates measured by
    tribench_b200.peaks (profiles/tensor_peaks.json), or None."""
    path = os.path.join(ROOT, "profiles", "tensor_peaks.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f)


def tensor_rooflines(tp: dict | None, clock_mhz, ops_qk: float, ops_pv: float, pv: str) -> dict:
    """Peaks (TOPS) for the attention kernel: INT8 QK^T and 16-bit or e4m3 P.V at their measured
    per-clock rates, at the clock the timed region ran at (the max clock when the median sample
    is within 5 % of it); the mixed peak is the harmonic combination for these op counts. Also
    the sustained (power-capped, seconds-long) mixed rate from the same measurement."""
    pv_kind = "e4m3" if pv == "fp8" else "f16"
    if tp is None:  # fallback: the driver's cuBLAS bf16 figure, INT8 / FP8 at twice it
        pk = read_peaks()
        i8, pvr = 2 * pk["bf16_burst"], (2 if pv == "fp8" else 1) * pk["bf16_burst"]
        return {"int8": i8, "pv": pvr, "mixed": (ops_qk + ops_pv) / (ops_qk / i8 + ops_pv / pvr), "clock_mhz": None,
                "source": f"{pk['source']} cuBLAS bf16 burst x2 (no tcgen05 measurement)"}
    max_mhz = tp["max_sm_mhz"]
    use = max_mhz if (clock_mhz is None or clock_mhz >= 0.95 * max_mhz) else float(clock_mhz)
    rate = lambda k: tp["ops_per_clk_per_sm"][k]["128"] * tp["sms"] * use * 1e6 / 1e12
    i8, pvr = rate("i8"), rate(pv_kind)
    si8, spv = tp["sustained"]["i8"]["tops"], tp["sustained"][pv_kind]["tops"]
    return {"int8": round(i8, 1), "pv": round(pvr, 1), "mixed": round((ops_qk + ops_pv) / (ops_qk / i8 + ops_pv / pvr), 1),
            "mixed_sustained": round((ops_qk + ops_pv) / (ops_qk / si8 + ops_pv / spv), 1),
            "int8_sustained": si8, "clock_mhz": use,
            "source": f"measured tcgen05 rates (profiles/tensor_peaks.json): {tp['ops_per_clk_per_sm']['i8']['128']:.0f} "
                      f"int8 / {tp['ops_per_clk_per_sm'][pv_kind]['128']:.0f} {pv_kind} ops per SM clock x {tp['sms']} "
                      f"SMs x {use:.0f} MHz" + (" (max clock; the run held it)" if use == max_mhz else
                                               " (the run's median SM clock)")}


def load_triton_reference(pack: str):
    """The reference's own Triton entry point from the TriBench installed in baseline/_ref
    (run_sage_attn, kernels/sage_attn/triton_impl.py:162; run_flash_attn,
    kernels/flash_attn/triton_impl.py:110), or (None, reason)."""
    import importlib.util

    path = os.path.join(ROOT, "baseline", "_ref", "kernels", pack, "triton_impl.py")
    if not os.path.exists(path):
        return None, f"no installed reference at {os.path.relpath(path, ROOT)}"
    try:
        spec = importlib.util.spec_from_file_location(f"tribench_ref_{pack}_triton_impl", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return getattr(mod, "run_sage_attn" if pack == "sage_attn" else "run_flash_attn"), None
    except Exception as e:  # pragma: no cover - reported in the line
        return None, f"{type(e).__name__}: {str(e).splitlines()[0] if str(e) else ''}"


def time_triton_reference(pack: str, q, k, v, causal: bool, ops: float, our_ms: float, ours=None, reps: int = 20):
    """CUDA-event time of the reference's Triton kernel on the same device-resident inputs."""
    fn, why = load_triton_reference(pack)
    if fn is None:
        return {"unavailable": why}
    out = {"call": f"{pack} triton_impl.{'run_sage_attn' if pack == 'sage_attn' else 'run_flash_attn'}"
                   "(q, k, v) from baseline/_ref (stock reference code, Triton-compiled for this GPU)",
           "note": "the reference's Triton kernels ignore causal; timed non-causal only"}
    if causal:
        out["unavailable"] = "causal workload: the reference's Triton sage kernel ignores causal"
        return out
    try:
        for _ in range(3):
            o = fn(q, k, v)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for _ in range(reps):
            e0.record()
            fn(q, k, v)
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
    except Exception as e:
        out["unavailable"] = f"{type(e).__name__}: {str(e).splitlines()[0] if str(e) else ''}"
        return out
    p50 = statistics.median(times)
    out.update({"p50_ms": round(p50, 4), "min_ms": round(min(times), 4), "reps": reps,
                "value": round(ops / (p50 * 1e-3) / 1e12, 2),
                "speedup_ours_vs_triton": round(p50 / our_ms, 3)})
    if ours is not None:
        out["max_abs_diff_vs_ours"] = float((o.float() - ours.float()).abs().max().item())
    return out


def read_traffic() -> dict:
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every INTERVAL_MS; summary() describes the
    samples taken after mark() (call it when the warm-up steps start), so the median SM clock
    is that of the loaded GPU during warm-up + timed steps."""

    INTERVAL_MS = 20

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None
        self.t_mark = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.INTERVAL_MS)], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark(self):
        import datetime

        self.t_mark = datetime.datetime.now()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        import datetime

        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        with open(self.file.name) as f:
            rows = [r.strip().split(", ") for r in f if r.strip()]
        os.unlink(self.file.name)
        sm, smax, power, reasons, n_all = [], None, [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f")
                clk, cmax, pw = float(r[2]), float(r[3]), float(r[4])
            except ValueError:
                continue
            n_all += 1
            if self.t_mark is not None and ts < self.t_mark:
                continue
            sm.append(clk)
            smax = cmax
            power.append(pw)
            for n, v in zip(names, r[6:10]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "sm_mhz_min": min(sm) if sm else None, "reasons": sorted(reasons), "samples": len(sm),
                "samples_all": n_all, "interval_ms": self.INTERVAL_MS,
                "over": "warm-up + timed steps (samples after the first warm-up step was queued)",
                "power_w_median": statistics.median(power) if power else None,
                "power_w_max": max(power) if power else None}


def cpu_baseline(case: dict, seconds: float) -> dict:
    """The reference's PyTorch `ref` on the host CPU, one (b, h) head at a time (bounded sample)."""
    import oracle
    import tribench_b200 as tb

    S, D = case["seq_len"], case["head_dim"]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    one = dict(case, batch_size=1, num_heads=1)
    inp = tb.make_inputs(one, "cpu", seed=case["seed"], dtype="fp32")
    ops_head = tb.estimate(dict(one))["ops_alg"]
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.ref_attention_torch(inp["q"], inp["k"], inp["v"], causal=case["causal"])
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(ops_head * n / dt / 1e12, 6), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} head(s) of S={S} D={D} (causal={case['causal']}) through the reference's fp32 "
                      f"PyTorch ref, {dt:.1f} s, extrapolated per op"}


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    case = workload_case(args.workload, 1)
    import oracle
    import tribench_b200 as tb

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    one = dict(case, batch_size=1, num_heads=1)
    inp = tb.make_inputs(one, "cpu", seed=case["seed"], dtype="fp32")
    ops_head = tb.estimate(one)["ops_alg"]
    for _ in range(args.warmup):
        oracle.ref_attention_torch(inp["q"], inp["k"], inp["v"], causal=case["causal"])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.ref_attention_torch(inp["q"], inp["k"], inp["v"], causal=case["causal"])
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = ops_head * len(times) / total / 1e12
    flash = args.workload.startswith("fa_")
    metric = "flash_attn TFLOPS (fp16 QK^T and P.V) vs fp16 tensor peak" if flash else METRIC
    unit = "TFLOP/s" if flash else UNIT
    line = {
        "impl": "reference", "metric": metric, "value": round(value, 6), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / len(times), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(case, world),
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"one (b,h) head of the workload per step (S={case['seq_len']}, "
                                   f"D={case['head_dim']}), reference.py ref in fp32 PyTorch on the host"},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(case: dict, world: int) -> dict:
    nbytes = 2 * case["batch_size"] * case["num_heads"] * case["seq_len"] * case["head_dim"] // max(1, world)
    return {
        "workload": case["name"],
        "batch": case["batch_size"], "heads": case["num_heads"], "seq_len": case["seq_len"],
        "head_dim": case["head_dim"], "causal": case["causal"], "input_dtype": case["dtype"],
        "pv": case["pv"], "smooth_k": True, "sharding": f"(batch x head) grid, {case['shard']} scaling",
        "parallelism": f"shard{world}",
        "l2": f"inputs {3 * nbytes / 1e6:.0f} MB per rank > 126 MB L2 (no flush needed)"
              if 3 * nbytes > L2_BYTES else "L2 flushed between steps",
    }


def run_e2e(args, case, q, k, v, o, dev, stream, barrier, pg) -> float:
    """Device time of e2e steps through the public host-buffer API (HostPipeline.run: pinned host
    q/k/v in, host output back; chunks of heads go host -> device, through sage_run and back on
    overlapping streams), max over ranks."""
    import tribench_b200 as tb

    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
    _, nh, S, D = q.shape
    pipe = tb.HostPipeline(1, nh, nh, S, S, D, q.dtype, dev, chunks=args.e2e_chunks, pv=case["pv"], smooth_k=True,
                           causal=case["causal"])

    def e2e_step():
        pipe.run(hq, hk, hv, ho)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    return e2e_ms


def main_flash(args):
    """The flash_attn pack: one sage_flash_attn_fwd launch per step on resident inputs."""
    import tribench_b200 as tb

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        pg = dist
    case = dict(tb.flash_attn.FLASH_CONFIGS[args.workload], name=args.workload, pv="16bit", shard="weak")
    case["batch_size"] *= world
    sd = shard.make_shard(case, rank, world)
    inp = tb.make_inputs(case, dev, seed=case["seed"], dtype=case["dtype"], heads=(sd.lo, sd.hi))
    q, k, v = inp["q"], inp["k"], inp["v"]
    o = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    est_rank = tb.estimate(dict(case, batch_size=1, num_heads=sd.heads))
    est_total = tb.estimate(case)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        time.sleep(0.3)
        clk.mark()
        for _ in range(args.warmup):
            tb.run_flash_attn(q, k, v, causal=case["causal"], out=o)
        torch.cuda.synchronize(dev)
        assert tb.device_status(dev) == 0
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            tb.run_flash_attn(q, k, v, causal=case["causal"], out=o)
            evs[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    total_ms = t0.elapsed_time(t1)
    launch_ms = [a.elapsed_time(b) for a, b in evs]
    if pg is not None:
        t = torch.tensor([total_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms = float(t.item())
    # e2e through the public call with host buffers: inputs up, one launch, output down
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, args.e2e_steps)
    e0.record(stream)
    for _ in range(e2e_steps):
        for d, h_ in ((dq, hq), (dk, hk), (dv, hv)):
            d.copy_(h_, non_blocking=True)
        ho.copy_(tb.run_flash_attn(dq, dk, dv, causal=case["causal"], out=o), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    tri = None
    if world == 1 and not args.no_tribench_timing:
        B_, H_, S_, D_ = case["batch_size"], case["num_heads"], case["seq_len"], case["head_dim"]
        qv, kv_, vv = (t.view(B_, H_, S_, D_) for t in (q, k, v))
        lat = timing.do_bench(lambda: tb.run_flash_attn(qv, kv_, vv, causal=case["causal"]), device=dev)
        tri = timing.summarize(lat, flops=est_total["flops"])
        tri["call"] = "tribench_b200.run_flash_attn(q, k, v, causal) (the plugin's run; output allocated per call)"
        tri["timer"] = "do_bench restated without Triton: 256 MB L2 flush per rep, warmup 200 ms, rep 2000 ms"
    triton_ref = None
    if world == 1 and not args.no_triton_reference:
        B_, H_, S_, D_ = case["batch_size"], case["num_heads"], case["seq_len"], case["head_dim"]
        qv, kv_, vv = (t.view(B_, H_, S_, D_) for t in (q, k, v))
        triton_ref = time_triton_reference("flash_attn", qv, kv_, vv, case["causal"], est_total["ops_alg"],
                                           statistics.median(launch_ms), ours=o.view(B_, H_, S_, D_))
    cpu = cpu_baseline(dict(case, seq_len=case["seq_len"]), args.cpu_baseline_seconds) \
        if rank == 0 and world == 1 and not args.no_cpu_baseline else None
    if rank == 0:
        clocks = clk.summary()
        # both products at the fp16 rate: the mixed roofline with P.V's kind for QK^T too
        rl = tensor_rooflines(read_tensor_peaks(), clocks.get("sm_mhz"), 0.0, 1.0, "16bit")
        bf16 = rl["pv"]
        value = est_total["ops_alg"] * args.steps / (total_ms * 1e-3) / 1e12
        achieved = est_rank["ops_alg"] / (statistics.mean(launch_ms) * 1e-3) / 1e12
        line = {
            "metric": "flash_attn TFLOPS (fp16 QK^T and P.V) vs fp16 tensor peak", "value": round(value, 2),
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4), "p50_ms": round(statistics.median(launch_ms), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 QK^T + fp16 P.V (fp32 accumulate, fp32 softmax)",
            "data": "synthetic (seeded per (batch, head) slab; q, k, v ~ N(0, 1))",
            "config": config_dict(case, world),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": bf16, "unit": "TFLOP/s",
                         "frac": round(achieved / bf16, 4), "traffic": None, "kernel": "sage_attn_kernel (FLASH)",
                         "peak_source": rl["source"] + " (the fp16 rate for both products)",
                         "peak_sustained": rl.get("mixed_sustained"),
                         "frac_vs_sustained": round(achieved / rl["mixed_sustained"], 4)
                         if rl.get("mixed_sustained") else None},
            "clocks": clocks,
            "e2e": {"value": round(est_total["ops_alg"] * e2e_steps / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 3 * q.numel() * q.element_size(),
                    "d2h_bytes_per_step": o.numel() * o.element_size(),
                    "ms_per_step": round(e2e_ms / e2e_steps, 3)},
            "gpu_launches": args.steps,
        }
        if tri is not None:
            line["tribench_timing"] = {k_: (round(v_, 5) if isinstance(v_, float) else v_) for k_, v_ in tri.items()}
        if triton_ref is not None:
            line["triton_reference"] = triton_ref
        if cpu is not None:
            cpu["unit"] = "TFLOP/s"
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.workload.startswith("fa_"):
        if args.impl == "reference":
            return run_reference(args)
        return main_flash(args)
    if args.impl == "reference":
        return run_reference(args)
    rank, world, local = dist_env()
    import tribench_b200 as tb

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        pg = dist
    case = workload_case(args.workload, world)
    B, H, S, D = case["batch_size"], case["num_heads"], case["seq_len"], case["head_dim"]
    strong = case["shard"] == "strong"
    gather = world > 1  # the final output gather to rank 0
    sd = shard.make_shard(case, rank, world)
    nh_total, lo, hi = sd.total, sd.lo, sd.hi
    inp = tb.make_inputs(case, dev, seed=case["seed"], dtype=case["dtype"], heads=(lo, hi))
    q, k, v = inp["q"], inp["k"], inp["v"]
    causal, pv = case["causal"], case["pv"]
    peer, gather_note = None, None
    if gather and args.gather in ("copy", "peer"):
        # the whole output on rank 0, mapped into every rank: the kernels store into it directly
        try:
            peer = shard.PeerOutput((1, nh_total, S, D), q.dtype, 0, dev)
        except Exception as e:  # no IPC / peer access: the NCCL gather instead
            gather_note = f"peer mapping unavailable ({type(e).__name__}: {e}); NCCL gather used"
    nccl_gather = gather and peer is None
    copy_gather = peer is not None and args.gather == "copy"
    if args.waves:
        n_waves = args.waves
    elif nccl_gather:
        n_waves = 8 if strong else 4
    elif copy_gather:
        n_waves = 8
    else:
        n_waves = 1 if not strong or gather else 8
    waves = shard.wave_ranges(lo, hi, n_waves)

    def make_plans(blkq=128):
        out = {}
        for (a, b) in waves:
            if b - a not in out:
                out[b - a] = tb.SagePlan(1, b - a, b - a, S, S, D, q.dtype, dev, pv=pv, smooth_k=True, causal=causal,
                                         blkq=blkq)
        return out

    plans = make_plans() if not copy_gather else {}
    # copy gather: one pre-pass over all this rank's heads, then the attention waves read its
    # buffers (disjoint head ranges) from two streams
    plan_all = (tb.SagePlan(1, hi - lo, hi - lo, S, S, D, q.dtype, dev, pv=pv, smooth_k=True, causal=causal)
                if copy_gather else None)
    plan = plan_all if copy_gather else plans[waves[0][1] - waves[0][0]]
    full = None
    if copy_gather:
        # rank 0 computes straight into its slice of the mapped buffer; the others compute
        # locally and the copy engine moves each finished wave into the mapping
        full = peer.tensor
        o = full[:, lo:hi] if rank == 0 else torch.empty_like(q)
    elif peer is not None:
        # every rank's slice of rank 0's buffer (local on rank 0, a peer mapping elsewhere)
        full = peer.tensor
        o = full[:, lo:hi]
    elif gather and rank == 0:
        # the whole job's output lives on rank 0; its own heads are computed straight into it
        full = torch.empty((1, nh_total, S, D), dtype=q.dtype, device=dev)
        o = full[:, lo:hi]
    else:
        o = torch.empty_like(q)
    est_rank = tb.estimate(dict(case, batch_size=1, num_heads=hi - lo))
    est_total = tb.estimate(case)
    stream = torch.cuda.current_stream(dev)
    flush = None
    if 3 * q.numel() * q.element_size() <= L2_BYTES:
        flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)

    def barrier():
        if pg is not None:
            pg.barrier()

    # one wave = pre-pass + attention over a range of heads: the two C calls sage_run makes
    # (sage_prepass, then sage_attn_fwd, or at head_dim 128 sage_attn_fwd_fused_q, which quantises
    # Q itself), split so that CUDA events bracket the attention kernel
    def wave(a, b, ev=None, pls=None):
        i, j = a - lo, b - lo
        pl = (pls or plans)[j - i]
        cur = torch.cuda.current_stream(dev)
        if ev is not None:
            ev[0].record(cur)
        pl.prepass(q[:, i:j], k[:, i:j], v[:, i:j])
        if ev is not None:
            ev[1].record(cur)
        pl.attention(v[:, i:j], o[:, i:j], q=q[:, i:j])
        if ev is not None:
            ev[2].record(cur)

    # one step = every wave of this rank; N > 1: with the copy gather each finished wave is
    # copied into rank 0's buffer while the next ones compute, with peer stores the output is on
    # rank 0 already, with the NCCL gather each wave is sent while the next one is computed
    cg = shard.CopyGather(peer, lo, o) if copy_gather else None
    cg_events = []

    def step(wave_events=None, pls=None):
        if flush is not None:
            flush.zero_()
        it = iter(wave_events) if wave_events is not None else None

        def compute(a, b):
            wave(a, b, next(it) if it is not None else None, pls)

        if cg is not None:
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(stream)
            plan_all.prepass(q, k, v)
            p1.record(stream)

            def attention_wave(a, b, slot):
                ev = next(it) if it is not None else None
                cur = torch.cuda.current_stream(dev)
                i, j = a - lo, b - lo
                if ev is not None:
                    ev[0].record(cur)
                    ev[1].record(cur)
                plan_all.attention(v[:, i:j], o[:, i:j], q=q[:, i:j], heads=(i, j))
                if ev is not None:
                    ev[2].record(cur)

            evs_ = cg.step(waves, attention_wave)
            if wave_events is not None:
                cg_events.append((p0, p1, *evs_))
        elif nccl_gather:
            shard.gather_to(0, o, sd, full, waves=n_waves, compute=compute, timeout_s=300.0)
        else:
            for (a, b) in waves:
                compute(a, b)

    # our kernels per wave: K-stats + finalize + quantise, then attention (copy gather: the
    # three pre-pass launches once per step, one attention launch per wave)
    launches_per_step = ((3 if plan_all.route == "fused" else 4) + len(waves)) if copy_gather else 4 * len(waves)

    evs = [[tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in waves] for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        time.sleep(0.3)  # let nvidia-smi start before the GPU is loaded
        clk.mark()
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        assert tb.device_status(dev) == 0
        # ---- timed region: K steps, device time, max over ranks
        barrier()
        torch.cuda.synchronize(dev)
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            step(evs[i])
            ends[i].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [evs[i][0][0].elapsed_time(ends[i]) for i in range(args.steps)]
    attn_ms = [sum(w[1].elapsed_time(w[2]) for w in evs[i]) for i in range(args.steps)]
    pre_ms = [sum(w[0].elapsed_time(w[1]) for w in evs[i]) for i in range(args.steps)]
    status = tb.device_status(dev)
    if cg is not None:
        # waves overlap on two streams: this rank's compute span is start -> the later stream end
        compute_ms = statistics.mean(max(p0.elapsed_time(em), p0.elapsed_time(ea)) for p0, _, _, em, ea, _ in cg_events)
        pre_ms = [p0.elapsed_time(p1) for p0, p1, *_ in cg_events]
        step_ms = [ev[0].elapsed_time(ends[i]) for i, ev in enumerate(cg_events)]
    else:
        compute_ms = statistics.mean(a + b for a, b in zip(attn_ms, pre_ms))
    if pg is not None:
        # rank 0 stores its own rows into local memory: its compute time is the step without
        # any gather traffic of its own, the yardstick for what the gather costs
        t = torch.tensor([total_ms, compute_ms, compute_ms if rank == 0 else 0.0], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        total_ms, compute_ms_max, compute_ms_r0 = (float(x) for x in t.tolist())
    else:
        compute_ms_max = compute_ms_r0 = compute_ms

    # ---- end to end through the public API: host (pinned) inputs -> device -> run -> host output
    e2e_ms = None
    if args.e2e_steps > 0 and not strong:
        e2e_ms = run_e2e(args, case, q, k, v, o, dev, stream, barrier, pg)

    # the drop-in run(q, k, v, causal) measured the way `tribench run` measures a variant
    tri = None
    if world == 1 and not args.no_tribench_timing:
        qv, kv_, vv = (t.view(B, H, S, D) for t in (q, k, v)) if not strong else (q, k, v)
        lat = timing.do_bench(lambda: tb.run(qv, kv_, vv, causal=causal, pv=pv), device=dev)
        tri = timing.summarize(lat, flops=est_total["flops"])
        tri["call"] = "tribench_b200.run(q, k, v, causal) (the plugin's run; output allocated per call)"
        tri["timer"] = "do_bench restated without Triton: 256 MB L2 flush per rep, warmup 200 ms, rep 2000 ms"

    # the same step with one Q scale per token (blkq=1), beside the default 128-row blocks
    blkq1 = None
    if world == 1 and not args.no_blkq1:
        p1 = make_plans(blkq=1)
        reps = max(3, min(args.steps, 50))
        for _ in range(3):
            step(pls=p1)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            step(pls=p1)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms1 = e0.elapsed_time(e1) / reps
        # the default step again right after, so both see the same clock
        e0.record(stream)
        for _ in range(reps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms128 = e0.elapsed_time(e1) / reps
        blkq1 = {"ms_per_step": round(ms1, 4), "value": round(est_total["ops_alg"] / (ms1 * 1e-3) / 1e12, 2),
                 "default_ms_per_step_same_window": round(ms128, 4), "steps": reps,
                 "note": "one Q scale per token (per_block_int8 BLKQ=1) on every route; same step otherwise"}
        del p1
        assert tb.device_status(dev) == 0

    # the reference's own Triton kernel on the same inputs (non-causal only: it ignores causal)
    triton_ref = None
    if world == 1 and not args.no_triton_reference:
        qv, kv_, vv = (t.view(B, H, S, D) for t in (q, k, v))
        triton_ref = time_triton_reference("sage_attn", qv, kv_, vv, causal, est_total["ops_alg"],
                                           statistics.median(step_ms), ours=o.view(B, H, S, D))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(case, args.cpu_baseline_seconds)

    if rank == 0:
        ops_total = est_total["ops_alg"]
        value = ops_total * args.steps / (total_ms * 1e-3) / 1e12
        clocks = clk.summary()
        rl = tensor_rooflines(read_tensor_peaks(), clocks.get("sm_mhz"), est_rank["ops_qk"], est_rank["ops_pv"], pv)
        # copy gather: the waves overlap on two streams, so the attention time is rank 0's
        # compute span (pre-pass start to the later stream's end) minus its pre-pass
        attn_avg = compute_ms - statistics.mean(pre_ms) if cg is not None else statistics.mean(attn_ms)
        achieved = est_rank["ops_alg"] / (attn_avg * 1e-3) / 1e12
        traffic = read_traffic().get(f"attn_{args.workload}_bytes_per_launch")
        peaks = read_peaks()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
            "p50_ms": round(statistics.median(step_ms), 4), "higher_is_better": True,
            "scaling": "strong" if case["shard"] == "strong" else "weak", "vs_baseline": None,
            "dtype": "int8 QK^T + " + ("e4m3" if pv == "fp8" else case["dtype"]) + " P.V (fp32 accumulate)",
            "data": "synthetic (seeded per (batch, head) slab; BASELINE distributions)",
            "config": config_dict(case, world),
            "frac_of_int8_peak": round(value / world / rl["int8"], 4),
            "int8_peak": {"tops": rl["int8"], "sustained_tops": rl.get("int8_sustained"),
                          "frac_vs_sustained": round(value / world / rl["int8_sustained"], 4)
                          if rl.get("int8_sustained") else None, "source": rl["source"]},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": rl["mixed"],
                         "unit": "TFLOP/s", "frac": round(achieved / rl["mixed"], 4), "traffic": traffic,
                         "kernel": "sage_attn_kernel",
                         "peak_source": rl["source"] + f": QK^T at the int8 rate ({rl['int8']} TOPS), P.V at the "
                                        f"{'e4m3' if pv == 'fp8' else 'fp16'} rate ({rl['pv']} TOPS), harmonic mix",
                         "peak_sustained_mixed": rl.get("mixed_sustained"),
                         "frac_vs_sustained_mixed": round(achieved / rl["mixed_sustained"], 4)
                         if rl.get("mixed_sustained") else None,
                         "attn_ms": round(attn_avg, 4), "prepass_ms": round(statistics.mean(pre_ms), 4),
                         **({"note": "attention waves overlap on two streams: attn_ms is rank 0's span from the "
                                     "first wave's start to the last wave's end (compute span minus pre-pass)"}
                            if cg is not None else {})},
            "prepass_roofline": {"bound": "hbm", "achieved": round(tb.prepass_bytes(dict(case, batch_size=1,
                                 num_heads=hi - lo), fused_q=plan.fused_q) / (statistics.mean(pre_ms) * 1e-3) / 1e9, 1),
                                 "peak": peaks["hbm"], "unit": "GB/s",
                                 "kernels": "kv_stats + kv_finalize + quant (3 launches)",
                                 "q_quantised_in": "attention kernel" if plan.fused_q else "pre-pass"},
            "clocks": clocks,
            "e2e": None if e2e_ms is None else {
                "value": round(ops_total * args.e2e_steps / (e2e_ms * 1e-3) / 1e12, 2), "unit": UNIT,
                "h2d_bytes_per_step": 3 * q.numel() * q.element_size(),
                "d2h_bytes_per_step": o.numel() * o.element_size(),
                "ms_per_step": round(e2e_ms / args.e2e_steps, 3),
                "api": f"HostPipeline.run, {args.e2e_chunks} chunks (pinned host buffers)"},
            "gpu_launches": launches_per_step * args.steps,
            "waves_per_rank": len(waves),
            "device_status": status,
        }
        if gather:
            line["gather"] = {"dst_rank": 0,
                              "bytes_received_per_step": (nh_total - (hi - lo)) * S * D * q.element_size(),
                              "method": "NCCL point to point per wave" if nccl_gather else
                              "copy engine: each rank's finished waves copied (cudaMemcpyAsync) into rank 0's "
                              "output over NVLink (CUDA IPC mapping), no collective" if copy_gather else
                              "peer stores: each rank's attention epilogue writes its rows into rank 0's "
                              "output over NVLink (CUDA IPC mapping), no collective",
                              "overlapped": "each rank sends wave w while computing wave w+1" if nccl_gather else
                              f"{len(waves)} waves alternating over two compute streams; wave w copied on a "
                              "third stream while later waves compute" if copy_gather else
                              "the stores are the kernel's own output stores, spread over its run",
                              "compute_ms_per_step_rank0": round(compute_ms_r0, 4),
                              "compute_ms_per_step_max_over_ranks": round(compute_ms_max, 4),
                              "exposed_ms_per_step": round(total_ms / args.steps - compute_ms_max, 4),
                              "cost_vs_rank0_ms_per_step": round(total_ms / args.steps - compute_ms_r0, 4)}
        if gather_note:
            line["gather"]["note"] = gather_note
        if strong:
            line["e2e_note"] = "not measured for the sharded workload (25.8 GB of host inputs per step)"
        if tri is not None:
            line["tribench_timing"] = {k_: (round(v_, 5) if isinstance(v_, float) else v_) for k_, v_ in tri.items()}
        if blkq1 is not None:
            line["blkq_1"] = blkq1
        if triton_ref is not None:
            line["triton_reference"] = triton_ref
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del plan, plans, q, k, v, o, full
    if peer is not None:
        peer.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
