"""Measured tensor-core peaks of this B200 (libsm100_peaks.so, include/sm100_peaks.h).

``measure(kind, n)`` times the dense tcgen05 microbenchmark two ways:
  * burst: a few launches of ~``burst_ms`` each after a warm-up, best and median rate — the
    denominator for a kernel timed on its own at full clock;
  * sustained: launches back to back for ``sustained_s`` seconds, median rate over the second
    half — the denominator for work that runs long enough for the power cap to lower the clock.
Each rate comes with the SM clocks nvidia-smi saw while it was measured.

``python -m tribench_b200.peaks [--sustained-s 4] [--json out.json]`` measures kind::i8,
kind::f16 and kind::f8f6f4 (e4m3) at N = 256 (the largest single-CTA MMA) and N = 128 (the
attention kernel's QK^T shape) and prints one JSON line per measurement.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import tempfile
import threading
import time

import torch

from ._build import PEAKS_LIB_PATH

KINDS = {"i8": 0, "f16": 1, "e4m3": 2}
_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(PEAKS_LIB_PATH):
                raise RuntimeError(f"{PEAKS_LIB_PATH} not found; build it with `python -m tribench_b200._build`")
            lib = ctypes.CDLL(PEAKS_LIB_PATH)
            lib.sm100_peak_last_error.restype = ctypes.c_char_p
            lib.sm100_peak_last_error.argtypes = []
            lib.sm100_peak_ops_per_mma.restype = ctypes.c_double
            lib.sm100_peak_ops_per_mma.argtypes = [ctypes.c_int, ctypes.c_int]
            lib.sm100_tensor_peak_launch.restype = ctypes.c_int
            lib.sm100_tensor_peak_launch.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_longlong,
                                                     ctypes.c_uint, ctypes.c_uint, ctypes.c_void_p, ctypes.c_void_p,
                                                     ctypes.c_void_p]
            _lib = lib
    return _lib


class _Clocks:
    """nvidia-smi SM clock / power samples every 20 ms while the block runs."""

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.file = gpu, None, None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", "--query-gpu=clocks.sm,power.draw,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "20"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "samples": 0}
        self.file.flush()
        sm, pw, capped = [], [], 0
        with open(self.file.name) as f:
            for row in f:
                parts = [x.strip() for x in row.split(",")]
                try:
                    sm.append(float(parts[0]))
                    pw.append(float(parts[1]))
                    capped += parts[2].lower() == "active"
                except (ValueError, IndexError):
                    continue
        os.unlink(self.file.name)
        loaded = [s for s, p in zip(sm, pw) if p > 300.0] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "samples": len(sm),
                "samples_under_load": len(loaded), "power_w_max": max(pw) if pw else None,
                "sw_power_cap_samples": capped}


def _launch(lib, kind: int, n: int, ctas: int, mmas: int, status: torch.Tensor, timing, stream) -> None:
    rc = lib.sm100_tensor_peak_launch(kind, n, ctas, mmas, 12345, 10000, ctypes.c_void_p(status.data_ptr()),
                                      ctypes.c_void_p(timing.data_ptr()) if timing is not None else None,
                                      ctypes.c_void_p(stream.cuda_stream))
    if rc != 0:
        raise RuntimeError(f"sm100_tensor_peak_launch failed ({rc}): {lib.sm100_peak_last_error().decode()}")


MAX_SM_MHZ = 1965.0  # B200 clocks.max.sm


def measure(kind: str, n: int = 256, *, burst_ms: float = 20.0, burst_reps: int = 8, sustained_s: float = 0.0,
            device: int = 0, clocks: bool = True) -> dict:
    """Dense tcgen05 rate of `kind` ("i8", "f16", "e4m3") with M128 x n MMAs on every SM, in
    TOPS (= TFLOP/s for the float kinds).

    Besides the event-timed rates, each CTA reports the SM cycles and nanoseconds its MMAs took
    (clock64 / globaltimer), which give the rate per SM clock (``ops_per_clk_per_sm``, clock
    independent) and the SM clock the launch actually ran at (``kernel_mhz``)."""
    lib = load()
    k = KINDS[kind]
    dev = torch.device("cuda", device)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    ops_mma = lib.sm100_peak_ops_per_mma(k, n)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    timing = torch.zeros(2 * sms, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)

        def timed(mmas: int) -> tuple[float, float, float]:
            """(event ms, median SM cycles per CTA, median in-kernel SM MHz)"""
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            _launch(lib, k, n, sms, mmas, status, timing, stream)
            e1.record(stream)
            e1.synchronize()
            t = timing.view(sms, 2).double().cpu()
            cyc, ns = t[:, 0], t[:, 1].clamp(min=1)
            return e0.elapsed_time(e1), float(cyc.median()), float((cyc / ns).median() * 1e3)

        # warm up, calibrate the launch length, warm up again
        probe = 4096
        timed(probe)
        ms, _, _ = timed(probe)
        mmas = max(4, int(probe * burst_ms / max(ms, 1e-3)) // 4 * 4)
        for _ in range(3):
            timed(mmas)
        ops = ops_mma * mmas * sms
        out = {"kind": kind, "n": n, "m": 128, "sms": sms, "mma_per_cta": mmas, "ops_per_launch": ops}
        with _Clocks(device) if clocks else _NoClocks() as ck:
            runs = [timed(mmas) for _ in range(burst_reps)]
        times = [r[0] for r in runs]
        rates = [ops / (t * 1e-3) / 1e12 for t in times]
        per_clk = statistics.median(ops_mma * mmas / r[1] for r in runs)
        out["burst"] = {"tops_best": round(max(rates), 1), "tops_median": round(statistics.median(rates), 1),
                        "launch_ms_median": round(statistics.median(times), 3),
                        "kernel_mhz": round(statistics.median(r[2] for r in runs), 1),
                        "ops_per_clk_per_sm": round(per_clk, 1),
                        "tops_at_max_clock": round(per_clk * sms * MAX_SM_MHZ * 1e6 / 1e12, 1),
                        "clocks": ck.summary()}
        if sustained_s > 0:
            with _Clocks(device) if clocks else _NoClocks() as ck:
                evs = []
                t_end = time.time() + sustained_s
                while time.time() < t_end:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    _launch(lib, k, n, sms, mmas, status, timing, stream)
                    e1.record(stream)
                    evs.append((e0, e1))
                    if len(evs) > 4:
                        evs[-4][1].synchronize()  # keep a few launches queued, not seconds of them
                torch.cuda.synchronize(dev)
            ts = [a.elapsed_time(b) for a, b in evs]
            tail = ts[len(ts) // 2:]
            rates = [ops / (t * 1e-3) / 1e12 for t in tail]
            t = timing.view(sms, 2).double().cpu()  # the last launch
            out["sustained"] = {"tops_median": round(statistics.median(rates), 1), "seconds": sustained_s,
                                "launches": len(ts),
                                "kernel_mhz_last_launch": round(float((t[:, 0] / t[:, 1].clamp(min=1)).median() * 1e3), 1),
                                "clocks": ck.summary()}
        torch.cuda.synchronize(dev)
        st = int(status.item())
    if st:
        raise RuntimeError(f"tensor peak kernel reported a timed-out wait (status {st})")
    return out


class _NoClocks:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def summary(self):
        return {"sm_mhz": None, "samples": 0}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sustained-s", type=float, default=4.0)
    ap.add_argument("--json", default=None, help="also write all results to this file")
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args()
    results = []
    # every burst first (a cool GPU at full clock), then the seconds-long sustained runs with a
    # pause before each, so one measurement's power-cap history does not leak into the next
    for kind in ("i8", "f16", "e4m3"):
        for n in (256, 128):
            r = measure(kind, n, device=args.device)
            results.append(r)
            print(json.dumps(r), flush=True)
            time.sleep(1.0)
    if args.sustained_s > 0:
        for kind in ("i8", "f16", "e4m3"):
            time.sleep(3.0)
            r = measure(kind, 256, sustained_s=args.sustained_s, device=args.device)
            r["run"] = "sustained"
            results.append(r)
            print(json.dumps(r), flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"gpu": torch.cuda.get_device_name(args.device), "results": results}, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
