"""The tcgen05 peak microbenchmark (libsm100_peaks.so): CPU checks of its C ABI, and one short
GPU measurement per operand kind (a sanity bound, not a performance gate)."""
import ctypes
import os
import re

import pytest

from tribench_b200 import peaks

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sm100_peaks.h")


def test_library_exports_every_declared_symbol():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    names = set(re.findall(r"\b(sm100_\w+)\s*\(", text))
    assert names == {"sm100_peak_last_error", "sm100_peak_ops_per_mma", "sm100_tensor_peak_launch"}
    lib = peaks.load()
    for name in names:
        assert hasattr(lib, name)


def test_ops_per_mma():
    lib = peaks.load()
    assert lib.sm100_peak_ops_per_mma(peaks.KINDS["i8"], 256) == 2 * 128 * 256 * 32
    assert lib.sm100_peak_ops_per_mma(peaks.KINDS["f16"], 128) == 2 * 128 * 128 * 16
    assert lib.sm100_peak_ops_per_mma(peaks.KINDS["e4m3"], 64) == 2 * 128 * 64 * 32
    assert lib.sm100_peak_ops_per_mma(7, 256) == 0.0
    assert lib.sm100_peak_ops_per_mma(0, 96) == 0.0


def test_launch_rejects_bad_arguments_before_any_cuda_call():
    lib = peaks.load()
    status = ctypes.c_int(0)
    sp = ctypes.cast(ctypes.pointer(status), ctypes.c_void_p)
    assert lib.sm100_tensor_peak_launch(0, 256, 148, 6, 1, 1000, sp, None, None) == -1  # not a multiple of 4
    assert lib.sm100_tensor_peak_launch(0, 256, 0, 8, 1, 1000, sp, None, None) == -1
    assert lib.sm100_tensor_peak_launch(0, 256, 148, 8, 1, 1000, None, None, None) == -1
    assert "multiple of 4" in lib.sm100_peak_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["i8", "f16", "e4m3"])
def test_tensor_peak_runs_and_reports_a_sane_rate(kind):
    r = peaks.measure(kind, 256, burst_ms=5.0, burst_reps=3, clocks=False)
    print(kind, r["burst"])
    # the in-kernel clock is a real SM clock and the per-clock rate at most the tcgen05 design rate
    # (8192 int8 / e4m3 or 4096 fp16 multiply-adds per clock per SM)
    assert 500.0 < r["burst"]["kernel_mhz"] < 2100.0
    assert r["burst"]["ops_per_clk_per_sm"] <= 1.02 * (8192 if kind == "f16" else 16384)
    # dense B200 rates are in the PFLOP/s range; this only guards against a kernel that does
    # not do the work (a rate far above the datasheet) or does not run (far below)
    lo, hi = (500.0, 6000.0) if kind != "f16" else (250.0, 3000.0)
    assert lo < r["burst"]["tops_best"] < hi
