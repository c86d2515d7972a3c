"""GPU: the Triton-free restatement of TriBench's do_bench timer on the drop-in run()."""
import pytest
import torch

import tribench_b200 as tb
from tribench_b200 import timing

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def test_do_bench_times_the_plugin_call():
    g = torch.Generator(device=DEV).manual_seed(0)
    q, k, v = (torch.randn(1, 4, 1024, 128, generator=g, device=DEV).half() for _ in range(3))
    lat = timing.do_bench(lambda: tb.run(q, k, v), warmup_ms=20, rep_ms=100, device=DEV)
    assert len(lat) >= 5 and all(x > 0 for x in lat)
    s = timing.summarize(lat, flops=tb.estimate(dict(batch_size=1, num_heads=4, seq_len=1024, head_dim=128))["flops"])
    assert s["latency_ms_min"] <= s["latency_ms_p50"] <= s["latency_ms_p99"] <= s["latency_ms_max"]
    assert s["tflops"] > 0
    assert tb.device_status(DEV) == 0
