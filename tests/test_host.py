"""CPU: host-side logic of tribench_b200 — layouts, seeded inputs, estimates, the plugin entry
point's signature, and the absence of any CPU fallback."""
import inspect
import json
import os

import pytest
import torch

import tribench_b200 as tb
from tribench_b200 import sage_attn as sa

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_dims_hnd_and_nhd():
    x = torch.empty(2, 3, 5, 64)
    assert sa._dims(x, "HND") == (2, 3, 5, 64, (3 * 5 * 64, 5 * 64, 64))
    y = torch.empty(2, 5, 3, 64)  # NHD: [B, S, H, D]
    assert sa._dims(y, "NHD") == (2, 3, 5, 64, (5 * 3 * 64, 64, 3 * 64))
    with pytest.raises(ValueError):
        sa._dims(x, "XYZ")
    with pytest.raises(ValueError):
        sa._dims(x.transpose(2, 3), "HND")


def test_make_inputs_deterministic_and_shardable():
    case = dict(batch_size=2, num_heads=3, seq_len=16, head_dim=64, dist="offset", k_offset_std=2.0)
    a = tb.make_inputs(case, "cpu", seed=5, dtype="fp16")
    b = tb.make_inputs(case, "cpu", seed=5, dtype="fp16")
    assert a["q"].shape == (2, 3, 16, 64) and a["q"].dtype == torch.float16 and a["causal"] is False
    for n in ("q", "k", "v"):
        assert torch.equal(a[n], b[n])
    shard = tb.make_inputs(case, "cpu", seed=5, dtype="fp16", heads=(2, 5))
    for n in ("q", "k", "v"):
        assert torch.equal(shard[n][0], a[n].reshape(6, 16, 64)[2:5])
    c = tb.make_inputs(case, "cpu", seed=6, dtype="fp16")
    assert not torch.equal(a["q"], c["q"])


def test_make_inputs_distributions():
    S, D = 4096, 64
    off = tb.make_inputs(dict(batch_size=1, num_heads=1, seq_len=S, head_dim=D, dist="offset", k_offset_std=2.0),
                         "cpu", 0, "fp32")
    kmean = off["k"][0, 0].mean(0)
    assert kmean.std() > 1.0  # per-channel offsets ~ N(0, 4)
    assert abs(off["q"].std().item() - 1.0) < 0.05
    vc = tb.make_inputs(dict(batch_size=1, num_heads=1, seq_len=S, head_dim=D, dist="vchan"), "cpu", 0, "fp32")
    chan_std = vc["v"][0, 0].std(0)
    assert chan_std.min() > 0.4 and chan_std.max() < 4.4 and chan_std.max() / chan_std.min() > 2
    st = tb.make_inputs(dict(batch_size=1, num_heads=1, seq_len=S, head_dim=D, dist="studentt", k_offset_std=3.0),
                        "cpu", 0, "fp32")
    q = st["q"][0, 0]
    assert q.abs().max() > 8 * q.abs().median()  # heavy tails


def test_estimate_matches_tribench_formula_and_counts_causal_pairs():
    case = dict(batch_size=2, num_heads=32, seq_len=8192, head_dim=128)
    e = tb.estimate(case)
    assert e["flops"] == 4 * 2 * 32 * 8192 * 8192 * 128
    assert e["bytes"] == 4 * 2 * 32 * 8192 * 128 * 2
    assert e["ops_alg"] == e["flops"]
    ec = tb.estimate(dict(case, causal=True))
    assert ec["ops_alg"] == 4 * 2 * 32 * (8192 * 8193 // 2) * 128


def test_configs_cover_baseline():
    for name in ("c1", "c2", "c3", "c4", "c5", "h8k"):
        assert name in tb.CONFIGS
    assert tb.CONFIGS["c5"]["batch_size"] * tb.CONFIGS["c5"]["num_heads"] == 1024
    assert tb.CONFIGS["c4"]["pv"] == "fp8" and tb.CONFIGS["c4"]["dtype"] == "bf16"


def test_plugin_entry_point_matches_reference_signature():
    import importlib.util

    path = os.path.join(ROOT, "kernels", "sage_attn", "cuda_impl.py")
    spec = importlib.util.spec_from_file_location("tribench.kernels.sage_attn.cuda_impl", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sig = inspect.signature(mod.run)
    # run_sage_attn(q, k, v, causal=False, sm_scale=None) — kernels/sage_attn/triton_impl.py:162
    assert list(sig.parameters) == ["q", "k", "v", "causal", "sm_scale"]
    assert sig.parameters["causal"].default is False and sig.parameters["sm_scale"].default is None


def test_meta_patch_registers_cuda_variant():
    patch = json.load(open(os.path.join(ROOT, "kernels", "sage_attn", "meta_patch.json")))
    variants = patch["entrypoints"]["variants"]
    assert isinstance(variants, dict) and variants == {"cuda": "cuda_impl.py:run"}
    file_part, symbol = variants["cuda"].rsplit(":", 1)
    assert os.path.exists(os.path.join(ROOT, "kernels", "sage_attn", file_part)) and symbol == "run"


def test_no_cpu_fallback():
    q = torch.randn(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        tb.run(q, q, q)
    with pytest.raises(ValueError, match="CUDA"):
        tb.per_block_int8(q, q)


def test_per_block_int8_rejects_other_block_sizes():
    """BLKQ takes the five sizes the kernels implement (128, 64, 32, 16, 1); BLKK only 64. Both
    are checked before any tensor is looked at (these are CPU tensors)."""
    q = torch.randn(1, 1, 8, 64, dtype=torch.float16)
    for blkq in (8, 48, 256):
        with pytest.raises(ValueError, match="BLKQ"):
            tb.per_block_int8(q, q, BLKQ=blkq)
    with pytest.raises(ValueError, match="BLKK"):
        tb.per_block_int8(q, q, BLKK=32)
    with pytest.raises(ValueError, match="blkq|BLKQ"):
        tb.SagePlan(1, 1, 1, 8, 8, 64, torch.float16, "cpu", blkq=3)


def test_product_does_not_import_oracle():
    pkg = os.path.join(ROOT, "tribench_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f


def test_host_pipeline_rejects_cpu_device_and_bad_heads():
    with pytest.raises(ValueError):
        tb.HostPipeline(1, 4, 4, 128, 128, 64, torch.float16, "cpu")
    with pytest.raises(ValueError):
        tb.HostPipeline(1, 6, 4, 128, 128, 64, torch.float16, "cuda:0")


def test_tribench_latency_summary_matches_numpy_definitions():
    import numpy as np

    from tribench_b200 import timing

    lat = [1.0, 1.2, 0.9, 1.1, 3.0, 1.05, 0.95, 1.0]
    got = timing.summarize(lat, flops=2e12, nbytes=4e9)
    a = np.array(lat)
    for key, q in (("latency_ms_p50", 50), ("latency_ms_p90", 90), ("latency_ms_p95", 95), ("latency_ms_p99", 99)):
        assert got[key] == pytest.approx(float(np.percentile(a, q)))
    assert got["latency_ms_std"] == pytest.approx(float(np.std(a)))
    assert got["latency_ms_mean"] == pytest.approx(float(np.mean(a)))
    assert got["tail_ratio_p99_p50"] == pytest.approx(float(np.percentile(a, 99) / np.percentile(a, 50)))
    assert got["jitter_cv"] == pytest.approx(float(np.std(a) / np.mean(a)))
    assert got["tflops"] == pytest.approx(2e12 / (float(np.percentile(a, 50)) * 1e-3) / 1e12)
    assert got["gbps"] == pytest.approx(4e9 / (float(np.percentile(a, 50)) * 1e-3) / 1e9)
