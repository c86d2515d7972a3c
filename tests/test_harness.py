"""CPU: the chunked form of TriBench's correctness gate (tribench_b200.harness).

``ref_chunked`` must equal the packs' ``ref`` (kernels/sage_attn/reference.py:15-24, restated
unchunked below) whatever the chunking, and ``gate_chunked`` must give TriBench's verdict
(tolerance resolution of correctness.py:22-38, allclose of :80-82) and its error statistics.
"""
import pytest
import torch

from tribench_b200 import harness


def ref_unchunked(q, k, v, causal=False, sm_scale=None):
    """The packs' ref as written (one matmul over all heads; GQA by repeating K/V heads)."""
    g = q.shape[1] // k.shape[1]
    k, v = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    p = torch.matmul(q, k.transpose(2, 3)) * sm_scale
    if causal:
        S = q.shape[2]
        p = p.masked_fill(torch.tril(torch.ones((S, S))) == 0, float("-inf"))
    return torch.matmul(torch.softmax(p, dim=-1), v)


def _qkv(B, Hq, Hkv, Sq, Skv, D, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, Hq, Sq, D, generator=g).to(dtype), torch.randn(B, Hkv, Skv, D, generator=g).to(dtype),
            torch.randn(B, Hkv, Skv, D, generator=g).to(dtype))


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("budget", [1 << 30, 3 * 200 * 4 * 7, 1])  # one chunk per head, 7 rows, 1 row
def test_ref_chunked_equals_ref(causal, budget):
    q, k, v = _qkv(2, 3, 3, 200, 200, 32, seed=1)
    want = ref_unchunked(q, k, v, causal)
    got = harness.ref_chunked(q, k, v, causal, budget_bytes=budget)
    torch.testing.assert_close(got, want, atol=2e-6, rtol=1e-5)


def test_ref_chunked_gqa_cross_nhd_and_scale():
    q, k, v = _qkv(1, 4, 2, 70, 130, 16, seed=2)
    want = ref_unchunked(q, k, v, False, sm_scale=0.3)
    got = harness.ref_chunked(q, k, v, False, 0.3, budget_bytes=3 * 130 * 4 * 16)
    torch.testing.assert_close(got, want, atol=2e-6, rtol=1e-5)
    qn, kn, vn = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    gotn = harness.ref_chunked(qn, kn, vn, False, 0.3, tensor_layout="NHD")
    torch.testing.assert_close(gotn.transpose(1, 2), want, atol=2e-6, rtol=1e-5)


def test_ref_chunked_rejects_causal_cross_lengths():
    q, k, v = _qkv(1, 1, 1, 8, 16, 8, seed=3)
    with pytest.raises(ValueError):
        harness.ref_chunked(q, k, v, causal=True)


def test_tolerance_resolution():
    assert harness.tolerance("fp16", 5e-2, 5e-2) == (5e-2, 5e-2)  # pack override
    assert harness.tolerance("fp16", 1e-2, 1e-2) == (1e-2, 1e-2)
    assert harness.tolerance("fp32", 1e-2, 1e-2) == (1e-5, 1e-4)  # framework default
    assert harness.tolerance("bf16", 5e-2, 5e-2, {"bf16": {"atol": 0.1}}) == (0.1, 5e-2)


@pytest.mark.parametrize("causal", [False, True])
def test_gate_chunked_matches_unchunked_gate(causal):
    q, k, v = _qkv(1, 2, 2, 96, 96, 16, seed=4, dtype=torch.float16)
    ref = ref_unchunked(q.float(), k.float(), v.float(), causal)
    out = (ref + 3e-3 * torch.randn(ref.shape, generator=torch.Generator().manual_seed(5))).half()
    for atol in (1e-2, 2e-3):
        want = torch.allclose(ref_unchunked(q, k, v, causal).float(), out.float(), atol=atol, rtol=atol)
        r = harness.gate_chunked(out, q, k, v, causal, dtype_str="fp16", atol=atol, rtol=atol, budget_bytes=2000)
        assert r["passed"] == want and r["numel"] == out.numel()
        assert r["max_abs_err"] < 2e-2


def test_gate_chunked_counts_a_planted_error():
    q, k, v = _qkv(1, 2, 2, 64, 64, 16, seed=6, dtype=torch.float16)
    out = harness.ref_chunked(q, k, v)
    r = harness.gate_chunked(out, q, k, v, dtype_str="fp16", atol=5e-2, rtol=5e-2)
    assert r["passed"] and r["n_fail"] == 0 and r["max_abs_err"] == 0.0
    out[0, 1, 17, 3] += 0.5
    r = harness.gate_chunked(out, q, k, v, dtype_str="fp16", atol=5e-2, rtol=5e-2, budget_bytes=1)
    assert not r["passed"] and r["n_fail"] == 1 and r["max_abs_err"] >= 0.49


def test_gate_chunked_reports_worst_location():
    q, k, v = _qkv(2, 3, 3, 50, 50, 16, seed=7, dtype=torch.float16)
    out = harness.ref_chunked(q, k, v, causal=True)
    out[1, 2, 33, 9] += 0.25
    r = harness.gate_chunked(out, q, k, v, True, dtype_str="fp16", atol=5e-2, rtol=5e-2, budget_bytes=600)
    assert r["worst"] == (1, 2, 33, 9) and r["n_fail"] == 1
