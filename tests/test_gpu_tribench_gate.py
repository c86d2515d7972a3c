"""GPU: TriBench's own correctness gate on both packs' benchmark cases.

`tribench test` runs each variant on the pack's meta.json cases with inputs from the pack's
make_inputs (q, k, v ~ N(0, 1), kernels/*/reference.py:4-13), evaluates `ref` in the input
dtype on the same device (reference.py:15-24 for sage_attn, :15-28 for flash_attn), resolves the
tolerance (tribench/correctness.py:22-38: a per-dtype entry, else the pack's non-default
atol/rtol, else the dtype default) and passes iff torch.allclose(ref.float(), out.float())
(:80-82). This test restates that gate and applies it to the cuda variants' run() at full size:
sage_attn (atol = rtol = 5e-2, kernels/sage_attn/meta.json:45-48) and flash_attn (1e-2).
"""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
DEFAULT_TOL = {"fp16": (1e-2, 1e-2), "bf16": (1e-2, 1e-2)}
CASES = {"s4k_d64": (8, 16, 4096, 64), "s8k_d64": (4, 16, 8192, 64)}


def tolerance(dtype_str, atol, rtol, per_dtype=None):
    """tribench/correctness.py:_get_tolerance."""
    if per_dtype and dtype_str in per_dtype:
        return per_dtype[dtype_str].get("atol", atol), per_dtype[dtype_str].get("rtol", rtol)
    if atol != 1e-2 or rtol != 1e-2:
        return atol, rtol
    return DEFAULT_TOL.get(dtype_str, (atol, rtol))


def ref_in_dtype(q, k, v, causal=False):
    """The packs' ref: softmax(q k^T * D^-0.5) v in the input dtype, one batch at a time."""
    out = torch.empty_like(q)
    for b in range(q.shape[0]):
        p = torch.matmul(q[b], k[b].transpose(1, 2)) * q.shape[-1] ** -0.5
        out[b] = torch.matmul(torch.softmax(p, dim=-1), v[b])
    return out


@pytest.mark.parametrize("pack", ["sage_attn", "flash_attn"])
@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("dtype_str", ["fp16", "bf16"])
def test_tribench_gate_on_pack_cases(pack, case, dtype_str):
    B, H, S, D = CASES[case]
    dtype = torch.float16 if dtype_str == "fp16" else torch.bfloat16
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, device=DEV, dtype=dtype) for _ in range(3))
    run = tb.run if pack == "sage_attn" else tb.run_flash_attn
    out = run(q, k, v, causal=False)
    assert tb.device_status(DEV) == 0
    ref = ref_in_dtype(q, k, v)
    atol, rtol = tolerance(dtype_str, *((5e-2, 5e-2) if pack == "sage_attn" else (1e-2, 1e-2)))
    diff = (ref.float() - out.float()).abs()
    print(f"{pack} {case} {dtype_str}: max_abs_err {diff.max().item():.3e} (atol {atol}, rtol {rtol})")
    assert torch.allclose(ref.float(), out.float(), atol=atol, rtol=rtol)
