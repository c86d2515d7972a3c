"""GPU: the head_dim-64 route of sage_run — INT8 codes held as fp16 values, QK^T as kind::f16.

The pre-pass stores each code c in [-127, 127] as the fp16 value c (exact), and the f16 MMA's
fp32 scores are the INT8 MMA's integer scores exactly (every partial sum is an integer below
2^24), so this route evaluates the same block scheme; only the softmax's float rounding differs
from the INT8 route (no 1.5 * 2^23 bias term). Checked here: the codes are the INT8 codes (bit
for bit, through sage_prepass with SAGE_FLAG_CODES16), the split form equals sage_run bit for
bit, and the output stays within the INT8 route's own rounding distance of it (16-bit P.V) or
within the FP8 P.V bound relative to |V| max. Against the oracle the route is covered by every
head_dim-64 case of tests/test_gpu_parity.py, which now runs through it.
"""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _qkv(B, Hq, Hkv, S, dtype, seed, Skv=None):
    g = torch.Generator(device=DEV).manual_seed(seed)
    Skv = S if Skv is None else Skv
    q = torch.randn(B, Hq, S, 64, generator=g, device=DEV).to(dtype)
    k = (torch.randn(B, Hkv, Skv, 64, generator=g, device=DEV) + 2 * torch.randn(B, Hkv, 1, 64, generator=g,
                                                                                 device=DEV)).to(dtype)
    v = torch.randn(B, Hkv, Skv, 64, generator=g, device=DEV).to(dtype)
    return q, k, v


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_codes16_are_the_int8_codes(dtype):
    B, H, S = 2, 3, 1000
    q, k, v = _qkv(B, H, H, S, dtype, seed=1)
    plan = tb.SagePlan(B, H, H, S, S, 64, dtype, DEV)
    assert plan.route == "codes16"
    plan.prepass(q, k, v)
    qi, qs, ki, ks, km = tb.per_block_int8(q, k, smooth_k=True, return_km=True)
    assert tb.device_status(DEV) == 0
    qc, kc = plan.codes16
    assert torch.equal(qc, qi.half()) and torch.equal(kc, ki.half())
    assert torch.equal(plan.quant.q_scale, qs) and torch.equal(plan.quant.k_scale, ks)
    assert torch.equal(plan.quant.k_mean, km)


@pytest.mark.parametrize("B,Hq,Hkv,S,Skv,dtype,causal,pv", [
    (2, 4, 4, 1000, None, torch.float16, False, "16bit"),
    (2, 4, 2, 777, None, torch.float16, True, "16bit"),
    (1, 8, 1, 300, 1537, torch.bfloat16, False, "16bit"),
    (1, 4, 4, 2048, None, torch.bfloat16, True, "fp8"),
    (3, 2, 2, 129, None, torch.float16, True, "fp8"),
])
def test_codes16_route_matches_int8_route(B, Hq, Hkv, S, Skv, dtype, causal, pv):
    q, k, v = _qkv(B, Hq, Hkv, S, dtype, seed=S, Skv=Skv)
    out = tb.run(q, k, v, causal=causal, pv=pv)  # head_dim 64: the fp16-code route
    ref = tb.run(q, k, v, causal=causal, pv=pv, fused_q=False)  # INT8 operands
    assert tb.device_status(DEV) == 0
    err = (out.float() - ref.float()).abs().max().item()
    if pv == "fp8":
        # a different float rounding may move a lazy-rescale decision, and then P's e4m3 rounding
        bound = 2.5e-2 * v.float().abs().max().item()
    else:
        bound = 4e-3 if dtype == torch.float16 else 1.6e-2
    print(f"codes16 vs int8 route: max-abs {err:.2e} (bound {bound:.2e})")
    assert err <= bound
    # the split form (sage_prepass + SAGE_FLAG_CODES16, sage_attn_fwd_codes16) is sage_run exactly
    plan = tb.SagePlan(B, Hq, Hkv, S, S if Skv is None else Skv, 64, dtype, DEV, pv=pv, causal=causal)
    o2 = torch.empty_like(q)
    plan.prepass(q, k, v)
    plan.attention(v, o2)
    assert torch.equal(o2, out)


def test_codes16_nhd_output_holds_the_q_codes_in_flight():
    """sage_run keeps the Q codes in o until the kernel overwrites them: an NHD o (strided rows)
    must give the HND result."""
    q, k, v = _qkv(2, 3, 3, 640, torch.float16, seed=9)
    ref = tb.run(q, k, v)
    qn, kn, vn = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    out = tb.run(qn, kn, vn, tensor_layout="NHD")
    assert tb.device_status(DEV) == 0
    assert torch.equal(out.transpose(1, 2), ref)
