"""GPU: Q quantised inside the attention kernel (SAGE_FLAG_FUSED_Q) against the pre-pass path.

The fused kernel applies the pre-pass's arithmetic to each 128-row query tile, so its INT8 codes
and scales, and therefore the whole output, must be BIT-IDENTICAL to the default path (which is
bit-exact against the oracle for the codes and within the written tolerances for the output in
tests/test_gpu_parity.py).
"""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _qkv(B, Hq, Hkv, S, D, dtype, seed, Skv=None):
    g = torch.Generator(device=DEV).manual_seed(seed)
    Skv = S if Skv is None else Skv
    q = torch.randn(B, Hq, S, D, generator=g, device=DEV).to(dtype)
    k = (torch.randn(B, Hkv, Skv, D, generator=g, device=DEV) + 2 * torch.randn(B, Hkv, 1, D, generator=g,
                                                                                device=DEV)).to(dtype)
    v = torch.randn(B, Hkv, Skv, D, generator=g, device=DEV).to(dtype)
    return q, k, v


@pytest.mark.parametrize("B,Hq,Hkv,S,Skv,D,dtype,causal,pv", [
    (2, 4, 4, 1000, None, 128, torch.float16, False, "16bit"),
    (2, 4, 2, 777, None, 64, torch.float16, True, "16bit"),
    (1, 4, 4, 2048, None, 128, torch.bfloat16, True, "fp8"),
    (1, 8, 1, 300, 1537, 64, torch.bfloat16, False, "fp8"),
    (1, 2, 2, 1, None, 128, torch.float16, False, "16bit"),
    (3, 2, 2, 129, None, 64, torch.float16, True, "16bit"),
])
def test_fused_q_output_bit_identical(B, Hq, Hkv, S, Skv, D, dtype, causal, pv):
    q, k, v = _qkv(B, Hq, Hkv, S, D, dtype, seed=S + D, Skv=Skv)
    ref = tb.run(q, k, v, causal=causal, pv=pv, fused_q=False)
    out = tb.run(q, k, v, causal=causal, pv=pv, fused_q=True)
    assert tb.device_status(DEV) == 0
    assert torch.equal(out, ref)
    if D == 128:  # sage_run's own choice there is the fused route
        assert torch.equal(tb.run(q, k, v, causal=causal, pv=pv), ref)


@pytest.mark.parametrize("D", [64, 128])
def test_fused_q_codes_and_scales_equal_prepass(D):
    B, H, S = 2, 3, 1000
    q, k, v = _qkv(B, H, H, S, D, torch.float16, seed=D)
    qn, kn, vn = (t.transpose(1, 2).contiguous() for t in (q, k, v))  # NHD
    plan = tb.SagePlan(B, H, H, S, S, D, q.dtype, DEV, fused_q=True, keep_q_int8=True)
    out = plan.run(qn, kn, vn, tensor_layout="NHD")
    assert tb.device_status(DEV) == 0
    qi, qs, _, _ = tb.per_block_int8(qn, kn, tensor_layout="NHD")
    assert torch.equal(plan.quant.q_int8, qi) and torch.equal(plan.quant.q_scale, qs)
    assert torch.equal(out, tb.run(qn, kn, vn, tensor_layout="NHD", fused_q=False))
    # the split form bench.py times: sage_prepass(FUSED_Q) + sage_attn_fwd_fused_q
    out2 = torch.empty_like(qn)
    plan.prepass(qn, kn, vn, tensor_layout="NHD")
    plan.attention(vn, out2, tensor_layout="NHD", q=qn)
    assert torch.equal(out2, out)


def test_fused_q_packed_sequences():
    lens = [(1, 1), (129, 200), (300, 513), (0, 5), (777, 1000), (5, 0)]
    g = torch.Generator(device=DEV).manual_seed(5)
    tq, tk = sum(a for a, _ in lens), sum(b for _, b in lens)
    q = torch.randn(tq, 4, 128, generator=g, device=DEV).half()
    k = torch.randn(tk, 2, 128, generator=g, device=DEV).half()
    v = torch.randn(tk, 2, 128, generator=g, device=DEV).half()
    cu_q, cu_k = [0], [0]
    for a, b in lens:
        cu_q.append(cu_q[-1] + a)
        cu_k.append(cu_k[-1] + b)
    ref = tb.run_sage_attn_varlen(q, k, v, cu_q, cu_k, fused_q=False)
    out = tb.run_sage_attn_varlen(q, k, v, cu_q, cu_k, fused_q=True)
    assert tb.device_status(DEV) == 0
    assert torch.equal(out, ref)
