"""GPU: SagePlan.attention over head ranges (``heads=(i, j)``) after one prepass() over all heads.

The multi-GPU copy gather runs one pre-pass per step and then the attention in waves of heads on
two streams, each wave reading its heads' slices of the plan's buffers. Every wave split must
give the single run()'s output bit for bit, on each operand route (Q quantised in the attention
kernel, INT8 codes from the pre-pass, fp16 codes at head_dim 64) and with FP8 P.V; and waves
issued on two streams must too.
"""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("D,fused_q,pv,causal", [
    (128, None, "16bit", False),
    (128, False, "16bit", True),
    (64, None, "16bit", True),
    (64, None, "fp8", False),
])
def test_head_waves_equal_one_run(D, fused_q, pv, causal):
    H, S = 6, 700
    g = torch.Generator(device=DEV).manual_seed(D + S)
    q = torch.randn(1, H, S, D, generator=g, device=DEV).half()
    k = (torch.randn(1, H, S, D, generator=g, device=DEV) + 1.0).half()
    v = torch.randn(1, H, S, D, generator=g, device=DEV).half()
    plan = tb.SagePlan(1, H, H, S, S, D, torch.float16, DEV, pv=pv, causal=causal, fused_q=fused_q)
    ref = plan.run(q, k, v).clone()
    for waves in ([(0, 6)], [(0, 1), (1, 3), (3, 6)], [(i, i + 1) for i in range(6)]):
        out = torch.full_like(ref, float("nan"))
        plan.prepass(q, k, v)
        for i, j in waves:
            plan.attention(v[:, i:j], out[:, i:j], q=q[:, i:j], heads=(i, j))
        torch.cuda.synchronize(DEV)
        assert tb.device_status(DEV) == 0
        assert torch.equal(out, ref), waves


def test_head_waves_on_two_streams():
    H, S, D = 8, 1024, 128
    g = torch.Generator(device=DEV).manual_seed(3)
    q, k, v = (torch.randn(1, H, S, D, generator=g, device=DEV).half() for _ in range(3))
    plan = tb.SagePlan(1, H, H, S, S, D, torch.float16, DEV)
    ref = plan.run(q, k, v).clone()
    out = torch.full_like(ref, float("nan"))
    main, alt = torch.cuda.current_stream(DEV), torch.cuda.Stream(DEV)
    plan.prepass(q, k, v)
    alt.wait_stream(main)
    for w, (i, j) in enumerate([(0, 2), (2, 4), (4, 6), (6, 8)]):
        with torch.cuda.stream(main if w % 2 == 0 else alt):
            plan.attention(v[:, i:j], out[:, i:j], q=q[:, i:j], heads=(i, j))
    main.wait_stream(alt)
    torch.cuda.synchronize(DEV)
    assert torch.equal(out, ref)


def test_head_range_is_validated():
    plan = tb.SagePlan(2, 4, 4, 256, 256, 128, torch.float16, DEV)
    q = torch.zeros(2, 4, 256, 128, dtype=torch.float16, device=DEV)
    with pytest.raises(ValueError):
        plan.attention(q[:, :2], q[:, :2].clone(), q=q[:, :2], heads=(0, 2))  # batch 2
    plan1 = tb.SagePlan(1, 4, 4, 256, 256, 128, torch.float16, DEV)
    with pytest.raises(ValueError):
        plan1.attention(q[:1], q[:1].clone(), q=q[:1], heads=(2, 5))
