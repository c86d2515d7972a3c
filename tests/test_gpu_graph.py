"""GPU: a CUDA graph of SagePlan.run replays the same kernels and gives the same bits."""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("pv,causal,dtype", [("16bit", False, torch.float16), ("fp8", True, torch.bfloat16)])
def test_graph_replay_matches_eager(pv, causal, dtype):
    B, H, S, D = 1, 4, 640, 64
    g = torch.Generator(device=DEV).manual_seed(7)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=DEV).to(dtype) for _ in range(3))
    plan = tb.SagePlan(B, H, H, S, S, D, dtype, DEV, pv=pv, causal=causal)
    ref = plan.run(q, k, v).clone()
    out = torch.empty_like(q)
    graph = plan.cuda_graph(q, k, v, out)
    graph.replay()
    torch.cuda.synchronize(DEV)
    assert torch.equal(out, ref)
    # new inputs in place: the replay recomputes everything from them
    q2, k2, v2 = (torch.randn(B, H, S, D, generator=g, device=DEV).to(dtype) for _ in range(3))
    q.copy_(q2), k.copy_(k2), v.copy_(v2)
    graph.replay()
    torch.cuda.synchronize(DEV)
    assert torch.equal(out, tb.SagePlan(B, H, H, S, S, D, dtype, DEV, pv=pv, causal=causal).run(q2, k2, v2))
    assert tb.device_status(DEV) == 0
