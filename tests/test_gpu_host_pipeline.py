"""GPU: HostPipeline (host q/k/v -> host output, chunks of heads streamed through the device).

Every (batch, head) is computed by the same kernels as one sage_run over the whole tensor, so
the chunked, copy-overlapped pipeline must reproduce SagePlan.run bit for bit, including GQA
chunks, FP8 P.V, causal masking, ragged lengths and back-to-back calls that reuse the device
slots.
"""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _case(B, Hq, Hkv, S, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=g).to(dtype)
    k = (torch.randn(B, Hkv, S, D, generator=g) + 2.0 * torch.randn(1, 1, 1, D, generator=g)).to(dtype)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    return q, k, v


def _device_reference(q, k, v, pv, causal):
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    plan = tb.SagePlan(B, Hq, Hkv, S, S, D, q.dtype, DEV, pv=pv, causal=causal)
    out = plan.run(q.to(DEV), k.to(DEV), v.to(DEV))
    return out.cpu()


@pytest.mark.parametrize("B,Hq,Hkv,S,D,dtype,pv,causal,chunks", [
    (2, 4, 4, 1000, 128, torch.float16, "16bit", False, 3),
    (1, 8, 2, 777, 64, torch.bfloat16, "fp8", True, 5),
    (2, 6, 6, 512, 128, torch.bfloat16, "16bit", True, 1),
])
def test_pipeline_matches_device_run_bitwise(B, Hq, Hkv, S, D, dtype, pv, causal, chunks):
    q, k, v = _case(B, Hq, Hkv, S, D, dtype, seed=B * 100 + Hq)
    ref = _device_reference(q, k, v, pv, causal)
    pipe = tb.HostPipeline(B, Hq, Hkv, S, S, D, dtype, DEV, chunks=chunks, pv=pv, causal=causal)
    hq, hk, hv = (t.pin_memory() for t in (q, k, v))
    out = torch.empty(B, Hq, S, D, dtype=dtype).pin_memory()
    pipe.run(hq, hk, hv, out)
    torch.cuda.synchronize(DEV)
    assert torch.equal(out, ref)
    assert tb.device_status(DEV) == 0


def test_pipeline_back_to_back_calls_reuse_slots_safely():
    B, H, S, D = 2, 8, 640, 128
    pipe = tb.HostPipeline(B, H, H, S, S, D, torch.float16, DEV, chunks=4)
    results = []
    inputs = [_case(B, H, H, S, D, torch.float16, seed=s) for s in (1, 2, 3)]
    outs = [torch.empty(B, H, S, D, dtype=torch.float16).pin_memory() for _ in inputs]
    for (q, k, v), out in zip(inputs, outs):  # no synchronisation between the calls
        pipe.run(q.pin_memory(), k.pin_memory(), v.pin_memory(), out)
    torch.cuda.synchronize(DEV)
    for (q, k, v), out in zip(inputs, outs):
        results.append(torch.equal(out, _device_reference(q, k, v, "16bit", False)))
    assert results == [True, True, True]
