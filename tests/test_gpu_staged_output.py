"""GPU: the attention epilogue's staged, line-coalesced store path.

When the output is not memory of the launching GPU (a peer GPU's buffer mapped for the
multi-GPU gather), the epilogue writes each half tile through shared memory and stores whole
lines. On one GPU the same path is taken for an output in pinned host memory (mapped into the
device's address space and handed to the public API as a CUDA-tensor view of that memory), so
these tests run it against the direct-store path on the same inputs: the two must agree bit for
bit, for both head dims, both output types, causal and ragged lengths, HND and NHD output
strides, packed variable-length batches and the flash_attn pack.
"""
import pytest
import torch

import tribench_b200 as tb
from tribench_b200.flash_attn import run_flash_attn
from tribench_b200.shard import _CudaArray
from tribench_b200.varlen import run_sage_attn_varlen

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def host_out(shape, dtype):
    """A NaN-filled pinned host tensor and a CUDA-tensor view of the same memory."""
    host = torch.full(shape, float("nan"), dtype=dtype).pin_memory()
    with torch.cuda.device(DEV):
        view = torch.as_tensor(_CudaArray(host.data_ptr(), host.numel() * host.element_size()))
    return host, view.view(dtype).view(*shape)


def check(host, direct):
    torch.cuda.synchronize(DEV)
    assert tb.device_status(DEV) == 0
    assert torch.equal(host, direct.cpu())


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("D,dtype,causal,S", [
    (128, torch.float16, True, 1000),
    (128, torch.bfloat16, False, 777),
    (64, torch.float16, False, 1000),
    (64, torch.bfloat16, True, 333),
])
def test_staged_store_equals_direct_store(D, dtype, causal, S, layout):
    B, Hq, Hkv = 2, 4, 2
    g = torch.Generator(device=DEV).manual_seed(S + D)
    shp = lambda h: (B, h, S, D) if layout == "HND" else (B, S, h, D)  # noqa: E731
    q = torch.randn(shp(Hq), generator=g, device=DEV).to(dtype)
    k = (torch.randn(shp(Hkv), generator=g, device=DEV) + 1.5).to(dtype)
    v = torch.randn(shp(Hkv), generator=g, device=DEV).to(dtype)
    plan = tb.SagePlan(B, Hq, Hkv, S, S, D, dtype, DEV, causal=causal)
    direct = plan.run(q, k, v, tensor_layout=layout)
    host, view = host_out(shp(Hq), dtype)
    plan.run(q, k, v, view, tensor_layout=layout)
    check(host, direct)


@pytest.mark.parametrize("D", [64, 128])
def test_flash_staged_store_equals_direct_store(D):
    B, H, S = 1, 3, 901
    g = torch.Generator(device=DEV).manual_seed(D)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=DEV).half() for _ in range(3))
    direct = run_flash_attn(q, k, v, causal=True)
    host, view = host_out((B, H, S, D), torch.float16)
    run_flash_attn(q, k, v, causal=True, out=view)
    check(host, direct)


@pytest.mark.parametrize("D,causal", [(128, True), (64, False)])
def test_varlen_staged_store_equals_direct_store(D, causal):
    lens_q = [300, 0, 1, 517]
    lens_k = lens_q if causal else [290, 40, 128, 700]  # causal: equal lengths per sequence
    cu_q = torch.tensor([0] + torch.tensor(lens_q).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0] + torch.tensor(lens_k).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    Hq, Hkv = 4, 2
    g = torch.Generator(device=DEV).manual_seed(7 + D)
    q = torch.randn(sum(lens_q), Hq, D, generator=g, device=DEV).half()
    k = torch.randn(sum(lens_k), Hkv, D, generator=g, device=DEV).half()
    v = torch.randn(sum(lens_k), Hkv, D, generator=g, device=DEV).half()
    direct = run_sage_attn_varlen(q, k, v, cu_q, cu_k, causal=causal)
    host, view = host_out(tuple(q.shape), torch.float16)
    run_sage_attn_varlen(q, k, v, cu_q, cu_k, causal=causal, out=view)
    check(host, direct)
