"""GPU: the attention epilogue's staged, line-coalesced store path.

When the output is not memory of the launching GPU (a peer GPU's buffer mapped for the
multi-GPU gather), the epilogue writes each half tile through shared memory and stores whole
lines. On one GPU the same path is taken for an output in pinned host memory (mapped into the
device's address space), so these tests run it against the direct-store path on the same
inputs: the two must agree bit for bit, for both head dims, both output types, causal and
ragged lengths, HND and NHD output strides, and the flash_attn pack.
"""
import pytest
import torch

import tribench_b200 as tb
from tribench_b200 import _native as N
from tribench_b200.flash_attn import run_flash_attn
from tribench_b200.sage_attn import _DTYPES, _dims, _stream_ptr, _vp

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def sage_run_into(plan, q, k, v, out, layout):
    """plan.run with `out` passed straight to the C ABI (it may live in pinned host memory)."""
    B, Hq, Hkv, Sq, Skv, D = plan.shape
    strides = [_dims(t, layout)[4] for t in (q, k, v, out)]
    qd = plan.quant
    rc = N.load().sage_run(
        _vp(q), _vp(k), _vp(v), _vp(out), _DTYPES[plan.dtype], B, Hq, Hkv, Sq, Skv, D,
        *(N.strides3(*s) for s in strides), int(plan.causal), plan._sm_scale(), plan.pv_mode,
        plan.flags | plan.route_flag, _vp(qd.q_int8), _vp(qd.q_scale), _vp(qd.k_int8), _vp(qd.k_scale),
        _vp(qd.k_mean), _vp(qd.v_fp8), _vp(qd.v_scale), _vp(plan.ws), plan.ws_bytes, _stream_ptr(DEV))
    N.check("sage_run", rc)


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
    host = torch.full(shp(Hq), float("nan"), dtype=dtype).pin_memory()
    sage_run_into(plan, q, k, v, host, layout)
    torch.cuda.synchronize(DEV)
    assert tb.device_status(DEV) == 0
    assert torch.equal(host, direct.cpu())


@pytest.mark.parametrize("D", [64, 128])
def test_flash_staged_store_equals_direct_store(D):
    B, H, S = 1, 3, 901
    g = torch.Generator(device=DEV).manual_seed(D)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device=DEV).half() for _ in range(3))
    direct = run_flash_attn(q, k, v, causal=True)
    host = torch.full((B, H, S, D), float("nan"), dtype=torch.float16).pin_memory()
    rc = N.load().sage_flash_attn_fwd(
        _vp(q), _vp(k), _vp(v), _vp(host), _DTYPES[torch.float16], B, H, H, S, S, D,
        *(N.strides3(*_dims(t, "HND")[4]) for t in (q, k, v, host)), 1, 0.0, _stream_ptr(DEV))
    N.check("sage_flash_attn_fwd", rc)
    torch.cuda.synchronize(DEV)
    assert tb.device_status(DEV) == 0
    assert torch.equal(host, direct.cpu())
