"""GPU: the flash_attn pack (sage_flash_attn_fwd: fp16/bf16 QK^T, no quantisation).

Compared with a plain PyTorch fp32 evaluation of the reference's ref
(kernels/flash_attn/reference.py:15-28: softmax(Q K^T * sm_scale [causal mask]) V) on the same
inputs. The kernel keeps the softmax in fp32 and rounds only P (to the input dtype) before P.V,
which accumulates in fp32, so its error is far inside the pack's tolerance (atol = rtol = 1e-2,
kernels/flash_attn/meta.json:45-48): max-abs <= 4e-3 for fp16 and 1.6e-2 for bf16 outputs below,
with the same bounds as the sage path's 16-bit P.V.
"""
import pytest
import torch

import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def ref_fp32(q, k, v, causal, sm_scale=None):
    """reference.py:15-28 in fp32 (GQA: kv head h // (Hq / Hkv))."""
    q, k, v = q.float(), k.float(), v.float()
    g = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    scale = q.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    s = torch.matmul(q, k.transpose(2, 3)) * scale
    if causal:
        Sq, Sk = s.shape[-2:]
        mask = torch.ones(Sq, Sk, dtype=torch.bool, device=s.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v)


def _inputs(B, Hq, Hkv, S, D, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=g, device=DEV).to(dtype)
    k = torch.randn(B, Hkv, S, D, generator=g, device=DEV).to(dtype)
    v = torch.randn(B, Hkv, S, D, generator=g, device=DEV).to(dtype)
    return q, k, v


def _tol(dtype):
    return 1.6e-2 if dtype == torch.bfloat16 else 4e-3


@pytest.mark.parametrize("B,Hq,Hkv,S,D,dtype,causal", [
    (2, 4, 4, 1000, 64, torch.float16, False),
    (2, 4, 4, 1000, 128, torch.float16, True),
    (1, 8, 2, 777, 128, torch.bfloat16, True),
    (1, 3, 3, 200, 64, torch.bfloat16, False),
    (1, 2, 2, 4096, 128, torch.float16, False),
    (1, 2, 1, 2048, 64, torch.float16, True),
])
def test_flash_matches_fp32_reference(B, Hq, Hkv, S, D, dtype, causal):
    q, k, v = _inputs(B, Hq, Hkv, S, D, dtype, seed=S + D)
    o = tb.run_flash_attn(q, k, v, causal=causal)
    assert tb.device_status(DEV) == 0
    assert o.shape == q.shape and o.dtype == q.dtype
    ref = ref_fp32(q, k, v, causal)
    err = (o.float() - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(o.float().flatten(), ref.flatten(), dim=0).item()
    print(f"flash B{B} H{Hq}/{Hkv} S{S} D{D} {dtype} causal={causal}: max-abs {err:.2e} cos {cos:.6f}")
    assert err <= _tol(dtype) and cos >= 0.9999


def test_flash_nhd_layout_sm_scale_and_out_buffer():
    B, H, S, D = 2, 3, 640, 64
    q, k, v = _inputs(B, H, H, S, D, torch.float16, seed=11)
    qn, kn, vn = (t.transpose(1, 2).contiguous() for t in (q, k, v))  # [B, S, H, D]
    out = torch.empty_like(qn)
    o = tb.run_flash_attn(qn, kn, vn, causal=False, sm_scale=0.05, tensor_layout="NHD", out=out)
    assert o.data_ptr() == out.data_ptr()
    ref = ref_fp32(q, k, v, False, sm_scale=0.05).transpose(1, 2)
    assert (o.float() - ref).abs().max().item() <= 4e-3


def test_flash_reference_case_sampled_heads():
    """The pack's s4k_d64 case (B=8, H=16, S=4096, D=64) at full size; sampled heads checked."""
    inp = tb.flash_attn.flash_inputs("fa_s4k_d64", DEV)
    q, k, v = inp["q"], inp["k"], inp["v"]
    o = tb.run_flash_attn(q, k, v)
    assert tb.device_status(DEV) == 0
    for b, h in [(0, 0), (3, 7), (7, 15)]:
        sl = (slice(b, b + 1), slice(h, h + 1))
        ref = ref_fp32(q[sl], k[sl], v[sl], False)
        assert (o[sl].float() - ref).abs().max().item() <= 4e-3


def test_flash_deterministic():
    q, k, v = _inputs(1, 4, 4, 1536, 128, torch.float16, seed=3)
    a = tb.run_flash_attn(q, k, v, causal=True)
    b = tb.run_flash_attn(q, k, v, causal=True)
    assert torch.equal(a, b)


@pytest.mark.parametrize("Sq,Skv,D,causal", [(1, 1, 64, False), (17, 17, 128, True), (300, 777, 64, False),
                                             (1000, 129, 128, False)])
def test_flash_tiny_and_cross_lengths(Sq, Skv, D, causal):
    g = torch.Generator(device=DEV).manual_seed(Sq * 7 + Skv)
    q = torch.randn(1, 2, Sq, D, generator=g, device=DEV).half()
    k = torch.randn(1, 2, Skv, D, generator=g, device=DEV).half()
    v = torch.randn(1, 2, Skv, D, generator=g, device=DEV).half()
    o = tb.run_flash_attn(q, k, v, causal=causal)
    assert tb.device_status(DEV) == 0
    assert (o.float() - ref_fp32(q, k, v, causal)).abs().max().item() <= 4e-3
