"""Python mirror of TriBench's flash_attn pack on sm_100a (kernels/flash_attn/).

``run_flash_attn(q, k, v, causal=False, sm_scale=None)`` has the signature and meaning of the
reference's ``run_flash_attn`` (kernels/flash_attn/triton_impl.py:110-128) and ``ref``
(kernels/flash_attn/reference.py:15-28): O = softmax(Q K^T * sm_scale) V over [B, H, S, D]
fp16/bf16 tensors, sm_scale defaulting to D**-0.5, key <= query when causal, output in q's
dtype. It is one call of the C ABI's ``sage_flash_attn_fwd``: the attention pipeline of the
sage path with fp16/bf16 QK^T on the tensor cores instead of INT8 (no quantisation). Unlike the
Triton kernel it also masks ragged sequence lengths and supports GQA (heads_q a multiple of
heads_kv) and the NHD layout.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .inputs import make_inputs
from .sage_attn import _DTYPES, _check_tensor, _dims, _stream_ptr, _vp

# The flash_attn pack's benchmark cases (kernels/flash_attn/meta.json:25-39), non-causal fp16,
# with q, k, v ~ N(0, 1) as reference.py:4-13 draws them (seeded per (batch, head) slab here).
FLASH_CONFIGS = {
    "fa_s4k_d64": dict(batch_size=8, num_heads=16, seq_len=4096, head_dim=64, causal=False, dtype="fp16",
                       seed=5, dist="normal"),
    "fa_s8k_d64": dict(batch_size=4, num_heads=16, seq_len=8192, head_dim=64, causal=False, dtype="fp16",
                       seed=6, dist="normal"),
}


def run_flash_attn(q, k, v, causal=False, sm_scale=None, *, tensor_layout="HND", out=None):
    """Drop-in for run_flash_attn (kernels/flash_attn/triton_impl.py:110-128) on sm_100a.

    q: [B, Hq, Sq, D], k/v: [B, Hkv, Skv, D] (HND; NHD with tensor_layout="NHD"), fp16 or bf16,
    D in {64, 128}. Returns o with q's shape and dtype (written into ``out`` when given).
    """
    _check_tensor("q", q)
    for name, t in (("k", k), ("v", v)):
        _check_tensor(name, t, q.dtype)
        if t.device != q.device:
            raise ValueError(f"{name} is on {t.device}, q on {q.device}")
    if q.dtype not in _DTYPES:
        raise TypeError(f"q/k/v must be float16 or bfloat16, got {q.dtype}")
    B, Hq, Sq, D, qs = _dims(q, tensor_layout)
    Bk, Hkv, Skv, Dk, ks = _dims(k, tensor_layout)
    Bv, Hv, Sv, Dv, vs = _dims(v, tensor_layout)
    if (Bk, Dk) != (B, D) or (Bv, Hv, Sv, Dv) != (Bk, Hkv, Skv, Dk):
        raise ValueError(f"shapes do not match: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}")
    if out is None:
        out = torch.empty_like(q) if q.is_contiguous() else torch.empty(q.shape, dtype=q.dtype, device=q.device)
    _check_tensor("out", out, q.dtype)
    if tuple(out.shape) != tuple(q.shape):
        raise ValueError(f"out shape {tuple(out.shape)} differs from q {tuple(q.shape)}")
    *_, os_ = _dims(out, tensor_layout)
    with torch.cuda.device(q.device):
        rc = N.load().sage_flash_attn_fwd(
            _vp(q), _vp(k), _vp(v), _vp(out), _DTYPES[q.dtype], B, Hq, Hkv, Sq, Skv, D, N.strides3(*qs),
            N.strides3(*ks), N.strides3(*vs), N.strides3(*os_), int(bool(causal)),
            ctypes.c_float(0.0 if sm_scale is None else float(sm_scale)), _stream_ptr(q.device))
    N.check("sage_flash_attn_fwd", rc)
    return out


run = run_flash_attn


def flash_inputs(name: str, device, dtype=None, heads=None):
    """Inputs of one flash_attn benchmark case (FLASH_CONFIGS), like reference.make_inputs."""
    case = dict(FLASH_CONFIGS[name])
    return make_inputs(case, device, seed=case["seed"], dtype=dtype or case["dtype"], heads=heads)
