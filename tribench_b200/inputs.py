"""Seeded synthetic inputs and cost estimates for the sage_attn path.

``make_inputs(case, device, seed, dtype)`` keeps the signature and case keys of the
reference's make_inputs (kernels/sage_attn/reference.py:4-13: batch_size, num_heads, seq_len,
head_dim; returns {"q","k","v","causal"}) and adds the distributions of the BASELINE
configurations. Every (batch, head) slab is drawn on the device from its own generator
seeded by (seed, b, h), so a rank that owns a shard of the (B x H) grid regenerates exactly
its slabs and a 1-GPU run sees the same data as an N-GPU run.

Distributions (``case["dist"]``):
  normal    q, k, v ~ N(0, 1)                                        (the reference's make_inputs)
  offset    q, v ~ N(0,1); k = N(0,1) + c_d, c_d ~ N(0, k_offset_std^2) drawn once per channel
  vchan     offset for q, k; v = N(0,1) * u_d, u_d ~ U(0.5, 4) per channel (FP8 P.V config)
  studentt  q = 0.5 * t(3); k = N(0,1) + c_d, c_d ~ N(0, k_offset_std^2); v ~ N(0,1)
"""
from __future__ import annotations

import math

import torch

# BASELINE configurations (+ the S=8K D=128 headline case the metric names).
CONFIGS = {
    "c1": dict(batch_size=1, num_heads=4, seq_len=512, head_dim=64, causal=False, dtype="fp16", pv="16bit",
               seed=0, dist="offset", k_offset_std=2.0),
    "c2": dict(batch_size=4, num_heads=32, seq_len=4096, head_dim=128, causal=False, dtype="fp16", pv="16bit",
               seed=1, dist="offset", k_offset_std=2.0),
    "h8k": dict(batch_size=2, num_heads=32, seq_len=8192, head_dim=128, causal=False, dtype="fp16", pv="16bit",
                seed=1, dist="offset", k_offset_std=2.0),
    "c3": dict(batch_size=2, num_heads=32, seq_len=16384, head_dim=128, causal=True, dtype="fp16", pv="16bit",
               seed=2, dist="offset", k_offset_std=2.0),
    "c4": dict(batch_size=8, num_heads=16, seq_len=8192, head_dim=64, causal=True, dtype="bf16", pv="fp8",
               seed=3, dist="vchan", k_offset_std=2.0),
    "c5": dict(batch_size=16, num_heads=64, seq_len=32768, head_dim=128, causal=True, dtype="fp16", pv="16bit",
               seed=4, dist="studentt", k_offset_std=3.0),
    # the sage_attn pack's own benchmark cases (kernels/sage_attn/meta.json:25-39), with q, k, v
    # ~ N(0, 1) as its make_inputs draws them (reference.py:4-13)
    "s4k_d64": dict(batch_size=8, num_heads=16, seq_len=4096, head_dim=64, causal=False, dtype="fp16", pv="16bit",
                    seed=7, dist="normal"),
    "s8k_d64": dict(batch_size=4, num_heads=16, seq_len=8192, head_dim=64, causal=False, dtype="fp16", pv="16bit",
                    seed=8, dist="normal"),
}

_TORCH_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


def torch_dtype(name_or_dtype):
    if isinstance(name_or_dtype, torch.dtype):
        return name_or_dtype
    return _TORCH_DTYPES[name_or_dtype]


def slab_seed(seed: int, b: int, h: int) -> int:
    """Seed of the (b, h) slab's generator (a fixed mix; any 63-bit value is fine)."""
    x = (int(seed) * 0x9E3779B97F4A7C15 + int(b) * 0xBF58476D1CE4E5B9 + int(h) * 0x94D049BB133111EB) & ((1 << 63) - 1)
    return x ^ (x >> 29)


def _slab(gen, S, D, device, dist, k_offset_std):
    def randn(*shape):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32)

    if dist == "normal":
        return randn(S, D), randn(S, D), randn(S, D)
    c = randn(1, D) * k_offset_std
    if dist == "studentt":
        z = randn(S, D)
        chi2 = randn(3, S, D).pow(2).sum(0)
        q = 0.5 * z / torch.sqrt(chi2 / 3.0)
    else:
        q = randn(S, D)
    k = randn(S, D) + c
    v = randn(S, D)
    if dist == "vchan":
        u = 0.5 + 3.5 * torch.rand(1, D, generator=gen, device=device, dtype=torch.float32)
        v = v * u
    elif dist not in ("offset", "studentt"):
        raise ValueError(f"unknown dist {dist!r}")
    return q, k, v


def make_inputs(case: dict, device, seed: int, dtype, heads: tuple[int, int] | None = None, **kwargs):
    """Inputs of one case. ``heads=(lo, hi)`` generates only flattened (b*H + h) slabs lo..hi-1,
    returned as a [1, hi-lo, S, D] batch (a rank's shard); default: the whole [B, H, S, D]."""
    B = case.get("batch_size", 8)
    H = case.get("num_heads", 16)
    S = case.get("seq_len", 4096)
    D = case.get("head_dim", 64)
    dist = case.get("dist", "normal")
    std = float(case.get("k_offset_std", 2.0))
    dt = torch_dtype(dtype)
    lo, hi = (0, B * H) if heads is None else heads
    q = torch.empty((hi - lo, S, D), dtype=dt, device=device)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    for i, flat in enumerate(range(lo, hi)):
        b, h = divmod(flat, H)
        gen = torch.Generator(device=device)
        gen.manual_seed(slab_seed(seed, b, h))
        qs, ks, vs = _slab(gen, S, D, device, dist, std)
        q[i].copy_(qs)
        k[i].copy_(ks)
        v[i].copy_(vs)
    shape = (B, H, S, D) if heads is None else (1, hi - lo, S, D)
    return {"q": q.view(shape), "k": k.view(shape), "v": v.view(shape), "causal": bool(case.get("causal", False))}


def estimate(case: dict) -> dict:
    """TriBench's estimate (reference.py:26-34: flops = 4*B*H*S^2*D, bytes = 4*B*H*S*D*2) plus the
    algorithmic op count that skips masked pairs when causal (2*D ops per visible (i, j) pair
    for QK^T and again for P.V)."""
    B = case.get("batch_size", 8)
    H = case.get("num_heads", 16)
    S = case.get("seq_len", 4096)
    D = case.get("head_dim", 64)
    flops = 4 * B * H * S * S * D
    pairs = S * (S + 1) // 2 if case.get("causal", False) else S * S
    return {"flops": flops, "bytes": 4 * B * H * S * D * 2, "ops_alg": 4 * B * H * pairs * D,
            "ops_qk": 2 * B * H * pairs * D, "ops_pv": 2 * B * H * pairs * D}


def prepass_bytes(case: dict, fused_q: bool = False) -> int:
    """Algorithmic HBM bytes of the pre-pass: read Q and K at 2 B/elt, write int8 Q/K, fp32
    scales and the fp32 K mean; with FP8 P.V also read V (2 B) and write e4m3 V (1 B) + scales.
    ``fused_q``: Q is quantised by the attention kernel, so the pre-pass moves K's bytes only."""
    B = case.get("batch_size", 8)
    H = case.get("num_heads", 16)
    S = case.get("seq_len", 4096)
    D = case.get("head_dim", 64)
    n = B * H * S * D
    if fused_q:
        b = 3 * n + 4 * (B * H * math.ceil(S / 64) + B * H * D)
    else:
        b = 2 * (3 * n) + 4 * (B * H * math.ceil(S / 128) + B * H * math.ceil(S / 64) + B * H * D)
    if case.get("pv") == "fp8":
        b += 3 * n + 4 * B * H * D
    return b
