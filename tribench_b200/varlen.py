"""Packed variable-length batches on the sm_100a path.

A batch of sequences with different lengths is packed along one token axis, as
flash-attention's ``*_varlen`` functions take it: q is [total_q, Hq, D], k/v are
[total_k, Hkv, D] (any head and token strides, head_dim contiguous) and ``cu_seqlens_q`` /
``cu_seqlens_k`` are int32 prefix sums of the lengths ([batch + 1], starting at 0). Each
sequence is quantised and attended exactly as a dense batch of one would be — Q blocks of 128
rows and K blocks of 64 rows start at the sequence's first token, the smoothing mean is per
(sequence, head) — so every output row equals the dense path's output for that sequence alone.

The reference has no packed entry point (its per_block_int8 / run_sage_attn take dense
[B, H, S, D] tensors, kernels/sage_attn/triton_impl.py:35-82, :162-200); these functions extend
the same operators, and run_flash_attn (kernels/flash_attn/triton_impl.py:110-128), to packed
batches through the C ABI's ``sage_per_block_int8_varlen``, ``sage_run_varlen`` and
``sage_flash_attn_varlen_fwd``. The cu arrays are validated on the host (one small copy).
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .sage_attn import _DTYPES, _PV, _check_tensor, _stream_ptr, _vp, workspace_bytes


def seq_lengths(cu, total: int, name: str) -> list[int]:
    """Lengths of the sequences a prefix-sum list describes; raises unless it starts at 0, never
    decreases and ends at ``total``."""
    cu = [int(x) for x in cu]
    if len(cu) < 2:
        raise ValueError(f"{name} needs batch + 1 >= 2 entries, got {len(cu)}")
    if cu[0] != 0:
        raise ValueError(f"{name} must start at 0, got {cu[0]}")
    lens = [b - a for a, b in zip(cu[:-1], cu[1:])]
    if min(lens) < 0:
        raise ValueError(f"{name} decreases at entry {lens.index(min(lens)) + 1}")
    if cu[-1] != total:
        raise ValueError(f"{name} ends at {cu[-1]}, but the packed tensor has {total} tokens")
    return lens


def check_causal_lengths(lens_q: list[int], lens_k: list[int]) -> None:
    """Causal packed attention needs every sequence's query and key lengths to agree (the
    reference's causal mask is square, reference.py:19-22)."""
    if lens_q != lens_k:
        i = next(i for i, (a, b) in enumerate(zip(lens_q, lens_k)) if a != b)
        raise ValueError(f"causal attention needs equal query and key lengths per sequence "
                         f"(sequence {i}: {lens_q[i]} vs {lens_k[i]})")


def _packed(name: str, t: torch.Tensor):
    """(tokens, H, D, (head, token) element strides) of a packed [tokens, H, D] tensor."""
    if t.dim() != 3:
        raise ValueError(f"{name} must be a packed [tokens, heads, head_dim] tensor, got shape {tuple(t.shape)}")
    if t.stride(2) != 1:
        raise ValueError(f"{name}: the head dimension must be contiguous (stride 1)")
    T, H, D = t.shape
    return T, H, D, (t.stride(1), t.stride(0))


def _cu_tensor(name: str, cu, batch: int, device) -> torch.Tensor:
    if isinstance(cu, torch.Tensor):
        if cu.dtype != torch.int32 or cu.dim() != 1 or cu.numel() != batch + 1:
            raise ValueError(f"{name} must be an int32 vector of batch + 1 = {batch + 1} entries")
        if cu.device != device:
            raise ValueError(f"{name} is on {cu.device}, q on {device}")
        return cu.contiguous()
    return torch.tensor([int(x) for x in cu], dtype=torch.int32, device=device)


def _host(cu) -> list[int]:
    return cu.tolist() if isinstance(cu, torch.Tensor) else [int(x) for x in cu]


class _Batch:
    """Validated shapes of one packed call."""

    def __init__(self, q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal):
        _check_tensor("q", q)
        _check_tensor("k", k, q.dtype)
        if q.dtype not in _DTYPES:
            raise TypeError(f"q/k/v must be float16 or bfloat16, got {q.dtype}")
        if k.device != q.device:
            raise ValueError(f"k is on {k.device}, q on {q.device}")
        self.Tq, self.Hq, self.D, self.qs = _packed("q", q)
        self.Tk, self.Hkv, Dk, self.ks = _packed("k", k)
        if Dk != self.D:
            raise ValueError(f"q and k disagree on head_dim ({self.D} vs {Dk})")
        self.lens_q = seq_lengths(_host(cu_seqlens_q), self.Tq, "cu_seqlens_q")
        self.lens_k = seq_lengths(_host(cu_seqlens_k), self.Tk, "cu_seqlens_k")
        if len(self.lens_q) != len(self.lens_k):
            raise ValueError(f"cu_seqlens_q and cu_seqlens_k describe {len(self.lens_q)} and "
                             f"{len(self.lens_k)} sequences")
        if causal:
            check_causal_lengths(self.lens_q, self.lens_k)
        self.B = len(self.lens_q)
        self.max_q = max(self.lens_q) if max_seqlen_q is None else int(max_seqlen_q)
        self.max_k = max(self.lens_k) if max_seqlen_k is None else int(max_seqlen_k)
        if self.max_q < max(self.lens_q) or self.max_k < max(self.lens_k):
            raise ValueError(f"max_seqlen_q / max_seqlen_k ({self.max_q}, {self.max_k}) are below the longest "
                             f"sequences ({max(self.lens_q)}, {max(self.lens_k)})")
        # no sequence is longer than its packed tensor: larger bounds would only size idle CTAs
        self.max_q, self.max_k = min(self.max_q, self.Tq), min(self.max_k, self.Tk)
        self.dev = q.device
        self.cu_q = _cu_tensor("cu_seqlens_q", cu_seqlens_q, self.B, self.dev)
        self.cu_k = _cu_tensor("cu_seqlens_k", cu_seqlens_k, self.B, self.dev)

    @property
    def empty(self) -> bool:
        return self.Tq == 0 or self.Tk == 0 or self.max_q == 0 or self.max_k == 0


def per_block_int8_varlen(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q=None, max_seqlen_k=None, sm_scale=None,
                          *, smooth_k=False, km=None, return_km=False, BLKQ=128):
    """per_block_int8 for packed sequences. Returns (q_int8 [Hq, total_q, D],
    q_scale [B, Hq, ceil(max_seqlen_q/BLKQ)], k_int8 [Hkv, total_k, D],
    k_scale [B, Hkv, ceil(max_seqlen_k/64)]) (+ k_mean [B, Hkv, D] with ``return_km``).
    Scale entries past a sequence's own block count are left unwritten. ``km`` ([B, Hkv, D]
    fp32) is the caller's per-sequence channel mean; ``smooth_k`` computes it on the device."""
    qflag = N.qblk_flag(BLKQ)
    bt = _Batch(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, False)
    if bt.empty:
        raise ValueError("per_block_int8_varlen needs at least one query and one key token")
    dev, D = bt.dev, bt.D
    q_i8 = torch.empty((bt.Hq, bt.Tq, D), dtype=torch.int8, device=dev)
    k_i8 = torch.empty((bt.Hkv, bt.Tk, D), dtype=torch.int8, device=dev)
    q_scale = torch.empty((bt.B, bt.Hq, (bt.max_q + BLKQ - 1) // BLKQ), dtype=torch.float32, device=dev)
    k_scale = torch.empty((bt.B, bt.Hkv, (bt.max_k + 63) // 64), dtype=torch.float32, device=dev)
    flags, k_mean = 0, None
    if km is not None:
        k_mean = torch.as_tensor(km, device=dev).to(torch.float32).reshape(bt.B, bt.Hkv, D).contiguous()
        flags = N.SAGE_FLAG_SMOOTH_K | N.SAGE_FLAG_KM_GIVEN
    elif smooth_k:
        k_mean = torch.empty((bt.B, bt.Hkv, D), dtype=torch.float32, device=dev)
        flags = N.SAGE_FLAG_SMOOTH_K
    ws_n = 0 if (flags & N.SAGE_FLAG_KM_GIVEN) else workspace_bytes(bt.B, bt.Hkv, bt.max_k, D, "16bit", bool(flags))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = N.load().sage_per_block_int8_varlen(
            _vp(q), _vp(k), _DTYPES[q.dtype], bt.B, bt.Hq, bt.Hkv, bt.Tq, bt.Tk, bt.max_q, bt.max_k, D,
            _vp(bt.cu_q), _vp(bt.cu_k), N.strides2(*bt.qs), N.strides2(*bt.ks),
            ctypes.c_float(0.0 if sm_scale is None else float(sm_scale)), flags | qflag,
            _vp(q_i8), _vp(q_scale), _vp(k_i8), _vp(k_scale), _vp(k_mean), _vp(ws), ws_n, _stream_ptr(dev))
    N.check("sage_per_block_int8_varlen", rc)
    if return_km:
        return q_i8, q_scale, k_i8, k_scale, k_mean
    return q_i8, q_scale, k_i8, k_scale


def _out_and_v(bt: _Batch, q, v, out):
    _check_tensor("v", v, q.dtype)
    Tv, Hv, Dv, vs = _packed("v", v)
    if (Tv, Hv, Dv) != (bt.Tk, bt.Hkv, bt.D):
        raise ValueError(f"v {tuple(v.shape)} does not match k ({bt.Tk}, {bt.Hkv}, {bt.D})")
    if out is None:
        out = torch.empty((bt.Tq, bt.Hq, bt.D), dtype=q.dtype, device=bt.dev)
    _check_tensor("out", out, q.dtype)
    To, Ho, Do, os_ = _packed("out", out)
    if (To, Ho, Do) != (bt.Tq, bt.Hq, bt.D):
        raise ValueError(f"out {tuple(out.shape)} does not match q {tuple(q.shape)}")
    return vs, out, os_


def run_sage_attn_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q=None, max_seqlen_k=None, causal=False,
                         sm_scale=None, *, pv="16bit", smooth_k=True, out=None, fused_q=None, blkq=128):
    """run_sage_attn for packed sequences: q [total_q, Hq, D], k/v [total_k, Hkv, D] -> o like q.
    A sequence with query rows but no keys gets o = 0. ``fused_q`` picks the operand route as
    SagePlan does (None: Q quantised in the attention kernel at head_dim 128, fp16 codes at 64;
    True: Q in the kernel; False: INT8 operands from the pre-pass). ``blkq``: query rows per Q
    scale (128, 64, 32, 16 or 1), counted from each sequence's first token."""
    qflag = N.qblk_flag(blkq)
    bt = _Batch(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal)
    vs, out, os_ = _out_and_v(bt, q, v, out)
    if bt.Tq == 0:
        return out
    if bt.empty:
        return out.zero_()
    dev, D = bt.dev, bt.D
    pv_mode = _PV[pv]
    fp8 = pv_mode == N.SAGE_PV_FP8
    route = ("fused" if D == 128 else "codes16") if fused_q is None else ("fused" if fused_q else "int8")
    route_flag = {"fused": N.SAGE_FLAG_FUSED_Q, "int8": N.SAGE_FLAG_PREPASS_Q, "codes16": 0}[route]
    q_i8 = torch.empty((bt.Hq, bt.Tq, D), dtype=torch.int8, device=dev) if route == "int8" else None
    k_i8 = torch.empty((bt.Hkv, bt.Tk, D), dtype=torch.int8, device=dev) if route != "codes16" else None
    q_scale = None if route == "fused" else torch.empty((bt.B, bt.Hq, (bt.max_q + blkq - 1) // blkq),
                                                        dtype=torch.float32, device=dev)
    k_scale = torch.empty((bt.B, bt.Hkv, (bt.max_k + 63) // 64), dtype=torch.float32, device=dev)
    k_mean = torch.empty((bt.B, bt.Hkv, D), dtype=torch.float32, device=dev) if smooth_k else None
    v_fp8 = torch.empty((bt.Hkv, bt.Tk, D), dtype=torch.uint8, device=dev) if fp8 else None
    v_scale = torch.empty((bt.B, bt.Hkv, D), dtype=torch.float32, device=dev) if fp8 else None
    flags = (N.SAGE_FLAG_SMOOTH_K if smooth_k else 0) | route_flag | qflag
    ws_n = int(N.load().sage_workspace_bytes(bt.B, bt.Hkv, bt.max_k, D, pv_mode, flags))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = N.load().sage_run_varlen(
            _vp(q), _vp(k), _vp(v), _vp(out), _DTYPES[q.dtype], bt.B, bt.Hq, bt.Hkv, bt.Tq, bt.Tk, bt.max_q,
            bt.max_k, D, _vp(bt.cu_q), _vp(bt.cu_k), N.strides2(*bt.qs), N.strides2(*bt.ks), N.strides2(*vs),
            N.strides2(*os_), int(bool(causal)), ctypes.c_float(0.0 if sm_scale is None else float(sm_scale)),
            pv_mode, flags, _vp(q_i8), _vp(q_scale), _vp(k_i8), _vp(k_scale), _vp(k_mean), _vp(v_fp8),
            _vp(v_scale), _vp(ws), ws_n, _stream_ptr(dev))
    N.check("sage_run_varlen", rc)
    return out


def run_flash_attn_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q=None, max_seqlen_k=None, causal=False,
                          sm_scale=None, *, out=None):
    """run_flash_attn for packed sequences (fp16/bf16 QK^T, no quantisation)."""
    bt = _Batch(q, k, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal)
    vs, out, os_ = _out_and_v(bt, q, v, out)
    if bt.Tq == 0:
        return out
    if bt.empty:
        return out.zero_()
    with torch.cuda.device(bt.dev):
        rc = N.load().sage_flash_attn_varlen_fwd(
            _vp(q), _vp(k), _vp(v), _vp(out), _DTYPES[q.dtype], bt.B, bt.Hq, bt.Hkv, bt.Tq, bt.Tk, bt.max_q,
            bt.max_k, bt.D, _vp(bt.cu_q), _vp(bt.cu_k), N.strides2(*bt.qs), N.strides2(*bt.ks), N.strides2(*vs),
            N.strides2(*os_), int(bool(causal)), ctypes.c_float(0.0 if sm_scale is None else float(sm_scale)),
            _stream_ptr(bt.dev))
    N.check("sage_flash_attn_varlen_fwd", rc)
    return out
