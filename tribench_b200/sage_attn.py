"""Host side of the B200 sage_attn path: the reference's operator interface over the C ABI.

Mirrors kernels/sage_attn/triton_impl.py:
  * ``per_block_int8(q, k, km=None, BLKQ=128, BLKK=64, sm_scale=None, tensor_layout="HND")``
    — same arguments, same return tuple (q_int8, q_scale, k_int8, k_scale), :35-82;
  * ``run_sage_attn(q, k, v, causal=False, sm_scale=None)`` — :162-200, exported as ``run``
    too (the TriBench ``cuda`` variant entry point).
Differences from the reference are deliberate and documented: ``causal`` is honoured (the
Triton kernel ignores it), K is smoothed by default (``smooth_k=True``), P.V can run in FP8
(``pv="fp8"``), bf16 inputs keep P and V in bf16 instead of casting V to fp16, and the
attention path accepts Q scale blocks finer than 128 rows (``blkq``: per_block_int8's BLKQ,
which the reference's own attention kernel does not support, triton_impl.py:136, 148).

torch is used only for device memory, the current stream and dtype/shape bookkeeping; all
arithmetic runs in libsage_sm100.so. There is no CPU or Triton fallback.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as N

_DTYPES = {torch.float16: N.SAGE_DTYPE_F16, torch.bfloat16: N.SAGE_DTYPE_BF16}
_PV = {"16bit": N.SAGE_PV_16BIT, "fp16": N.SAGE_PV_16BIT, "fp8": N.SAGE_PV_FP8}


def _dims(t: torch.Tensor, layout: str):
    """(B, H, S, D, (batch, head, seq) element strides) of a 4-D tensor in HND or NHD layout."""
    if t.dim() != 4:
        raise ValueError(f"expected a 4-D tensor, got shape {tuple(t.shape)}")
    if t.stride(3) != 1:
        raise ValueError("the head dimension must be contiguous (stride 1)")
    if layout == "HND":
        B, H, S, D = t.shape
        return B, H, S, D, (t.stride(0), t.stride(1), t.stride(2))
    if layout == "NHD":
        B, S, H, D = t.shape
        return B, H, S, D, (t.stride(0), t.stride(2), t.stride(1))
    raise ValueError(f"tensor_layout must be 'HND' or 'NHD', got {layout!r}")


def _check_tensor(name: str, t: torch.Tensor, dtype=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (the sage_attn path has no CPU implementation)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} has dtype {t.dtype}, expected {dtype}")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _vp(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def workspace_bytes(batch, heads_kv, seq_kv, head_dim, pv: str = "16bit", smooth_k: bool = True) -> int:
    flags = N.SAGE_FLAG_SMOOTH_K if smooth_k else 0
    return int(N.load().sage_workspace_bytes(batch, heads_kv, seq_kv, head_dim, _PV[pv], flags))


@dataclass
class SageQuant:
    """Quantised operands of one call (all contiguous, [B, H, S, D]-ordered)."""
    q_int8: torch.Tensor
    q_scale: torch.Tensor
    k_int8: torch.Tensor
    k_scale: torch.Tensor
    k_mean: torch.Tensor | None = None
    v_fp8: torch.Tensor | None = None
    v_scale: torch.Tensor | None = None
    blkq: int = 128  # query rows per q_scale entry


def per_block_int8(q, k, km=None, BLKQ=128, BLKK=64, sm_scale=None, tensor_layout="HND", *, smooth_k=False,
                   return_km=False):
    """INT8 per-block quantisation of Q (BLKQ-row blocks) and K (64-row blocks).

    Same contract as the reference per_block_int8 (triton_impl.py:35-82): returns
    (q_int8 [B,Hq,Sq,D], q_scale [B,Hq,ceil(Sq/BLKQ)], k_int8 [B,Hkv,Skv,D], k_scale [B,Hkv,ceil(Skv/64)]);
    BLKQ is 128 (default), 64, 32, 16 or 1 (one scale per token), bit-identical to the
    reference at each; BLKK must be 64 (the attention kernel's K scale granularity).
    ``km`` (broadcastable to [B, Hkv, 1, D]) is subtracted from K in fp32 first. ``smooth_k=True``
    computes km on the device (the K channel mean); ``return_km`` appends it to the tuple.
    """
    if BLKK != 64:
        raise ValueError("the sm_100a kernels use BLKK=64 (triton_impl.py:167)")
    qflag = N.qblk_flag(BLKQ)
    _check_tensor("q", q)
    _check_tensor("k", k, q.dtype)
    if q.dtype not in _DTYPES:
        raise TypeError(f"q/k must be float16 or bfloat16, got {q.dtype}")
    if q.device != k.device:
        raise ValueError("q and k must be on the same device")
    B, Hq, Sq, D, qs = _dims(q, tensor_layout)
    Bk, Hkv, Skv, Dk, ks = _dims(k, tensor_layout)
    if Bk != B or Dk != D:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree on batch or head_dim")
    dev = q.device
    q_i8 = torch.empty((B, Hq, Sq, D), dtype=torch.int8, device=dev)
    k_i8 = torch.empty((B, Hkv, Skv, D), dtype=torch.int8, device=dev)
    q_scale = torch.empty((B, Hq, (Sq + BLKQ - 1) // BLKQ), dtype=torch.float32, device=dev)
    k_scale = torch.empty((B, Hkv, (Skv + 63) // 64), dtype=torch.float32, device=dev)
    flags = 0
    k_mean = None
    if km is not None:
        # The reference subtracts km from k by broadcasting (triton_impl.py:39-40): km is
        # broadcastable to [B, Hkv, 1, D] (HND) or [B, 1, Hkv, D] (NHD).
        kmt = torch.as_tensor(km, device=dev).to(torch.float32)
        if tensor_layout == "HND":
            k_mean = torch.broadcast_to(kmt, (B, Hkv, 1, D))[:, :, 0, :].contiguous()
        else:
            k_mean = torch.broadcast_to(kmt, (B, 1, Hkv, D))[:, 0, :, :].contiguous()
        flags = N.SAGE_FLAG_SMOOTH_K | N.SAGE_FLAG_KM_GIVEN
    elif smooth_k:
        k_mean = torch.empty((B, Hkv, D), dtype=torch.float32, device=dev)
        flags = N.SAGE_FLAG_SMOOTH_K
    ws_n = 0 if (flags & N.SAGE_FLAG_KM_GIVEN) else workspace_bytes(B, Hkv, Skv, D, "16bit", bool(flags))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    lib = N.load()
    with torch.cuda.device(dev):
        rc = lib.sage_per_block_int8(
            _vp(q), _vp(k), _DTYPES[q.dtype], B, Hq, Hkv, Sq, Skv, D, N.strides3(*qs), N.strides3(*ks),
            ctypes.c_float(0.0 if sm_scale is None else float(sm_scale)), flags | qflag,
            _vp(q_i8), _vp(q_scale), _vp(k_i8), _vp(k_scale), _vp(k_mean), _vp(ws), ws_n, _stream_ptr(dev))
    N.check("sage_per_block_int8", rc)
    if return_km:
        return q_i8, q_scale, k_i8, k_scale, k_mean
    return q_i8, q_scale, k_i8, k_scale


def quant_v_fp8(v, tensor_layout="HND"):
    """V -> (e4m3 codes as uint8 [B, Hkv, Skv, D], fp32 per-channel scales [B, Hkv, D])."""
    _check_tensor("v", v)
    if v.dtype not in _DTYPES:
        raise TypeError(f"v must be float16 or bfloat16, got {v.dtype}")
    B, H, S, D, vs = _dims(v, tensor_layout)
    dev = v.device
    v8 = torch.empty((B, H, S, D), dtype=torch.uint8, device=dev)
    vsc = torch.empty((B, H, D), dtype=torch.float32, device=dev)
    ws_n = workspace_bytes(B, H, S, D, "fp8", False)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = N.load().sage_quant_v_fp8(_vp(v), _DTYPES[v.dtype], B, H, S, D, N.strides3(*vs), _vp(v8), _vp(vsc),
                                       _vp(ws), ws_n, _stream_ptr(dev))
    N.check("sage_quant_v_fp8", rc)
    return v8, vsc


def attn_fwd(quant: SageQuant, v, causal=False, *, pv="16bit", out_dtype=None, tensor_layout="HND", out=None):
    """Attention over already-quantised operands (the _attn_fwd launch, triton_impl.py:121-160)."""
    q_i8, k_i8 = quant.q_int8, quant.k_int8
    B, Hq, Sq, D = q_i8.shape
    _, Hkv, Skv, _ = k_i8.shape
    dev = q_i8.device
    pv_mode = _PV[pv]
    if pv_mode == N.SAGE_PV_FP8:
        vv, vs = quant.v_fp8, (Skv * D * Hkv, Skv * D, D)
        if vv is None or quant.v_scale is None:
            raise ValueError("pv='fp8' needs quant.v_fp8 and quant.v_scale")
        if out_dtype is None:
            raise ValueError("pv='fp8' needs out_dtype")
        dt = out_dtype
    else:
        _check_tensor("v", v)
        _, _, _, _, vs = _dims(v, tensor_layout)
        vv, dt = v, v.dtype
    if out is None:
        out = torch.empty((B, Hq, Sq, D) if tensor_layout == "HND" else (B, Sq, Hq, D), dtype=dt, device=dev)
    _, _, _, _, os_ = _dims(out, tensor_layout)
    with torch.cuda.device(dev):
        rc = N.load().sage_attn_fwd(
            _vp(q_i8), _vp(quant.q_scale), _vp(k_i8), _vp(quant.k_scale), _vp(vv), N.strides3(*vs),
            _vp(quant.v_scale), _vp(out), N.strides3(*os_), _DTYPES[dt], pv_mode, int(bool(causal)),
            N.qblk_flag(quant.blkq), B, Hq, Hkv, Sq, Skv, D, _stream_ptr(dev))
    N.check("sage_attn_fwd", rc)
    return out


class SagePlan:
    """Preallocated intermediates for repeated calls on one shape (no per-call allocation).

    ``plan.run(q, k, v, o)`` is one ``sage_run`` C call: pre-pass kernels + attention kernel.
    ``fused_q`` picks how the attention kernel gets its operands (``self.route``):
      * None (sage_run's choice): at head_dim 128 "fused" — Q quantised inside the attention
        kernel, the pre-pass handles K and V; at 64 "codes16" — the pre-pass stores the codes
        as fp16 values and QK^T runs as a kind::f16 MMA on them (same scores, no int32 -> float
        step; the Q codes live in the output buffer until the kernel overwrites them);
      * True: "fused" at either head_dim (no INT8 Q buffer unless ``keep_q_int8``);
      * False: "int8" — INT8 operands from the pre-pass (sage_prepass + sage_attn_fwd).
    "fused" and "int8" give bit-identical output; "codes16" matches them to float rounding.
    ``blkq``: query rows per Q scale (128, 64, 32, 16 or 1), on every route.
    """

    def __init__(self, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim, dtype, device, *, pv="16bit",
                 smooth_k=True, causal=False, sm_scale=None, fused_q=None, keep_q_int8=False, blkq=128):
        if dtype not in _DTYPES:
            raise TypeError(f"dtype must be float16 or bfloat16, got {dtype}")
        self.shape = (batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)
        self.dtype, self.device = dtype, torch.device(device)
        self.pv_mode = _PV[pv]
        self.blkq = int(blkq)
        self.qflag = N.qblk_flag(self.blkq)
        self.flags = (N.SAGE_FLAG_SMOOTH_K if smooth_k else 0) | self.qflag
        if fused_q is None:
            self.route = "fused" if head_dim == 128 else "codes16"
        else:
            self.route = "fused" if fused_q else "int8"
        self.fused_q = self.route == "fused"
        self.route_flag = {"fused": N.SAGE_FLAG_FUSED_Q, "int8": N.SAGE_FLAG_PREPASS_Q, "codes16": 0}[self.route]
        self.causal, self.sm_scale = bool(causal), sm_scale
        B, Hq, Hkv, Sq, Skv, D = self.shape
        dev = self.device
        want_q = self.route == "int8" or (self.fused_q and keep_q_int8)
        want_k = self.route != "codes16"
        self.quant = SageQuant(
            q_int8=torch.empty((B, Hq, Sq, D), dtype=torch.int8, device=dev) if want_q else None,
            q_scale=torch.empty((B, Hq, (Sq + self.blkq - 1) // self.blkq), dtype=torch.float32, device=dev)
            if (want_q or self.route == "codes16") else None,
            k_int8=torch.empty((B, Hkv, Skv, D), dtype=torch.int8, device=dev) if want_k else None,
            k_scale=torch.empty((B, Hkv, (Skv + 63) // 64), dtype=torch.float32, device=dev),
            k_mean=torch.empty((B, Hkv, D), dtype=torch.float32, device=dev) if smooth_k else None,
            v_fp8=torch.empty((B, Hkv, Skv, D), dtype=torch.uint8, device=dev) if self.pv_mode else None,
            v_scale=torch.empty((B, Hkv, D), dtype=torch.float32, device=dev) if self.pv_mode else None,
            blkq=self.blkq,
        )
        self.codes16 = None  # (q, k) fp16 code buffers of the split form, allocated by prepass()
        self.ws_bytes = int(N.load().sage_workspace_bytes(B, Hkv, Skv, D, self.pv_mode, self.flags | self.route_flag))
        self.ws = torch.empty(max(self.ws_bytes, 1), dtype=torch.uint8, device=dev)

    def _sm_scale(self):
        return ctypes.c_float(0.0 if self.sm_scale is None else float(self.sm_scale))

    def prepass(self, q, k, v, tensor_layout="HND"):
        """The pre-pass half of run() (sage_prepass) into the plan's buffers: INT8 codes, or (route
        "codes16") the codes as fp16 values in self.codes16, or (route "fused") K alone."""
        B, Hq, Hkv, Sq, Skv, D = self.shape
        *_, qs = _dims(q, tensor_layout)
        *_, ks = _dims(k, tensor_layout)
        *_, vs = _dims(v, tensor_layout)
        qd = self.quant
        flags = self.flags
        qi, ki = qd.q_int8, qd.k_int8
        if self.route == "fused":
            flags |= N.SAGE_FLAG_FUSED_Q
            qi = None
        elif self.route == "codes16":
            if self.codes16 is None:
                self.codes16 = (torch.empty((B, Hq, Sq, D), dtype=torch.float16, device=self.device),
                                torch.empty((B, Hkv, Skv, D), dtype=torch.float16, device=self.device))
            flags |= N.SAGE_FLAG_CODES16
            qi, ki = self.codes16
        rc = N.load().sage_prepass(
            _vp(q), _vp(k), _vp(v), _DTYPES[self.dtype], B, Hq, Hkv, Sq, Skv, D, N.strides3(*qs), N.strides3(*ks),
            N.strides3(*vs), self._sm_scale(), self.pv_mode, flags, _vp(qi), _vp(qd.q_scale if qi is not None else None),
            _vp(ki), _vp(qd.k_scale), _vp(qd.k_mean), _vp(qd.v_fp8), _vp(qd.v_scale), _vp(self.ws), self.ws_bytes,
            _stream_ptr(self.device))
        N.check("sage_prepass", rc)
        return self.quant

    def attention(self, v, out, tensor_layout="HND", q=None, heads=None):
        """The attention half of run() over the prepass() results: sage_attn_fwd (route "int8"),
        sage_attn_fwd_codes16 ("codes16") or sage_attn_fwd_fused_q ("fused", which needs ``q``).

        ``heads=(i, j)`` (plans with batch 1) runs it for kv heads [i, j) only — query heads
        [i*g, j*g) with g = heads_q / heads_kv — so that one prepass() over all heads can feed
        several attention launches; ``v``, ``out`` and ``q`` are then that head range's tensors."""
        B, Hq, Hkv, Sq, Skv, D = self.shape
        qd = self.quant
        codes16 = self.codes16
        if heads is not None:
            i, j = heads
            if B != 1 or not (0 <= i < j <= Hkv):
                raise ValueError(f"heads={heads}: needs a batch-1 plan and 0 <= i < j <= {Hkv}")
            g = Hq // Hkv
            qa, qb = i * g, j * g
            cut = lambda t, a, b: None if t is None else t[:, a:b]  # noqa: E731
            qd = SageQuant(cut(qd.q_int8, qa, qb), cut(qd.q_scale, qa, qb), cut(qd.k_int8, i, j),
                           cut(qd.k_scale, i, j), None, cut(qd.v_fp8, i, j), cut(qd.v_scale, i, j), qd.blkq)
            if codes16 is not None:
                codes16 = (codes16[0][:, qa:qb], codes16[1][:, i:j])
            Hq, Hkv = qb - qa, j - i
        pv = "fp8" if self.pv_mode == N.SAGE_PV_FP8 else "16bit"
        if self.route == "int8":
            return attn_fwd(qd, v, self.causal, pv=pv, out_dtype=self.dtype, tensor_layout=tensor_layout, out=out)
        *_, os_ = _dims(out, tensor_layout)
        if self.pv_mode == N.SAGE_PV_FP8:
            vv, vs = qd.v_fp8, (Skv * D * Hkv, Skv * D, D)
        else:
            vv = v
            *_, vs = _dims(v, tensor_layout)
        lib = N.load()
        if self.route == "codes16":
            if codes16 is None:
                raise ValueError("call prepass() first")
            rc = lib.sage_attn_fwd_codes16(
                _vp(codes16[0]), _vp(qd.q_scale), _vp(codes16[1]), _vp(qd.k_scale), _vp(vv),
                N.strides3(*vs), _vp(qd.v_scale), _vp(out), N.strides3(*os_), _DTYPES[self.dtype], self.pv_mode,
                int(self.causal), self.qflag, B, Hq, Hkv, Sq, Skv, D, _stream_ptr(self.device))
            N.check("sage_attn_fwd_codes16", rc)
            return out
        if q is None:
            raise ValueError("this plan quantises Q inside the attention kernel: pass q")
        *_, qs = _dims(q, tensor_layout)
        rc = lib.sage_attn_fwd_fused_q(
            _vp(q), N.strides3(*qs), self._sm_scale(), _vp(qd.k_int8), _vp(qd.k_scale), _vp(vv), N.strides3(*vs),
            _vp(qd.v_scale), _vp(out), N.strides3(*os_), _DTYPES[self.dtype], self.pv_mode, int(self.causal),
            self.qflag, B, Hq, Hkv, Sq, Skv, D, _vp(qd.q_int8), _vp(qd.q_scale), _stream_ptr(self.device))
        N.check("sage_attn_fwd_fused_q", rc)
        return out

    def cuda_graph(self, q, k, v, out, tensor_layout="HND") -> "SageGraph":
        """Capture run(q, k, v, out) into a CUDA graph (see SageGraph)."""
        return SageGraph(self, q, k, v, out, tensor_layout=tensor_layout)

    def run(self, q, k, v, out=None, tensor_layout="HND"):
        B, Hq, Hkv, Sq, Skv, D = self.shape
        for name, t, h, s in (("q", q, Hq, Sq), ("k", k, Hkv, Skv), ("v", v, Hkv, Skv)):
            _check_tensor(name, t, self.dtype)
            tb, th, ts, td, _ = _dims(t, tensor_layout)
            if (tb, th, ts, td) != (B, h, s, D):
                raise ValueError(f"{name} shape {tuple(t.shape)} does not match the plan {self.shape}")
        if out is None:
            out = torch.empty((B, Hq, Sq, D) if tensor_layout == "HND" else (B, Sq, Hq, D), dtype=self.dtype,
                              device=self.device)
        _check_tensor("out", out, self.dtype)
        *_, qs = _dims(q, tensor_layout)
        *_, ks = _dims(k, tensor_layout)
        *_, vs = _dims(v, tensor_layout)
        *_, os_ = _dims(out, tensor_layout)
        qd = self.quant
        rc = N.load().sage_run(
            _vp(q), _vp(k), _vp(v), _vp(out), _DTYPES[self.dtype], B, Hq, Hkv, Sq, Skv, D,
            N.strides3(*qs), N.strides3(*ks), N.strides3(*vs), N.strides3(*os_), int(self.causal), self._sm_scale(),
            self.pv_mode, self.flags | self.route_flag, _vp(qd.q_int8), _vp(qd.q_scale), _vp(qd.k_int8),
            _vp(qd.k_scale), _vp(qd.k_mean), _vp(qd.v_fp8), _vp(qd.v_scale), _vp(self.ws), self.ws_bytes,
            _stream_ptr(self.device))
        N.check("sage_run", rc)
        return out


class SageGraph:
    """A CUDA graph of one SagePlan.run on fixed buffers: ``replay()`` reruns all its launches
    (pre-pass and attention) with a single graph launch. Refill ``q``/``k``/``v`` in place
    between replays; the result is in ``out``."""

    def __init__(self, plan: "SagePlan", q, k, v, out, tensor_layout="HND"):
        self.plan, self.q, self.k, self.v, self.out = plan, q, k, v, out
        dev = plan.device
        with torch.cuda.device(dev):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                plan.run(q, k, v, out, tensor_layout=tensor_layout)  # first run: function attributes, lazy init
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                plan.run(q, k, v, out, tensor_layout=tensor_layout)

    def replay(self):
        self.graph.replay()
        return self.out


class HostPipeline:
    """Attention over q/k/v held in host memory, streamed through one GPU in chunks of heads.

    ``pipe.run(q, k, v, out)`` takes contiguous HND host tensors (pinned, for the copies to
    be asynchronous) and fills ``out`` on the host. The flattened (batch x kv-head) axis is cut
    into ``chunks`` pieces; each piece goes host -> device on a copy stream, through sage_run
    (a SagePlan per chunk size) on the caller's current stream, and device -> host on a second
    copy stream, alternating between two device slots, so the PCIe transfers of one chunk
    overlap the computation of the next. Every (batch, head) is computed exactly as in one
    sage_run over the whole tensor, so the output is bit-identical to SagePlan.run. When run()
    returns, the caller's stream is ordered after the last device -> host copy.
    """

    def __init__(self, batch, heads_q, heads_kv, seq_q, seq_kv, head_dim, dtype, device, *, chunks=16,
                 pv="16bit", smooth_k=True, causal=False, sm_scale=None, blkq=128):
        if heads_kv <= 0 or heads_q % heads_kv:
            raise ValueError(f"heads_q ({heads_q}) must be a multiple of heads_kv ({heads_kv})")
        self.shape = (batch, heads_q, heads_kv, seq_q, seq_kv, head_dim)
        self.dtype, self.device = dtype, torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("HostPipeline streams through a CUDA device")
        self.groups = heads_q // heads_kv
        n = batch * heads_kv
        nc = max(1, min(int(chunks), n))
        self.ranges = [(i * n // nc, (i + 1) * n // nc) for i in range(nc)]
        self.plans = {}
        for a, b in self.ranges:
            m = b - a
            if m not in self.plans:
                self.plans[m] = SagePlan(1, m * self.groups, m, seq_q, seq_kv, head_dim, dtype, self.device, pv=pv,
                                         smooth_k=smooth_k, causal=causal, sm_scale=sm_scale, blkq=blkq)
        mmax = max(b - a for a, b in self.ranges)
        g = self.groups
        self.slots = [dict(q=torch.empty((1, mmax * g, seq_q, head_dim), dtype=dtype, device=self.device),
                           k=torch.empty((1, mmax, seq_kv, head_dim), dtype=dtype, device=self.device),
                           v=torch.empty((1, mmax, seq_kv, head_dim), dtype=dtype, device=self.device),
                           o=torch.empty((1, mmax * g, seq_q, head_dim), dtype=dtype, device=self.device))
                      for _ in range(2)]
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)

    def run(self, q, k, v, out):
        B, Hq, Hkv, Sq, Skv, D = self.shape
        for name, t, shp in (("q", q, (B, Hq, Sq, D)), ("k", k, (B, Hkv, Skv, D)), ("v", v, (B, Hkv, Skv, D)),
                             ("out", out, (B, Hq, Sq, D))):
            if t.device.type != "cpu" or t.dtype != self.dtype or tuple(t.shape) != shp or not t.is_contiguous():
                raise ValueError(f"{name}: expected a contiguous host tensor of shape {shp} and dtype {self.dtype}")
        g = self.groups
        qf, kf, vf, of = (t.view(-1, t.shape[2], D) for t in (q, k, v, out))
        comp = torch.cuda.current_stream(self.device)
        # the copy streams start after everything already queued on the caller's stream,
        # including the previous run() on these slots
        start = torch.cuda.Event()
        start.record(comp)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)
        nc = len(self.ranges)
        h2d_done = [torch.cuda.Event() for _ in range(nc)]
        comp_done = [torch.cuda.Event() for _ in range(nc)]
        d2h_done = [torch.cuda.Event() for _ in range(nc)]
        for c, (a, b) in enumerate(self.ranges):
            m = b - a
            slot = self.slots[c % 2]
            dq, dk, dv, do = (slot[x][:, : (m * g if x in "qo" else m)] for x in ("q", "k", "v", "o"))
            with torch.cuda.stream(self.h2d):
                if c >= 2:
                    self.h2d.wait_event(comp_done[c - 2])  # the slot's inputs have been consumed
                dq[0].copy_(qf[a * g:b * g], non_blocking=True)
                dk[0].copy_(kf[a:b], non_blocking=True)
                dv[0].copy_(vf[a:b], non_blocking=True)
                h2d_done[c].record(self.h2d)
            comp.wait_event(h2d_done[c])
            if c >= 2:
                comp.wait_event(d2h_done[c - 2])  # the slot's output has left the device
            self.plans[m].run(dq, dk, dv, do)
            comp_done[c].record(comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(comp_done[c])
                of[a * g:b * g].copy_(do[0], non_blocking=True)
                d2h_done[c].record(self.d2h)
        comp.wait_event(d2h_done[-1])
        return out


def run_sage_attn(q, k, v, causal=False, sm_scale=None, *, pv="16bit", smooth_k=True, tensor_layout="HND",
                  out=None, fused_q=None, blkq=128):
    """Drop-in for run_sage_attn (triton_impl.py:162-200) on sm_100a.

    q: [B, Hq, Sq, D], k/v: [B, Hkv, Skv, D] (HND; NHD with tensor_layout="NHD"), fp16 or bf16,
    D in {64, 128}. Returns o with q's shape and dtype. ``fused_q``: where Q is quantised
    (SagePlan; None = sage_run's choice); the output is bit-identical either way. ``blkq``:
    query rows per Q scale (128 is the reference's scheme; 64, 32, 16 or 1 = per token are
    finer, for inputs whose query rows have outliers).
    """
    _check_tensor("q", q)
    for name, t in (("k", k), ("v", v)):
        _check_tensor(name, t, q.dtype)
        if t.device != q.device:
            raise ValueError(f"{name} is on {t.device}, q on {q.device}")
    if q.dtype not in _DTYPES:
        raise TypeError(f"q/k/v must be float16 or bfloat16, got {q.dtype}")
    B, Hq, Sq, D, _ = _dims(q, tensor_layout)
    _, Hkv, Skv, _, _ = _dims(k, tensor_layout)
    plan = SagePlan(B, Hq, Hkv, Sq, Skv, D, q.dtype, q.device, pv=pv, smooth_k=smooth_k, causal=causal,
                    sm_scale=sm_scale, fused_q=fused_q, blkq=blkq)
    with torch.cuda.device(q.device):
        return plan.run(q, k, v, out=out, tensor_layout=tensor_layout)


run = run_sage_attn


def device_status(device=None) -> int:
    """Synchronise the current stream and return (and clear) the device watchdog bits; raises
    SageError(SAGE_ERR_TIMEOUT) when a device-side wait ran out."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    bits = ctypes.c_int(0)
    with torch.cuda.device(dev):
        rc = N.load().sage_device_status(ctypes.byref(bits), _stream_ptr(dev))
    N.check("sage_device_status", rc)
    return bits.value


def watchdog_selftest(limit_us: int = 2000, device=None) -> int:
    """Run the bounded-wait self test and return the status bits it left (expected: the
    epilogue-timeout bit). The context stays usable."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    lib = N.load()
    with torch.cuda.device(dev):
        N.check("sage_watchdog_selftest", lib.sage_watchdog_selftest(int(limit_us), _stream_ptr(dev)))
        bits = ctypes.c_int(0)
        rc = lib.sage_device_status(ctypes.byref(bits), _stream_ptr(dev))
    if rc not in (N.SAGE_OK, N.SAGE_ERR_TIMEOUT):
        N.check("sage_device_status", rc)
    return bits.value
