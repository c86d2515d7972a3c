"""TriBench's correctness gate for cases too large for its unchunked ``ref``.

TriBench checks a variant by evaluating the pack's ``ref`` on the same inputs
(tribench/bench.py:150-154) and passing iff ``torch.allclose(ref.float(), out.float(), atol,
rtol)`` (tribench/correctness.py:74-82). The attention packs' ``ref``
(kernels/sage_attn/reference.py:15-24, kernels/flash_attn/reference.py:15-28) materialises the
whole [B, H, Sq, Skv] score matrix in the input dtype, and the gate makes fp32 copies of both
outputs: at the long-context config (B=16, H=64, S=32768) the scores alone would be 2.2 TB.

``ref_chunked`` evaluates the same expression — ``softmax(q k^T * sm_scale [causal mask]) v``
in the input dtype, torch matmul and softmax — over (batch, head, query-row) chunks whose score
block stays under a byte budget; each output row depends only on its own query row, so chunking
changes no operation, only the shapes handed to the GEMM. ``gate_chunked`` applies TriBench's
tolerance resolution and ``allclose`` chunk by chunk (``all`` over chunks is the same predicate)
and reports the same max_abs / max_rel errors as correctness.py:74-78.

This module is harness code: it checks outputs and is never on the sage/flash compute path.
"""
from __future__ import annotations

import torch

# tribench/correctness.py:13-18
DEFAULT_TOLERANCES = {
    "fp32": (1e-5, 1e-4),
    "fp64": (1e-7, 1e-5),
    "fp16": (1e-2, 1e-2),
    "bf16": (1e-2, 1e-2),
}

# kernels/*/meta.json "correctness" blocks of the two attention packs
PACK_TOLERANCE = {"sage_attn": (5e-2, 5e-2), "flash_attn": (1e-2, 1e-2)}

DEFAULT_BUDGET_BYTES = 1 << 30


def tolerance(dtype_str: str, atol: float, rtol: float, per_dtype: dict | None = None) -> tuple[float, float]:
    """tribench/correctness.py:22-38: a per-dtype entry, else the pack's non-default atol/rtol,
    else the framework default for the dtype."""
    if per_dtype and dtype_str in per_dtype:
        d = per_dtype[dtype_str]
        return d.get("atol", atol), d.get("rtol", rtol)
    if atol != 1e-2 or rtol != 1e-2:
        return atol, rtol
    return DEFAULT_TOLERANCES.get(dtype_str, (atol, rtol))


def _hnd(t: torch.Tensor, tensor_layout: str) -> torch.Tensor:
    if t.dim() != 4:
        raise ValueError(f"expected a 4-D tensor, got shape {tuple(t.shape)}")
    return t.transpose(1, 2) if tensor_layout == "NHD" else t


def _chunks(q: torch.Tensor, k: torch.Tensor, causal: bool, budget_bytes: int):
    """(b, h, r0, r1) chunks: one query head at a time, as many rows as fit the score budget."""
    B, Hq, Sq, _ = q.shape
    Skv = k.shape[2]
    if causal and Sq != Skv:
        raise ValueError("causal attention requires seq_q == seq_kv (reference.py:19-22)")
    # the score block and the softmax output, plus one temporary of the same size
    per_row = 3 * max(Skv, 1) * q.element_size()
    rows = max(1, min(Sq, budget_bytes // per_row))
    for b in range(B):
        for h in range(Hq):
            for r0 in range(0, Sq, rows):
                yield b, h, r0, min(Sq, r0 + rows)


def _ref_rows(q, k, v, b, h, r0, r1, causal, sm_scale):
    """reference.py:15-24 for query rows [r0, r1) of head (b, h), in the input dtype."""
    g = q.shape[1] // k.shape[1]
    qh = q[b, h, r0:r1]
    # causal: keys past the chunk's last row are masked for every row in it
    kend = r1 if causal else k.shape[2]
    kh, vh = k[b, h // g, :kend], v[b, h // g, :kend]
    p = torch.matmul(qh, kh.transpose(0, 1)) * sm_scale
    if causal:
        rows = torch.arange(r0, r1, device=q.device).unsqueeze(1)
        cols = torch.arange(kend, device=q.device).unsqueeze(0)
        p = p.masked_fill(cols > rows, float("-inf"))
    return torch.matmul(torch.softmax(p, dim=-1), vh)


def ref_chunked(q, k, v, causal: bool = False, sm_scale: float | None = None, *, tensor_layout: str = "HND",
                out: torch.Tensor | None = None, budget_bytes: int = DEFAULT_BUDGET_BYTES) -> torch.Tensor:
    """The packs' ``ref`` (q [B,Hq,Sq,D], k/v [B,Hkv,Skv,D]; GQA by query-head groups), evaluated
    chunk by chunk in the input dtype with at most ``budget_bytes`` of score temporaries."""
    qh, kh, vh = (_hnd(t, tensor_layout) for t in (q, k, v))
    if qh.shape[1] % kh.shape[1]:
        raise ValueError("heads_q must be a multiple of heads_kv")
    scale = qh.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    if out is None:
        out = torch.empty_like(q)
    oh = _hnd(out, tensor_layout)
    with torch.no_grad():
        for b, h, r0, r1 in _chunks(qh, kh, causal, budget_bytes):
            oh[b, h, r0:r1] = _ref_rows(qh, kh, vh, b, h, r0, r1, causal, scale)
    return out


def gate_chunked(out, q, k, v, causal: bool = False, sm_scale: float | None = None, *, dtype_str: str,
                 atol: float, rtol: float, per_dtype: dict | None = None, tensor_layout: str = "HND",
                 budget_bytes: int = DEFAULT_BUDGET_BYTES) -> dict:
    """TriBench's check_correctness (correctness.py:41-103) of ``out`` against the packs' ``ref``,
    computed chunk by chunk. Returns passed, atol, rtol, max_abs_err, max_rel_err, plus the
    number of elements outside the tolerance (``n_fail``), the element count and the HND index
    (b, h, row, channel) of the element furthest outside the tolerance, or closest to it when all
    pass (``worst``: the largest |ref - out| - (atol + rtol |out|))."""
    atol, rtol = tolerance(dtype_str, atol, rtol, per_dtype)
    qh, kh, vh, oh = (_hnd(t, tensor_layout) for t in (q, k, v, out))
    if oh.shape != qh.shape:
        raise ValueError(f"output shape {tuple(out.shape)} != query shape {tuple(q.shape)}")
    scale = qh.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    dev = oh.device
    chunks = list(_chunks(qh, kh, causal, budget_bytes))
    max_abs = torch.zeros((), dtype=torch.float32, device=dev)
    # per chunk: the largest excess |ref - out| - (atol + rtol |out|) and its flat index
    worst = torch.zeros(len(chunks), dtype=torch.float32, device=dev)
    where = torch.zeros(len(chunks), dtype=torch.int64, device=dev)
    max_rel = torch.zeros((), dtype=torch.float32, device=dev)
    n_fail = torch.zeros((), dtype=torch.int64, device=dev)
    with torch.no_grad():
        for i, (b, h, r0, r1) in enumerate(chunks):
            ref = _ref_rows(qh, kh, vh, b, h, r0, r1, causal, scale).float()
            tri = oh[b, h, r0:r1].float()
            diff = (ref - tri).abs()
            # NaN propagates through max as in the unchunked reductions
            max_abs = torch.maximum(max_abs, diff.max())
            worst[i], where[i] = (diff - (atol + rtol * tri.abs())).flatten().max(0)
            max_rel = torch.maximum(max_rel, (diff / ref.abs().clamp(min=1e-20)).max())
            n_fail += (~torch.isclose(ref, tri, atol=atol, rtol=rtol)).sum()
    n_fail = int(n_fail.item())
    ci = int(worst.argmax().item()) if chunks else 0
    b, h, r0, _ = chunks[ci] if chunks else (0, 0, 0, 0)
    flat = int(where[ci].item()) if chunks else 0
    D = qh.shape[-1]
    return {"passed": n_fail == 0, "atol": atol, "rtol": rtol, "max_abs_err": max_abs.item(),
            "max_rel_err": max_rel.item(), "n_fail": n_fail, "numel": out.numel(),
            "worst": (b, h, r0 + flat // D, flat % D)}
