"""TEST INFRASTRUCTURE ONLY — the CPU oracle of the sage_attn path.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import this package, and only as the checker / the timed CPU restatement. The product
(``tribench_b200``) never imports it and has no CPU fallback.

Contents:
  * bit-exact pre-pass restatement (C, ``sage_quant_ref.c``, via ctypes):
    ``quant_per_block_int8`` (kernels/sage_attn/triton_impl.py:7-33, 35-82),
    ``k_mean`` (the smoothing statistic), ``quant_v_fp8`` / ``e4m3_decode``;
  * ``ref_attention``: exact attention, restating ``ref`` (kernels/sage_attn/reference.py:15-24)
    in fp64 (numpy) one (batch, head) slice at a time so it never materialises B*H*S*S;
  * ``ref_attention_torch``: the same in fp32 through torch on the CPU (the reference's own
    PyTorch path, used as the timed CPU baseline);
  * ``sage_model``: the quantised algorithm evaluated exactly (int64 QK^T of the int8
    operands, dequantised scores, exact softmax, fp64 P.V) — the ideal output of the block
    scheme, against which the GPU's own rounding (exp2 approximation, 16-bit/FP8 P) is measured.

Parity is pinned by ``tests/golden/`` fixtures produced by running the reference's
``triton_impl.py`` under ``TRITON_INTERPRET=1`` (see ``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle_sage.so")
_lib = None

# Must match the CUDA pre-pass (tribench_b200/csrc/sage_quant.cuh).
STATS_CHUNK = 512
QUANT_THREADS = 256
LOG2E_LITERAL = 1.44269504  # triton_impl.py:69


def build() -> str:
    """Compile the C restatement (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        i8p = ctypes.POINTER(ctypes.c_int8)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        f64p = ctypes.POINTER(ctypes.c_double)
        i64 = ctypes.c_int64
        lib.oracle_quant_per_block_int8.argtypes = [f32p, i64, i64, i64, i64, ctypes.c_float, f32p, i8p, f32p]
        lib.oracle_quant_per_block_int8.restype = None
        lib.oracle_k_mean.argtypes = [f32p, i64, i64, i64, i64, i64, f64p, f32p]
        lib.oracle_k_mean.restype = None
        lib.oracle_e4m3_encode.argtypes = [ctypes.c_float]
        lib.oracle_e4m3_encode.restype = ctypes.c_uint8
        lib.oracle_e4m3_decode.argtypes = [ctypes.c_uint8]
        lib.oracle_e4m3_decode.restype = ctypes.c_float
        lib.oracle_quant_v_fp8.argtypes = [f32p, i64, i64, i64, u8p, f32p]
        lib.oracle_quant_v_fp8.restype = None
        _lib = lib
    return _lib


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


def q_multiplier(sm_scale: float | None, head_dim: int) -> np.float32:
    """fp32(sm_scale * 1.44269504), sm_scale defaulting to head_dim**-0.5 (triton_impl.py:60-69)."""
    if sm_scale is None:
        sm_scale = head_dim ** -0.5
    return np.float32(sm_scale * LOG2E_LITERAL)


def quant_per_block_int8(x: np.ndarray, blk: int, mult: float = 1.0, km: np.ndarray | None = None):
    """x: [..., S, D] values exactly representable in fp32 -> (int8 [..., S, D], fp32 [..., ceil(S/blk)])."""
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, S, D = x.shape
    nh = int(np.prod(lead)) if lead else 1
    nb = (S + blk - 1) // blk
    out = np.zeros(x.shape, dtype=np.int8)
    scales = np.zeros((*lead, nb), dtype=np.float32)
    kmp = None
    if km is not None:
        km = np.ascontiguousarray(km, dtype=np.float32).reshape(nh, D)
        kmp = _ptr(km, ctypes.c_float)
    lib.oracle_quant_per_block_int8(_ptr(x, ctypes.c_float), nh, S, D, blk, ctypes.c_float(mult), kmp,
                                    _ptr(out, ctypes.c_int8), _ptr(scales, ctypes.c_float))
    return out, scales


def k_mean(k: np.ndarray) -> np.ndarray:
    """Per-(batch, head) channel mean of K in the CUDA pre-pass's fp64 summation order."""
    lib = _load()
    k = np.ascontiguousarray(k, dtype=np.float32)
    *lead, S, D = k.shape
    nh = int(np.prod(lead)) if lead else 1
    rpp = QUANT_THREADS // (D // 8)
    scratch = np.zeros(rpp * D + D, dtype=np.float64)
    km = np.zeros((*lead, D), dtype=np.float32)
    lib.oracle_k_mean(_ptr(k, ctypes.c_float), nh, S, D, STATS_CHUNK, rpp, _ptr(scratch, ctypes.c_double),
                      _ptr(km, ctypes.c_float))
    return km


def quant_v_fp8(v: np.ndarray):
    """V [..., S, D] -> (e4m3 codes uint8 [..., S, D], per-channel scales fp32 [..., D])."""
    lib = _load()
    v = np.ascontiguousarray(v, dtype=np.float32)
    *lead, S, D = v.shape
    nh = int(np.prod(lead)) if lead else 1
    out = np.zeros(v.shape, dtype=np.uint8)
    scales = np.zeros((*lead, D), dtype=np.float32)
    lib.oracle_quant_v_fp8(_ptr(v, ctypes.c_float), nh, S, D, _ptr(out, ctypes.c_uint8), _ptr(scales, ctypes.c_float))
    return out, scales


_E4M3_TABLE = None


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    global _E4M3_TABLE
    if _E4M3_TABLE is None:
        lib = _load()
        _E4M3_TABLE = np.array([lib.oracle_e4m3_decode(i) for i in range(256)], dtype=np.float32)
    return _E4M3_TABLE[codes]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    lib = _load()
    flat = np.asarray(x, dtype=np.float32).ravel()
    return np.array([lib.oracle_e4m3_encode(float(v)) for v in flat], dtype=np.uint8).reshape(np.shape(x))


def _expand_kv(k: np.ndarray, hq: int) -> np.ndarray:
    hkv = k.shape[1]
    if hkv == hq:
        return k
    return np.repeat(k, hq // hkv, axis=1)


def ref_attention(q, k, v, causal: bool = False, sm_scale: float | None = None, heads=None,
                  rows=None) -> np.ndarray:
    """Exact attention in fp64 (restates reference.py:15-24), one (b, h) slice at a time.

    q: [B, Hq, Sq, D], k/v: [B, Hkv, Skv, D] (any float dtype). ``heads``: optional list of
    (b, h) pairs to evaluate; the others are left as NaN. ``rows``: optional array of query
    rows to evaluate (default all). Returns fp64 [B, Hq, len(rows), D].
    """
    q = np.asarray(q)
    B, H, Sq, D = q.shape
    Hkv = np.shape(k)[1]
    g = H // Hkv
    Skv = np.shape(k)[2]
    rows = np.arange(Sq) if rows is None else np.asarray(rows)
    if sm_scale is None:
        sm_scale = D ** -0.5
    out = np.full((B, H, len(rows), D), np.nan)
    pairs = heads if heads is not None else [(b, h) for b in range(B) for h in range(H)]
    for b, h in pairs:
        qq = np.asarray(q[b, h], dtype=np.float64)[rows]
        kk = np.asarray(k[b, h // g], dtype=np.float64)
        vv = np.asarray(v[b, h // g], dtype=np.float64)
        s = (qq @ kk.T) * sm_scale
        if causal:
            s = np.where(np.arange(Skv)[None, :] <= rows[:, None], s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[b, h] = (p / p.sum(axis=1, keepdims=True)) @ vv
    return out


def ref_attention_torch(q, k, v, causal: bool = False, sm_scale: float | None = None, heads=None):
    """The reference's PyTorch ``ref`` (reference.py:15-24) evaluated in fp32 on the CPU per
    (b, h) slice — mathematically identical, bounded memory. Returns a torch fp32 tensor."""
    import torch

    q = torch.as_tensor(q).float()
    k = torch.as_tensor(k).float()
    v = torch.as_tensor(v).float()
    B, H, Sq, D = q.shape
    g = H // k.shape[1]
    if sm_scale is None:
        sm_scale = D ** -0.5
    out = torch.full((B, H, Sq, D), float("nan"))
    pairs = heads if heads is not None else [(b, h) for b in range(B) for h in range(H)]
    mask = None
    if causal:
        mask = torch.tril(torch.ones((Sq, k.shape[2]))) == 0
    for b, h in pairs:
        p = torch.matmul(q[b, h], k[b, h // g].transpose(0, 1)) * sm_scale
        if mask is not None:
            p = p.masked_fill(mask, float("-inf"))
        out[b, h] = torch.matmul(torch.softmax(p, dim=-1), v[b, h // g])
    return out


def sage_model(q_i8, q_scale, k_i8, k_scale, v, causal: bool = False, heads=None, rows=None,
               blkq: int = 128, blkk: int = 64) -> np.ndarray:
    """Exact evaluation of the quantised scheme: s = (q_i8 . k_i8^T) * q_scale * k_scale (base-2
    logits; the int8 dot products are exact in fp64), softmax in base 2, P.V in fp64.
    ``v`` is the 16-bit V as floats, or (FP8 P.V) the e4m3 codes decoded times v_scale.
    ``heads`` / ``rows`` select (b, h) pairs and query rows as in ref_attention. Returns fp64."""
    q_i8 = np.asarray(q_i8)
    B, H, Sq, D = q_i8.shape
    Hkv = np.shape(k_i8)[1]
    g = H // Hkv
    Skv = np.shape(k_i8)[2]
    rows = np.arange(Sq) if rows is None else np.asarray(rows)
    qs = np.asarray(q_scale, dtype=np.float64)
    ks = np.asarray(k_scale, dtype=np.float64)
    out = np.full((B, H, len(rows), D), np.nan)
    pairs = heads if heads is not None else [(b, h) for b in range(B) for h in range(H)]
    rk = np.arange(Skv) // blkk
    for b, h in pairs:
        qq = np.asarray(q_i8[b, h], dtype=np.float64)[rows]
        kk = np.asarray(k_i8[b, h // g], dtype=np.float64)
        vv = np.asarray(v[b, h // g], dtype=np.float64)
        s = qq @ kk.T  # exact: |s| <= 127^2 * D < 2^53
        s = s * qs[b, h][rows // blkq][:, None] * ks[b, h // g][rk][None, :]
        if causal:
            s = np.where(np.arange(Skv)[None, :] <= rows[:, None], s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp2(s)
        out[b, h] = (p / p.sum(axis=1, keepdims=True)) @ vv
    return out
