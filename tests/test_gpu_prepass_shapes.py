"""GPU: the K pre-pass (statistics, channel mean and quantisation) at the shapes that stress
its chunking, against the oracle and between its two entry points.

The smoothing statistic keeps a fixed fp64 summation order (rows within a 512-row chunk per
thread, thread partials, then chunks in increasing order), so its bits must equal the oracle's
at ragged and chunk-boundary lengths, both head_dims and input types, NHD strides, many heads,
and a head of 157 chunks; and the workspace entry point must equal the allocation-free one.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import tribench_b200 as tb
from tribench_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def f32(t):
    return t.float().cpu().numpy()


def _check_vs_oracle(q, k, layout="HND"):
    qi, qs, ki, ks, km = tb.per_block_int8(q, k, smooth_k=True, return_km=True, tensor_layout=layout)
    assert tb.device_status(DEV) == 0
    if layout == "NHD":
        q, k = q.transpose(1, 2), k.transpose(1, 2)
    kf = f32(k)
    km_o = oracle.k_mean(kf)
    np.testing.assert_array_equal(km.cpu().numpy(), km_o)
    ki_o, ks_o = oracle.quant_per_block_int8(kf, 64, 1.0, km=km_o)
    np.testing.assert_array_equal(ki.cpu().numpy(), ki_o)
    np.testing.assert_array_equal(ks.cpu().numpy(), ks_o)
    qi_o, qs_o = oracle.quant_per_block_int8(f32(q), 128, oracle.q_multiplier(None, q.shape[-1]))
    np.testing.assert_array_equal(qi.cpu().numpy(), qi_o)
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_o)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [1, 63, 511, 512, 513, 1600, 4097])
def test_prepass_vs_oracle(dtype, D, S):
    case = dict(batch_size=2, num_heads=3, seq_len=S, head_dim=D, dist="offset", k_offset_std=3.0)
    inp = tb.make_inputs(case, DEV, seed=S + D, dtype=dtype)
    _check_vs_oracle(inp["q"], inp["k"])


def test_prepass_nhd_strides():
    case = dict(batch_size=1, num_heads=4, seq_len=1100, head_dim=128, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=3, dtype="fp16")
    q, k = (t.transpose(1, 2).contiguous() for t in (inp["q"], inp["k"]))  # [B, S, H, D]
    _check_vs_oracle(q, k, layout="NHD")


def test_many_heads():
    """1024 heads of 3 chunks each."""
    case = dict(batch_size=8, num_heads=128, seq_len=1300, head_dim=64, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=9, dtype="fp16")
    _check_vs_oracle(inp["q"], inp["k"])


def test_long_head():
    """80000 rows = 157 chunks of statistics in one head."""
    case = dict(batch_size=1, num_heads=1, seq_len=80000, head_dim=128, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=4, dtype="bf16")
    _check_vs_oracle(inp["q"], inp["k"])


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_workspace_and_allocation_free_entry_points_agree_bit_for_bit():
    """sage_per_block_int8 against sage_per_block_int8_noalloc on the H8K shape's Q and K
    (64 heads x 16 chunks)."""
    lib = N.load()
    case = dict(batch_size=2, num_heads=32, seq_len=8192, head_dim=128, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=1, dtype="fp16")
    q, k = inp["q"], inp["k"]  # [1, 64, 8192, 128]: the H8K heads flattened
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    qs = N.strides3(q.stride(0), q.stride(1), q.stride(2))
    ks = N.strides3(k.stride(0), k.stride(1), k.stride(2))
    stream = torch.cuda.current_stream(DEV).cuda_stream
    outs = []
    for noalloc in (False, True):
        o = (torch.empty((B, Hq, Sq, D), dtype=torch.int8, device=DEV),
             torch.empty((B, Hq, (Sq + 127) // 128), dtype=torch.float32, device=DEV),
             torch.empty((B, Hkv, Skv, D), dtype=torch.int8, device=DEV),
             torch.empty((B, Hkv, (Skv + 63) // 64), dtype=torch.float32, device=DEV),
             torch.empty((B, Hkv, D), dtype=torch.float32, device=DEV))
        if noalloc:
            rc = lib.sage_per_block_int8_noalloc(_vp(q), _vp(k), N.SAGE_DTYPE_F16, B, Hq, Hkv, Sq, Skv, D, qs, ks,
                                                 ctypes.c_float(0.0), N.SAGE_FLAG_SMOOTH_K, *(_vp(t) for t in o),
                                                 stream)
        else:
            nws = lib.sage_workspace_bytes(B, Hkv, Skv, D, N.SAGE_PV_16BIT, N.SAGE_FLAG_SMOOTH_K)
            ws = torch.empty(nws, dtype=torch.uint8, device=DEV)
            rc = lib.sage_per_block_int8(_vp(q), _vp(k), N.SAGE_DTYPE_F16, B, Hq, Hkv, Sq, Skv, D, qs, ks,
                                         ctypes.c_float(0.0), N.SAGE_FLAG_SMOOTH_K, *(_vp(t) for t in o), _vp(ws),
                                         nws, stream)
        N.check("per_block_int8", rc)
        torch.cuda.synchronize(DEV)
        outs.append(o)
    assert tb.device_status(DEV) == 0
    for a, b in zip(*outs):
        assert torch.equal(a, b)
