"""GPU: the allocation-free pre-pass entry point, sage_per_block_int8_noalloc.

Some callers cannot allocate device memory (their framework owns it, or cudaMalloc's implicit
device synchronisation is not allowed where they run). For them the library offers a variant of
sage_per_block_int8 that keeps its smoothing statistics in a scratch array compiled into the
library instead of a caller-provided workspace. This test calls it through the C ABI twice in a
row, on different inputs, and requires the same bits as the workspace entry point: the shared
scratch must not leak anything from one call into the next. It lives in its own file, named to
be collected last, and passes both alone and after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

import tribench_b200 as tb
from tribench_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _outputs(q, k):
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    return (torch.empty((B, Hq, Sq, D), dtype=torch.int8, device=DEV),
            torch.empty((B, Hq, (Sq + 127) // 128), dtype=torch.float32, device=DEV),
            torch.empty((B, Hkv, Skv, D), dtype=torch.int8, device=DEV),
            torch.empty((B, Hkv, (Skv + 63) // 64), dtype=torch.float32, device=DEV),
            torch.empty((B, Hkv, D), dtype=torch.float32, device=DEV))


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _call(lib, q, k, outs, noalloc):
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    qs = N.strides3(q.stride(0), q.stride(1), q.stride(2))
    ks = N.strides3(k.stride(0), k.stride(1), k.stride(2))
    stream = torch.cuda.current_stream(DEV).cuda_stream
    dt = N.SAGE_DTYPE_F16 if q.dtype == torch.float16 else N.SAGE_DTYPE_BF16
    qi, qsc, ki, ksc, km = outs
    if noalloc:
        rc = lib.sage_per_block_int8_noalloc(_vp(q), _vp(k), dt, B, Hq, Hkv, Sq, Skv, D, qs, ks, ctypes.c_float(0.0),
                                             N.SAGE_FLAG_SMOOTH_K, _vp(qi), _vp(qsc), _vp(ki), _vp(ksc), _vp(km),
                                             stream)
    else:
        nws = lib.sage_workspace_bytes(B, Hkv, Skv, D, N.SAGE_PV_16BIT, N.SAGE_FLAG_SMOOTH_K)
        ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=DEV)
        rc = lib.sage_per_block_int8(_vp(q), _vp(k), dt, B, Hq, Hkv, Sq, Skv, D, qs, ks, ctypes.c_float(0.0),
                                     N.SAGE_FLAG_SMOOTH_K, _vp(qi), _vp(qsc), _vp(ki), _vp(ksc), _vp(km), _vp(ws),
                                     nws, stream)
        torch.cuda.synchronize(DEV)  # keep the workspace alive until the kernels ran
    N.check("noalloc" if noalloc else "workspace", rc)
    torch.cuda.synchronize(DEV)
    return [t.cpu().numpy() for t in outs]


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = N.load()
    torch.cuda.set_device(DEV)
    cases = [
        (dict(batch_size=2, num_heads=4, seq_len=1500, head_dim=128, dist="offset", k_offset_std=2.0), 5, "fp16"),
        (dict(batch_size=1, num_heads=3, seq_len=777, head_dim=64, dist="offset", k_offset_std=3.0), 6, "bf16"),
    ]
    for case, seed, dtype in cases:  # two calls in a row on different inputs
        inp = tb.make_inputs(case, DEV, seed=seed, dtype=dtype)
        q, k = inp["q"], inp["k"]
        ref = _call(lib, q, k, _outputs(q, k), noalloc=False)
        got = _call(lib, q, k, _outputs(q, k), noalloc=True)
        for name, a, b in zip(("q_i8", "q_scale", "k_i8", "k_scale", "k_mean"), got, ref):
            np.testing.assert_array_equal(a, b, err_msg=f"{name} differs ({dtype}, seq {case['seq_len']})")
    assert tb.device_status(DEV) == 0
