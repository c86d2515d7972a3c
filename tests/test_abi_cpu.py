"""CPU: the C-ABI library loads, exports every symbol include/sage_sm100.h declares, and rejects
bad arguments with SAGE_ERR_INVALID_ARG before touching a GPU (no compute call is made here)."""
import ctypes
import os
import re

import pytest

from tribench_b200 import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sage_sm100.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(sage_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_entry_points():
    fns = declared_functions()
    for name in ("sage_per_block_int8", "sage_attn_fwd", "sage_run", "sage_quant_v_fp8", "sage_workspace_bytes",
                 "sage_last_error", "sage_abi_version", "sage_device_status"):
        assert name in fns


def test_library_exports_every_declared_symbol():
    lib = N.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in sage_sm100.h but not exported"
        assert name in N.SIGNATURES, f"{name} has no ctypes signature in _native.SIGNATURES"


def test_abi_version():
    assert N.load().sage_abi_version() == N.SAGE_ABI_VERSION == 2


def test_workspace_bytes():
    lib = N.load()
    assert lib.sage_workspace_bytes(2, 32, 8192, 128, N.SAGE_PV_16BIT, 0) == 0
    ws = lib.sage_workspace_bytes(2, 32, 8192, 128, N.SAGE_PV_16BIT, N.SAGE_FLAG_SMOOTH_K)
    assert ws == 2 * 32 * (8192 // 512) * 128 * 8
    ws8 = lib.sage_workspace_bytes(2, 32, 8192, 128, N.SAGE_PV_FP8, N.SAGE_FLAG_SMOOTH_K)
    assert ws8 == ws + 2 * 32 * 16 * 128 * 4
    # head_dim 64: sage_run's default route also keeps K's fp16 codes in the workspace
    stats64 = 2 * 32 * 16 * 64 * 8
    codes64 = 2 * 32 * 8192 * 64 * 2
    assert lib.sage_workspace_bytes(2, 32, 8192, 64, N.SAGE_PV_16BIT, N.SAGE_FLAG_SMOOTH_K) == stats64 + codes64
    for route in (N.SAGE_FLAG_PREPASS_Q, N.SAGE_FLAG_FUSED_Q):
        assert lib.sage_workspace_bytes(2, 32, 8192, 64, N.SAGE_PV_16BIT, N.SAGE_FLAG_SMOOTH_K | route) == stats64


def _dummy(n=1 << 12):
    buf = (ctypes.c_uint8 * (n + 16))()
    addr = (ctypes.addressof(buf) + 15) & ~15
    return buf, ctypes.c_void_p(addr)


def _pbi8(head_dim=128, strides=(8 * 128, 8 * 128, 128), flags=0, k_mean=True, ws_bytes=1 << 20):
    lib = N.load()
    keep, p = _dummy()
    s = N.strides3(*strides)
    return lib.sage_per_block_int8(p, p, N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, head_dim, s, s, ctypes.c_float(0.0),
                                   flags, p, p, p, p, p if k_mean else None, p, ws_bytes, None)


def test_rejects_unsupported_head_dim():
    assert _pbi8(head_dim=96) == N.SAGE_ERR_INVALID_ARG
    assert "head_dim" in N.load().sage_last_error().decode()


def test_rejects_bad_strides():
    assert _pbi8(strides=(1024, 1024, 100)) == N.SAGE_ERR_INVALID_ARG
    assert "stride" in N.load().sage_last_error().decode()


def test_smoothing_needs_k_mean_and_workspace():
    assert _pbi8(flags=N.SAGE_FLAG_SMOOTH_K, k_mean=False) == N.SAGE_ERR_INVALID_ARG
    assert _pbi8(flags=N.SAGE_FLAG_SMOOTH_K, ws_bytes=0) == N.SAGE_ERR_WORKSPACE


def test_attn_rejects_causal_with_unequal_lengths_and_bad_mode():
    lib = N.load()
    keep, p = _dummy()
    s = N.strides3(8 * 128, 8 * 128, 128)
    rc = lib.sage_attn_fwd(p, p, p, p, p, s, None, p, s, N.SAGE_DTYPE_F16, N.SAGE_PV_16BIT, 1, 0, 1, 1, 1, 8, 16, 128,
                           None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "causal" in lib.sage_last_error().decode()
    rc = lib.sage_attn_fwd(p, p, p, p, p, s, None, p, s, N.SAGE_DTYPE_F16, 7, 0, 0, 1, 1, 1, 8, 8, 128, None)
    assert rc == N.SAGE_ERR_INVALID_ARG
    rc = lib.sage_attn_fwd(p, p, p, p, p, s, None, p, s, 5, N.SAGE_PV_16BIT, 0, 0, 1, 1, 1, 8, 8, 128, None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "dtype" in lib.sage_last_error().decode()


def test_rejects_gqa_mismatch_and_empty():
    lib = N.load()
    keep, p = _dummy()
    s = N.strides3(8 * 128, 8 * 128, 128)
    rc = lib.sage_attn_fwd(p, p, p, p, p, s, None, p, s, N.SAGE_DTYPE_F16, N.SAGE_PV_16BIT, 0, 0, 1, 3, 2, 8, 8, 128,
                           None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "multiple" in lib.sage_last_error().decode()
    rc = lib.sage_attn_fwd(p, p, p, p, p, s, None, p, s, N.SAGE_DTYPE_F16, N.SAGE_PV_16BIT, 0, 0, 1, 1, 1, 0, 8, 128,
                           None)
    assert rc == N.SAGE_ERR_INVALID_ARG


def test_rejects_misaligned_pointer():
    lib = N.load()
    keep, p = _dummy()
    bad = ctypes.c_void_p(p.value + 4)
    s = N.strides3(8 * 128, 8 * 128, 128)
    rc = lib.sage_attn_fwd(bad, p, p, p, p, s, None, p, s, N.SAGE_DTYPE_F16, N.SAGE_PV_16BIT, 0, 0, 1, 1, 1, 8, 8, 128,
                           None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "aligned" in lib.sage_last_error().decode()


def test_error_message_is_cleared_by_next_call():
    lib = N.load()
    assert _pbi8(head_dim=96) == N.SAGE_ERR_INVALID_ARG
    assert lib.sage_last_error().decode() != ""
    assert lib.sage_workspace_bytes(1, 1, 1, 128, 0, 0) == 0
    assert _pbi8(strides=(1024, 1024, 100)) == N.SAGE_ERR_INVALID_ARG
    assert "head_dim" not in lib.sage_last_error().decode()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """Host-side validation only (no device here): the allocation-free variant refuses sizes
    whose statistics need more than its built-in 4 MiB scratch, before any CUDA call."""
    lib = N.load()
    keep, p = _dummy()
    s = N.strides3(8 * 128, 8 * 128, 128)
    # batch * heads_kv * ceil(seq_kv / 512) * head_dim = 128 * 64 * 1 * 128 = 1048576 > 524288
    rc = lib.sage_per_block_int8_noalloc(p, p, N.SAGE_DTYPE_F16, 128, 64, 64, 8, 8, 128, s, s, ctypes.c_float(0.0),
                                         N.SAGE_FLAG_SMOOTH_K, p, p, p, p, p, None)
    assert rc == N.SAGE_ERR_INVALID_ARG
    assert "scratch" in lib.sage_last_error().decode()


def test_flash_rejects_bad_arguments_before_any_cuda_call():
    lib = N.load()
    keep, p = _dummy()
    s = N.strides3(8 * 128, 8 * 128, 128)
    args = lambda **kw: dict(dict(dtype=N.SAGE_DTYPE_F16, B=1, Hq=1, Hkv=1, Sq=8, Skv=8, D=128, causal=0), **kw)

    def call(q=p, **kw):
        a = args(**kw)
        return lib.sage_flash_attn_fwd(q, p, p, p, a["dtype"], a["B"], a["Hq"], a["Hkv"], a["Sq"], a["Skv"], a["D"],
                                       s, s, s, s, a["causal"], 0.0, None)

    assert call(D=96) == N.SAGE_ERR_INVALID_ARG and "head_dim" in lib.sage_last_error().decode()
    assert call(causal=1, Skv=16) == N.SAGE_ERR_INVALID_ARG and "causal" in lib.sage_last_error().decode()
    assert call(Hq=3, Hkv=2) == N.SAGE_ERR_INVALID_ARG and "multiple" in lib.sage_last_error().decode()
    assert call(dtype=5) == N.SAGE_ERR_INVALID_ARG
    assert call(q=ctypes.c_void_p(p.value + 4)) == N.SAGE_ERR_INVALID_ARG
    assert "aligned" in lib.sage_last_error().decode()
    assert call(q=None) == N.SAGE_ERR_INVALID_ARG


def _distinct(n, size=1 << 12):
    """n non-overlapping 16-byte aligned host buffers (kept alive by the returned list)."""
    bufs = [_dummy(size) for _ in range(n)]
    return [b for b, _ in bufs], [ptr for _, ptr in bufs]


def test_fused_q_makes_q_buffers_optional():
    """Host-side validation (no device here): NULL q_i8 / q_scale are rejected unless Q is
    quantised in the attention kernel."""
    lib = N.load()
    keep, (q, k, v, o, ki, ksc, p) = _distinct(7)
    s = N.strides3(8 * 128, 8 * 128, 128)

    def run(flags, qi):
        return lib.sage_run(q, k, v, o, N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, 128, s, s, s, s, 0, 0.0, N.SAGE_PV_16BIT,
                            flags, qi, qi, ki, ksc, None, None, None, None, 0, None)

    assert run(N.SAGE_FLAG_PREPASS_Q, None) == N.SAGE_ERR_INVALID_ARG and "NULL" in lib.sage_last_error().decode()
    # fused (the flag, or head_dim 128 by default): the arguments pass validation and the call
    # then stops at the missing device
    assert run(N.SAGE_FLAG_FUSED_Q, None) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)
    assert run(0, None) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)
    assert run(N.SAGE_FLAG_FUSED_Q | N.SAGE_FLAG_PREPASS_Q, p) == N.SAGE_ERR_INVALID_ARG
    # sage_prepass needs q_i8 / q_scale unless told that Q is left to the attention kernel
    pre = lambda flags: lib.sage_prepass(p, p, p, N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, 128, s, s, s, 0.0,
                                         N.SAGE_PV_16BIT, flags, None, None, p, p, None, None, None, None, 0, None)
    assert pre(0) == N.SAGE_ERR_INVALID_ARG
    assert pre(N.SAGE_FLAG_FUSED_Q) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)


def test_output_aliasing_is_rejected_before_any_cuda_call():
    """Host-side validation (no device here): an output buffer that shares bytes with k, v, an
    intermediate or the workspace, or overlaps q as a different view, is rejected with
    SAGE_ERR_INVALID_ARG (the head_dim-64 route of sage_run parks Q's codes in o while K and V
    are still to be read). o = q as the identical view passes validation (in-place is safe:
    each CTA reads its query rows before writing the same rows of o)."""
    lib = N.load()
    keep, (q, k, v, o, qi, qsc, ki, ksc, ws) = _distinct(9, size=1 << 14)
    s = N.strides3(8 * 128, 8 * 128, 128)  # [1, 1, 8, 128] fp16: 2048 bytes
    off = lambda ptr, n: ctypes.c_void_p(ptr.value + n)

    def run(o_ptr, head_dim=128, flags=N.SAGE_FLAG_SMOOTH_K | N.SAGE_FLAG_PREPASS_Q, q_ptr=q, os=s):
        return lib.sage_run(q_ptr, k, v, o_ptr, N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, head_dim, s, s, s, os, 0, 0.0,
                            N.SAGE_PV_16BIT, flags, qi, qsc, ki, ksc, off(ws, 4096), None, None, ws, 4096, None)

    def msg():
        return lib.sage_last_error().decode()

    assert run(o) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)  # disjoint buffers: stops at the missing device
    assert run(off(k, 1024)) == N.SAGE_ERR_INVALID_ARG and "overlaps k" in msg()
    assert run(off(v, 16)) == N.SAGE_ERR_INVALID_ARG and "overlaps v" in msg()
    assert run(off(ki, 512)) == N.SAGE_ERR_INVALID_ARG and "overlaps k_i8" in msg()
    assert run(off(ws, 0)) == N.SAGE_ERR_INVALID_ARG and "overlaps workspace" in msg()
    assert run(off(q, 256)) == N.SAGE_ERR_INVALID_ARG and "overlaps q" in msg()
    # the same base as q but other strides is a different view
    assert run(q, os=N.strides3(8 * 256, 8 * 128, 256)) == N.SAGE_ERR_INVALID_ARG and "overlaps q" in msg()
    # in place (o = q, same strides) is allowed, on either route
    assert run(q) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)
    assert run(q, head_dim=64, flags=N.SAGE_FLAG_SMOOTH_K) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)
    assert run(off(k, 64), head_dim=64, flags=N.SAGE_FLAG_SMOOTH_K) == N.SAGE_ERR_INVALID_ARG

    # the split entry point and the flash pack check the same way
    rc = lib.sage_attn_fwd(qi, qsc, ki, ksc, v, s, None, off(ki, 128), s, N.SAGE_DTYPE_F16, N.SAGE_PV_16BIT, 0, 0, 1, 1,
                           1, 8, 8, 128, None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "overlaps k_i8" in msg()
    rc = lib.sage_flash_attn_fwd(q, k, v, off(v, 2032), N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, 128, s, s, s, s, 0, 0.0, None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "overlaps v" in msg()
    # one byte past v's last element is no overlap
    rc = lib.sage_flash_attn_fwd(q, k, v, off(v, 2048), N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, 128, s, s, s, s, 0, 0.0, None)
    assert rc not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)

    # packed sequences: o [total_q, H, D] against k
    cu_keep, cu = _dummy(64)
    s2 = N.strides2(128, 128)
    rc = lib.sage_run_varlen(q, k, v, off(k, 1024), N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, 8, 8, 128, cu, cu, s2, s2, s2, s2,
                             0, 0.0, N.SAGE_PV_16BIT, N.SAGE_FLAG_PREPASS_Q, qi, qsc, ki, ksc, None, None, None, None,
                             0, None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "overlaps k" in msg()


def test_q_block_field_is_validated():
    """Host-side validation (no device here): a SAGE_FLAG_QBLK_* field outside the five sizes,
    or any other flag on an attention-only entry point, is SAGE_ERR_INVALID_ARG."""
    lib = N.load()
    keep, (q, k, qi, qsc, ki, ksc, v, o) = _distinct(8)
    s = N.strides3(8 * 128, 8 * 128, 128)

    def pbi8(flags):
        return lib.sage_per_block_int8(q, k, N.SAGE_DTYPE_F16, 1, 1, 1, 8, 8, 128, s, s, ctypes.c_float(0.0), flags,
                                       qi, qsc, ki, ksc, None, None, 0, None)

    for blkq, bits in N.SAGE_FLAG_QBLK.items():
        assert pbi8(bits) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG), blkq  # valid: stops at the device
    for bad in (0x500, 0x600, 0x700):
        assert pbi8(bad) == N.SAGE_ERR_INVALID_ARG and "SAGE_FLAG_QBLK" in lib.sage_last_error().decode()

    def attn(flags):
        return lib.sage_attn_fwd(qi, qsc, ki, ksc, v, s, None, o, s, N.SAGE_DTYPE_F16, N.SAGE_PV_16BIT, 0, flags,
                                 1, 1, 1, 8, 8, 128, None)

    assert attn(N.SAGE_FLAG_QBLK[1]) not in (N.SAGE_OK, N.SAGE_ERR_INVALID_ARG)
    assert attn(N.SAGE_FLAG_SMOOTH_K) == N.SAGE_ERR_INVALID_ARG
    assert attn(0x500) == N.SAGE_ERR_INVALID_ARG
    with pytest.raises(ValueError, match="BLKQ=8"):
        N.qblk_flag(8)
