"""ctypes binding of libsage_sm100.so (C ABI in include/sage_sm100.h).

There is no fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from ._build import LIB_PATH

# Constants mirrored from include/sage_sm100.h.
SAGE_ABI_VERSION = 2
SAGE_OK = 0
SAGE_ERR_INVALID_ARG = -1
SAGE_ERR_UNSUPPORTED_ARCH = -2
SAGE_ERR_CUDA = -3
SAGE_ERR_TIMEOUT = -4
SAGE_ERR_WORKSPACE = -5
SAGE_DTYPE_F16 = 0
SAGE_DTYPE_BF16 = 1
SAGE_PV_16BIT = 0
SAGE_PV_FP8 = 1
SAGE_FLAG_SMOOTH_K = 1
SAGE_FLAG_KM_GIVEN = 2
SAGE_FLAG_FUSED_Q = 4
SAGE_FLAG_PREPASS_Q = 8
SAGE_FLAG_CODES16 = 16
# Q scale block size field (per_block_int8's BLKQ)
SAGE_FLAG_QBLK_MASK = 0x700
SAGE_FLAG_QBLK = {128: 0x000, 64: 0x100, 32: 0x200, 16: 0x300, 1: 0x400}


def qblk_flag(blkq: int) -> int:
    """SAGE_FLAG_QBLK_* bits for a Q block of `blkq` rows (128, 64, 32, 16 or 1)."""
    if blkq not in SAGE_FLAG_QBLK:
        raise ValueError(f"BLKQ={blkq} unsupported: the sm_100a kernels take Q blocks of 128, 64, 32, 16 or 1 rows")
    return SAGE_FLAG_QBLK[blkq]

# Every symbol the header declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I64P = ctypes.POINTER(ctypes.c_int64)
_I = ctypes.c_int
_U = ctypes.c_uint
_F = ctypes.c_float
_SZ = ctypes.c_size_t
SIGNATURES = {
    "sage_abi_version": (_I, []),
    "sage_last_error": (ctypes.c_char_p, []),
    "sage_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _I, _U]),
    "sage_per_block_int8": (_I, [_P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _F, _U,
                                 _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sage_per_block_int8_noalloc": (_I, [_P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _F, _U,
                                         _P, _P, _P, _P, _P, _P]),
    "sage_quant_v_fp8": (_I, [_P, _I, _I64, _I64, _I64, _I64, _I64P, _P, _P, _P, _SZ, _P]),
    "sage_attn_fwd": (_I, [_P, _P, _P, _P, _P, _I64P, _P, _P, _I64P, _I, _I, _I, _U,
                           _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "sage_attn_fwd_codes16": (_I, [_P, _P, _P, _P, _P, _I64P, _P, _P, _I64P, _I, _I, _I, _U,
                                   _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "sage_attn_fwd_fused_q": (_I, [_P, _I64P, _F, _P, _P, _P, _I64P, _P, _P, _I64P, _I, _I, _I, _U,
                                   _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "sage_prepass": (_I, [_P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _I64P, _F, _I, _U,
                          _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sage_run": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _I64P, _I64P,
                      _I, _F, _I, _U, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sage_flash_attn_fwd": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _I64P, _I64P,
                                 _I, _F, _P]),
    "sage_per_block_int8_varlen": (_I, [_P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P,
                                        _I64P, _I64P, _F, _U, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sage_run_varlen": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P,
                             _I64P, _I64P, _I64P, _I64P, _I, _F, _I, _U, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "sage_flash_attn_varlen_fwd": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P,
                                        _I64P, _I64P, _I64P, _I64P, _I, _F, _P]),
    "sage_device_status": (_I, [ctypes.POINTER(ctypes.c_int), _P]),
    "sage_watchdog_selftest": (_I, [_U, _P]),
}

_lib = None
_lock = threading.Lock()


class SageError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def lib_path() -> str:
    return os.environ.get("SAGE_SM100_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load the library once; raise if it is missing (no CPU or library fallback exists)."""
    global _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libsage_sm100.so not found at {path}; build it with `python -m tribench_b200._build` "
                    "(the sage_attn CUDA path has no fallback)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            ver = lib.sage_abi_version()
            if ver != SAGE_ABI_VERSION:
                raise RuntimeError(f"{path} has ABI version {ver}, expected {SAGE_ABI_VERSION}")
            _lib = lib
    return _lib


def check(fn: str, rc: int) -> None:
    if rc != SAGE_OK:
        msg = load().sage_last_error()
        raise SageError(fn, rc, msg.decode() if msg else "")


def strides3(*vals) -> ctypes.Array:
    arr = (ctypes.c_int64 * 3)(*[int(x) for x in vals])
    return arr


def strides2(*vals) -> ctypes.Array:
    return (ctypes.c_int64 * 2)(*[int(x) for x in vals])
