"""CPU: argument checks of the packed variable-length entry points (no GPU call is made).

The C ABI rejects bad shapes, strides and pointers with SAGE_ERR_INVALID_ARG before any CUDA call;
the Python layer validates the cu_seqlens prefix sums on the host.
"""
import ctypes

import pytest

from tribench_b200 import _native as N
from tribench_b200 import varlen


def test_seq_lengths_accepts_prefix_sums():
    assert varlen.seq_lengths([0, 3, 3, 10], 10, "cu") == [3, 0, 7]
    assert varlen.seq_lengths([0, 0], 0, "cu") == [0]


@pytest.mark.parametrize("cu,total,msg", [([0], 0, "entries"), ([1, 4], 4, "start at 0"), ([0, 5, 3], 3, "decreases"),
                                          ([0, 4, 9], 10, "ends at")])
def test_seq_lengths_rejects_bad_prefix_sums(cu, total, msg):
    with pytest.raises(ValueError, match=msg):
        varlen.seq_lengths(cu, total, "cu")


def test_causal_needs_equal_lengths_per_sequence():
    varlen.check_causal_lengths([3, 0, 7], [3, 0, 7])
    with pytest.raises(ValueError, match="sequence 1"):
        varlen.check_causal_lengths([3, 4, 7], [3, 5, 6])


def _buf():
    keep = (ctypes.c_char * 4096)()
    addr = (ctypes.addressof(keep) + 255) & ~255
    return keep, ctypes.c_void_p(addr)


def test_abi_varlen_rejects_bad_arguments_before_any_cuda_call():
    lib = N.load()
    keep, p = _buf()
    s2 = N.strides2(128, 8 * 128)
    base = dict(dtype=N.SAGE_DTYPE_F16, B=2, Hq=8, Hkv=8, Tq=100, Tk=100, mq=60, mk=60, D=128, cu=p, s=s2)

    def run(**kw):
        a = dict(base, **kw)
        return lib.sage_run_varlen(p, p, p, p, a["dtype"], a["B"], a["Hq"], a["Hkv"], a["Tq"], a["Tk"], a["mq"],
                                   a["mk"], a["D"], a["cu"], a["cu"], a["s"], a["s"], a["s"], a["s"], 0, 0.0,
                                   N.SAGE_PV_16BIT, 0, p, p, p, p, None, None, None, None, 0, None)

    def err():
        return lib.sage_last_error().decode()

    assert run(D=96) == N.SAGE_ERR_INVALID_ARG and "head_dim" in err()
    assert run(Tq=0) == N.SAGE_ERR_INVALID_ARG and "total_q" in err()
    assert run(mq=101) == N.SAGE_ERR_INVALID_ARG and "exceed" in err()
    assert run(cu=None) == N.SAGE_ERR_INVALID_ARG and "cu_seqlens" in err()
    assert run(cu=ctypes.c_void_p(p.value + 2)) == N.SAGE_ERR_INVALID_ARG and "aligned" in err()
    assert run(s=N.strides2(128, 100)) == N.SAGE_ERR_INVALID_ARG and "stride" in err()
    assert run(Hq=12) == N.SAGE_ERR_INVALID_ARG and "multiple" in err()
    rc = lib.sage_per_block_int8_varlen(p, p, N.SAGE_DTYPE_F16, 2, 8, 8, 100, 100, 60, 60, 128, p, p, s2, s2,
                                        ctypes.c_float(0.0), N.SAGE_FLAG_SMOOTH_K, p, p, p, p, p, None, 0, None)
    assert rc == N.SAGE_ERR_WORKSPACE
    rc = lib.sage_flash_attn_varlen_fwd(p, p, p, ctypes.c_void_p(p.value + 8), N.SAGE_DTYPE_F16, 2, 8, 8, 100, 100,
                                        60, 60, 128, p, p, s2, s2, s2, s2, 0, 0.0, None)
    assert rc == N.SAGE_ERR_INVALID_ARG and "aligned" in err()
