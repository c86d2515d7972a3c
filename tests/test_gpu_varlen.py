"""GPU: packed variable-length batches (tribench_b200.varlen) against the dense path.

Every sequence of a packed batch is quantised and attended exactly as a dense batch of one
(Q blocks of 128 and K blocks of 64 rows from the sequence's first token, a per-sequence
smoothing mean), so the packed results must be BIT-IDENTICAL to the dense path run on each
sequence alone — codes, scales, means and outputs. The dense path is itself bit-exact against
the oracle (pinned to the reference's golden vectors) and within the written tolerances of it
in tests/test_gpu_parity.py; the packed quantisation is also checked against the oracle here.
"""
import numpy as np
import pytest
import torch

import oracle
import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)

# (query length, key length) per sequence: 1-row and empty sequences, block and tile edges
CROSS = [(1, 1), (128, 64), (129, 200), (300, 513), (0, 5), (777, 1000), (64, 1), (5, 0)]
SELF = [1, 128, 129, 300, 0, 777, 256, 63]


def _pack(lens, H, D, dtype, gen, offset=0.0):
    T = sum(lens)
    t = torch.randn(T, H, D, generator=gen, device=DEV)
    if offset:
        t = t + offset * torch.randn(1, H, D, generator=gen, device=DEV)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    return t.to(dtype), cu


def _case(pairs, Hq, Hkv, D, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q, cu_q = _pack([a for a, _ in pairs], Hq, D, dtype, g)
    k, cu_k = _pack([b for _, b in pairs], Hkv, D, dtype, g, offset=2.0)
    v, _ = _pack([b for _, b in pairs], Hkv, D, dtype, g)
    return q, k, v, cu_q, cu_k


def _dense(t, cu, i):
    """Sequence i of a packed tensor as a dense NHD batch of one ([1, L, H, D])."""
    return t[cu[i]:cu[i + 1]].unsqueeze(0)


@pytest.mark.parametrize("D,dtype,causal,pv,Hq,Hkv", [
    (128, torch.float16, False, "16bit", 4, 4),
    (64, torch.float16, True, "16bit", 4, 2),
    (128, torch.bfloat16, True, "fp8", 2, 2),
    (64, torch.bfloat16, False, "fp8", 4, 1),
    (64, torch.float16, False, "16bit", 2, 2),
])
def test_packed_attention_equals_dense_per_sequence(D, dtype, causal, pv, Hq, Hkv):
    pairs = [(n, n) for n in SELF] if causal else CROSS
    q, k, v, cu_q, cu_k = _case(pairs, Hq, Hkv, D, dtype, seed=D + Hq)
    cuq_t = torch.tensor(cu_q, dtype=torch.int32, device=DEV)
    cuk_t = torch.tensor(cu_k, dtype=torch.int32, device=DEV)
    o = tb.run_sage_attn_varlen(q, k, v, cuq_t, cuk_t, causal=causal, pv=pv)
    assert tb.device_status(DEV) == 0
    for i, (lq, lk) in enumerate(pairs):
        if lq == 0:
            continue
        oi = o[cu_q[i]:cu_q[i + 1]]
        if lk == 0:
            assert torch.all(oi == 0), f"sequence {i} has no keys: O must be 0"
            continue
        ref = tb.run(_dense(q, cu_q, i), _dense(k, cu_k, i), _dense(v, cu_k, i), causal=causal, pv=pv,
                     tensor_layout="NHD")[0]
        assert torch.equal(oi, ref), f"sequence {i} ({lq}, {lk}): packed differs from dense"


def test_packed_quantisation_bit_exact_vs_dense_and_oracle():
    D, Hq, Hkv = 128, 4, 2
    q, k, _, cu_q, cu_k = _case(CROSS, Hq, Hkv, D, torch.float16, seed=3)
    qi, qs, ki, ks, km = tb.per_block_int8_varlen(q, k, cu_q, cu_k, smooth_k=True, return_km=True)
    assert tb.device_status(DEV) == 0
    assert qi.shape == (Hq, q.shape[0], D) and ki.shape == (Hkv, k.shape[0], D)
    for i, (lq, lk) in enumerate(CROSS):
        if lq == 0 or lk == 0:
            continue
        dq, dqs, dk, dks, dkm = tb.per_block_int8(_dense(q, cu_q, i), _dense(k, cu_k, i), tensor_layout="NHD",
                                                  smooth_k=True, return_km=True)
        nq, nk = (lq + 127) // 128, (lk + 63) // 64
        assert torch.equal(qi[:, cu_q[i]:cu_q[i + 1]], dq[0]) and torch.equal(qs[i, :, :nq], dqs[0])
        assert torch.equal(ki[:, cu_k[i]:cu_k[i + 1]], dk[0]) and torch.equal(ks[i, :, :nk], dks[0])
        assert torch.equal(km[i], dkm[0])
        # and directly against the oracle (HND [1, H, L, D] float32 inputs)
        kf = _dense(k, cu_k, i).transpose(1, 2).float().cpu().numpy()
        qf = _dense(q, cu_q, i).transpose(1, 2).float().cpu().numpy()
        okm = oracle.k_mean(kf)
        oqi, oqs = oracle.quant_per_block_int8(qf, 128, oracle.q_multiplier(None, D))
        oki, oks = oracle.quant_per_block_int8(kf, 64, 1.0, km=okm)
        np.testing.assert_array_equal(qi[:, cu_q[i]:cu_q[i + 1]].cpu().numpy(), oqi[0])
        np.testing.assert_array_equal(qs[i, :, :nq].cpu().numpy(), oqs[0])
        np.testing.assert_array_equal(ki[:, cu_k[i]:cu_k[i + 1]].cpu().numpy(), oki[0])
        np.testing.assert_array_equal(ks[i, :, :nk].cpu().numpy(), oks[0])
        np.testing.assert_array_equal(km[i].cpu().numpy(), okm[0])


@pytest.mark.parametrize("D,causal", [(64, False), (128, True)])
def test_packed_flash_equals_dense_per_sequence(D, causal):
    pairs = [(n, n) for n in SELF] if causal else CROSS
    q, k, v, cu_q, cu_k = _case(pairs, 4, 2, D, torch.float16, seed=11 + D)
    o = tb.run_flash_attn_varlen(q, k, v, cu_q, cu_k, causal=causal)
    assert tb.device_status(DEV) == 0
    for i, (lq, lk) in enumerate(pairs):
        if lq == 0:
            continue
        oi = o[cu_q[i]:cu_q[i + 1]]
        if lk == 0:
            assert torch.all(oi == 0)
            continue
        ref = tb.run_flash_attn(_dense(q, cu_q, i), _dense(k, cu_k, i), _dense(v, cu_k, i), causal=causal,
                                tensor_layout="NHD")[0]
        assert torch.equal(oi, ref), f"sequence {i} ({lq}, {lk}): packed differs from dense"


def test_packed_head_major_views_and_out_buffer():
    """Packed tensors given as [H, T, D]-major storage (token stride D, head stride T*D)."""
    D, H = 64, 3
    q, k, v, cu_q, cu_k = _case(CROSS, H, H, D, torch.float16, seed=21)
    qh, kh, vh = (t.transpose(0, 1).contiguous().transpose(0, 1) for t in (q, k, v))
    out = torch.empty(H, q.shape[0], D, dtype=q.dtype, device=DEV).transpose(0, 1)
    o = tb.run_sage_attn_varlen(qh, kh, vh, cu_q, cu_k, out=out)
    assert o.data_ptr() == out.data_ptr()
    assert torch.equal(o, tb.run_sage_attn_varlen(q, k, v, cu_q, cu_k))
