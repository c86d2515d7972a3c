"""GPU parity of Q scale blocks finer than 128 rows: per_block_int8's BLKQ argument
(kernels/sage_attn/triton_impl.py:35, 57, 63) at 64, 32, 16 and 1 (one scale per token).

Quantisation: bit-exact against the reference's own codes (golden fixtures made by running its
per_block_int8 at each BLKQ) and against the oracle on random shapes, on every route that
quantises Q (the pre-pass, and the attention kernel's in-kernel quantisation whose codes are
dumped on request). Attention: every operand route is held to the exact block scheme at that
BLKQ (oracle.sage_model) with the same bounds as the 128-row scheme — max-abs <= 4e-3 (fp16
output), 1.6e-2 (bf16) — and the two INT8 routes (Q from the pre-pass / Q in the kernel) are
bit-identical. On BASELINE config 5 (Student-t Q) per-token scales bring the scheme, and the
GPU with it, to cos >= 0.999 against exact attention, which 128-row blocks miss.
"""
import numpy as np
import pytest
import torch

import oracle
import tribench_b200 as tb

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
FINE = [64, 32, 16, 1]
GOLD = ["c1s", "ragged", "bf16", "gqa", "causal", "ties", "zeroblk"]


def f32(t):
    return t.float().cpu().numpy()


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def no_timeout():
    assert tb.device_status(DEV) == 0


def model(q, k, v, causal, blkq, rows=None, smooth=True, sm_scale=None):
    """Oracle quantisation at Q blocks of `blkq` rows + the exact scheme output (fp64)."""
    qf, kf, vf = f32(q), f32(k), f32(v)
    D = qf.shape[-1]
    km = oracle.k_mean(kf) if smooth else None
    qi, qs = oracle.quant_per_block_int8(qf, blkq, oracle.q_multiplier(sm_scale, D))
    ki, ks = oracle.quant_per_block_int8(kf, 64, 1.0, km=km)
    return oracle.sage_model(qi, qs, ki, ks, vf, causal=causal, rows=rows, blkq=blkq)


@pytest.mark.parametrize("blkq", FINE)
@pytest.mark.parametrize("case", GOLD)
def test_quant_matches_reference_golden(golden, case, blkq):
    dt = torch.bfloat16 if golden(case, "meta")[0] else torch.float16
    q, k = (torch.as_tensor(golden(case, n).astype(np.float32)).to(DEV, dt) for n in ("q", "k"))
    qi, qs, ki, ks = tb.per_block_int8(q, k, BLKQ=blkq)
    no_timeout()
    np.testing.assert_array_equal(qi.cpu().numpy(), golden(case, f"q_i8_b{blkq}"))
    np.testing.assert_array_equal(qs.cpu().numpy(), golden(case, f"q_scale_b{blkq}"))
    # K is untouched by BLKQ
    np.testing.assert_array_equal(ki.cpu().numpy(), golden(case, "k_i8"))
    np.testing.assert_array_equal(ks.cpu().numpy(), golden(case, "k_scale"))


@pytest.mark.parametrize("blkq", FINE)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quant_random_vs_oracle(blkq, D, dtype):
    g = torch.Generator(device="cpu").manual_seed(blkq * 1000 + D)
    for S in (1, 100, 129, 300):
        q = (torch.randn((2, 3, S, D), generator=g) * 2.0).to(DEV, dtype)
        q[0, 1, S // 2] *= 40.0  # an outlier row
        k = torch.randn((2, 3, S, D), generator=g).to(DEV, dtype)
        qi, qs, _, _ = tb.per_block_int8(q, k, BLKQ=blkq, sm_scale=0.07)
        no_timeout()
        oqi, oqs = oracle.quant_per_block_int8(f32(q), blkq, oracle.q_multiplier(0.07, D))
        np.testing.assert_array_equal(qi.cpu().numpy(), oqi)
        np.testing.assert_array_equal(qs.cpu().numpy(), oqs)


@pytest.mark.parametrize("blkq", FINE)
def test_quant_nhd_layout(blkq):
    q = (torch.randn((1, 200, 4, 128)) * 3.0).to(DEV, torch.float16)  # [B, S, H, D]
    k = torch.randn((1, 200, 4, 128)).to(DEV, torch.float16)
    qi, qs, _, _ = tb.per_block_int8(q, k, BLKQ=blkq, tensor_layout="NHD")
    oqi, oqs = oracle.quant_per_block_int8(f32(q.transpose(1, 2)), blkq, oracle.q_multiplier(None, 128))
    np.testing.assert_array_equal(qi.cpu().numpy(), oqi)
    np.testing.assert_array_equal(qs.cpu().numpy(), oqs)


def _inputs(B, Hq, Hkv, S, D, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn((B, Hq, S, D), generator=g)
    q[:, :, ::37] *= 12.0  # outlier rows, where finer Q blocks matter
    k = torch.randn((B, Hkv, S, D), generator=g) + 2.0 * torch.randn((B, Hkv, 1, D), generator=g)
    v = torch.randn((B, Hkv, S, D), generator=g)
    return (t.to(DEV, dtype) for t in (q, k, v))


@pytest.mark.parametrize("blkq", FINE)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_routes_vs_scheme(blkq, D, causal):
    """Every operand route at this BLKQ against the exact scheme; the two INT8 routes (Q from
    the pre-pass, Q in the kernel) bit-identical, with the in-kernel codes and scales equal to
    the pre-pass's."""
    q, k, v = _inputs(2, 4, 2, 383, D, torch.float16, seed=blkq + D + int(causal))
    ref = model(q, k, v, causal, blkq)
    outs = {}
    for route in (["int8", "fused", "codes16"] if D == 64 else ["int8", "fused"]):
        fused = {"int8": False, "fused": True, "codes16": None}[route]
        plan = tb.SagePlan(2, 4, 2, 383, 383, D, torch.float16, DEV, causal=causal, fused_q=fused, blkq=blkq,
                           keep_q_int8=True)
        assert plan.route == route
        outs[route] = plan.run(q, k, v)
        no_timeout()
        err = float(np.abs(f32(outs[route]) - ref).max())
        print(f"blkq={blkq} D={D} causal={causal} {route}: vs scheme {err:.2e}")
        assert err <= 4e-3
        if route == "fused":
            qi, qs, _, _ = tb.per_block_int8(q, k, BLKQ=blkq)
            assert torch.equal(plan.quant.q_int8, qi) and torch.equal(plan.quant.q_scale, qs)
    assert torch.equal(outs["int8"], outs["fused"])


@pytest.mark.parametrize("blkq", [32, 1])
def test_attention_bf16_and_split_entry_points(blkq):
    """bf16 output, and the split calls (prepass + attention) equal to the one-call run."""
    q, k, v = _inputs(1, 2, 2, 640, 128, torch.bfloat16, seed=7)
    plan = tb.SagePlan(1, 2, 2, 640, 640, 128, torch.bfloat16, DEV, fused_q=False, blkq=blkq)
    o = plan.run(q, k, v)
    o2 = torch.empty_like(o)
    plan.prepass(q, k, v)
    plan.attention(v, o2)
    no_timeout()
    assert torch.equal(o, o2)
    err = float(np.abs(f32(o) - model(q, k, v, False, blkq)).max())
    assert err <= 1.6e-2


@pytest.mark.parametrize("blkq", [64, 16, 1])
def test_varlen_matches_dense_per_sequence(blkq):
    """Packed sequences: each sequence's Q codes, scales and output equal a dense call on it."""
    lens = [1, 130, 257, 64]
    cu = torch.tensor(np.r_[0, np.cumsum(lens)], dtype=torch.int32, device=DEV)
    T = sum(lens)
    g = torch.Generator(device="cpu").manual_seed(blkq)
    q = (torch.randn((T, 2, 128), generator=g) * 2.0).to(DEV, torch.float16)
    k = torch.randn((T, 2, 128), generator=g).to(DEV, torch.float16)
    v = torch.randn((T, 2, 128), generator=g).to(DEV, torch.float16)
    qi, qs, _, _ = tb.per_block_int8_varlen(q, k, cu, cu, BLKQ=blkq)
    o = tb.run_sage_attn_varlen(q, k, v, cu, cu, blkq=blkq)
    no_timeout()
    for i, L in enumerate(lens):
        a, b = int(cu[i]), int(cu[i + 1])
        dq, dk, dv = (t[a:b].transpose(0, 1).unsqueeze(0).contiguous() for t in (q, k, v))
        dqi, dqs, _, _ = tb.per_block_int8(dq, dk, BLKQ=blkq)
        nb = (L + blkq - 1) // blkq
        assert torch.equal(qi[:, a:b], dqi[0])
        assert torch.equal(qs[i, :, :nb], dqs[0])
        assert torch.equal(o[a:b].transpose(0, 1), tb.run(dq, dk, dv, blkq=blkq)[0])


def test_config_c5_per_token_sampled_heads():
    """BASELINE config 5 (S=32K causal, Q = 0.5 * Student-t(3)): with one Q scale per token the
    scheme meets cos >= 0.999 against exact attention on one head of each 8-GPU shard, and the
    GPU stays within 4e-3 of it. The 128-row scheme reaches only ~0.9989 on the same heads."""
    case = dict(tb.CONFIGS["c5"])
    rows = np.r_[0:128, 16000:16128, 32640:32768]
    worst = (0.0, 1.0, 0.0)
    for flat in (0, 130, 260, 390, 520, 650, 780, 1023):
        inp = tb.make_inputs(case, DEV, seed=case["seed"], dtype=case["dtype"], heads=(flat, flat + 1))
        q, k, v = inp["q"], inp["k"], inp["v"]
        out = f32(tb.run(q, k, v, causal=True, blkq=1))[0, 0][rows]
        no_timeout()
        sch = model(q, k, v, True, 1, rows=rows)[0, 0]
        ref = oracle.ref_attention(f32(q), f32(k), f32(v), causal=True, rows=rows)[0, 0]
        worst = (max(worst[0], float(np.abs(out - sch).max())), min(worst[1], cos(out, ref)),
                 max(worst[2], float(np.abs(out - ref).max())))
    print(f"c5 per-token: vs scheme {worst[0]:.2e}; vs exact cos {worst[1]:.6f} max-abs {worst[2]:.3e}")
    assert worst[0] <= 4e-3
    assert worst[1] >= 0.999


def test_config_c3_per_token_sampled():
    """BASELINE config 3 (S=16K causal) with one Q scale per token: the max-abs error against
    exact attention, measured and reported; the GPU within 4e-3 of the scheme."""
    case = dict(tb.CONFIGS["c3"])
    rows = np.r_[0:256, 8100:8228, 16256:16384]
    worst = (0.0, 1.0, 0.0, 0.0)
    for flat in (0, 63):
        inp = tb.make_inputs(case, DEV, seed=case["seed"], dtype=case["dtype"], heads=(flat, flat + 1))
        q, k, v = inp["q"], inp["k"], inp["v"]
        out = f32(tb.run(q, k, v, causal=True, blkq=1))[0, 0][rows]
        no_timeout()
        sch = model(q, k, v, True, 1, rows=rows)[0, 0]
        ref = oracle.ref_attention(f32(q), f32(k), f32(v), causal=True, rows=rows)[0, 0]
        worst = (max(worst[0], float(np.abs(out - sch).max())), min(worst[1], cos(out, ref)),
                 max(worst[2], float(np.abs(out - ref).max())), max(worst[3], float(np.abs(sch - ref).max())))
    print(f"c3 per-token: vs scheme {worst[0]:.2e}; vs exact cos {worst[1]:.6f} max-abs {worst[2]:.3e}; "
          f"scheme's own max-abs {worst[3]:.3e}")
    assert worst[0] <= 4e-3
    assert worst[1] >= 0.999 and worst[2] <= worst[3] + 5e-3
