"""GPU parity of the sm_100a path against the CPU oracle and the reference's golden vectors.

Quantisation: bit-exact (int8 codes, fp32 scales, fp32 K mean, e4m3 V codes).
Attention, tolerances written per test:
  * vs the exact block scheme (oracle.sage_model): the GPU only adds the rounding of P to the
    P.V operand type and the ex2 approximation — max-abs <= 4e-3 (fp16 output), 1.6e-2 (bf16
    output); FP8 P.V is measured relative to the V scale;
  * vs fp32 exact attention (the reference's ref): cos >= 0.999 and max-abs <= 2e-2 where the
    INT8 scheme itself meets that bound (all non-causal fixture cases); causal early rows are
    checked at <= 2.5e-2 (the scheme's own error there is ~2.2e-2).
"""
import numpy as np
import pytest
import torch

import oracle
import tribench_b200 as tb
from tribench_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def to_dev(a, dtype):
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).to(DEV, dtype)


def f32(t):
    return t.float().cpu().numpy()


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def dtype_of(golden, case):
    return torch.bfloat16 if golden(case, "meta")[0] else torch.float16


def no_timeout():
    assert tb.device_status(DEV) == 0


GOLD = ["c1s", "ragged", "bf16", "gqa", "causal", "ties", "zeroblk"]


# ----------------------------------------------------------------------------- quantisation
@pytest.mark.parametrize("case", GOLD)
def test_quant_matches_reference_golden(golden, case):
    dt = dtype_of(golden, case)
    q, k = to_dev(golden(case, "q"), dt), to_dev(golden(case, "k"), dt)
    qi, qs, ki, ks = tb.per_block_int8(q, k)
    no_timeout()
    np.testing.assert_array_equal(qi.cpu().numpy(), golden(case, "q_i8"))
    np.testing.assert_array_equal(qs.cpu().numpy(), golden(case, "q_scale"))
    np.testing.assert_array_equal(ki.cpu().numpy(), golden(case, "k_i8"))
    np.testing.assert_array_equal(ks.cpu().numpy(), golden(case, "k_scale"))


@pytest.mark.parametrize("case", GOLD)
def test_smoothing_matches_reference_km_path(golden, case):
    dt = dtype_of(golden, case)
    q, k = to_dev(golden(case, "q"), dt), to_dev(golden(case, "k"), dt)
    # device-computed mean
    _, _, ki, ks, km = tb.per_block_int8(q, k, smooth_k=True, return_km=True)
    no_timeout()
    np.testing.assert_array_equal(km.cpu().numpy(), golden(case, "km"))
    np.testing.assert_array_equal(ki.cpu().numpy(), golden(case, "k_i8_sm"))
    np.testing.assert_array_equal(ks.cpu().numpy(), golden(case, "k_scale_sm"))
    # caller-supplied km, the reference's own argument (broadcast [B, Hkv, 1, D])
    kmt = torch.as_tensor(golden(case, "km")).unsqueeze(2).to(DEV)
    _, _, ki2, ks2 = tb.per_block_int8(q, k, km=kmt)
    np.testing.assert_array_equal(ki2.cpu().numpy(), golden(case, "k_i8_sm"))
    np.testing.assert_array_equal(ks2.cpu().numpy(), golden(case, "k_scale_sm"))


def test_quant_nhd_layout(golden):
    q, k = to_dev(golden("c1s", "q"), torch.float16), to_dev(golden("c1s", "k"), torch.float16)
    qn, kn = q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous()  # [B, S, H, D]
    qi, qs, ki, ks = tb.per_block_int8(qn, kn, tensor_layout="NHD")
    np.testing.assert_array_equal(qi.cpu().numpy(), golden("c1s", "q_i8"))
    np.testing.assert_array_equal(ks.cpu().numpy(), golden("c1s", "k_scale"))
    np.testing.assert_array_equal(ki.cpu().numpy(), golden("c1s", "k_i8"))


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("D,S", [(128, 1000), (64, 1537), (128, 1)])
def test_quant_random_vs_oracle(dtype, D, S):
    case = dict(batch_size=2, num_heads=3, seq_len=S, head_dim=D, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=11, dtype=dtype)
    q, k = inp["q"], inp["k"]
    qi, qs, ki, ks, km = tb.per_block_int8(q, k, smooth_k=True, return_km=True, sm_scale=0.3)
    no_timeout()
    qf, kf = f32(q), f32(k)
    km_o = oracle.k_mean(kf)
    np.testing.assert_array_equal(km.cpu().numpy(), km_o)
    qi_o, qs_o = oracle.quant_per_block_int8(qf, 128, oracle.q_multiplier(0.3, D))
    ki_o, ks_o = oracle.quant_per_block_int8(kf, 64, 1.0, km=km_o)
    np.testing.assert_array_equal(qi.cpu().numpy(), qi_o)
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_o)
    np.testing.assert_array_equal(ki.cpu().numpy(), ki_o)
    np.testing.assert_array_equal(ks.cpu().numpy(), ks_o)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("D,S", [(64, 700), (128, 1024)])
def test_quant_v_fp8_vs_oracle(dtype, D, S):
    case = dict(batch_size=1, num_heads=2, seq_len=S, head_dim=D, dist="vchan", k_offset_std=2.0)
    v = tb.make_inputs(case, DEV, seed=3, dtype=dtype)["v"].clone()
    v[0, 1, :, 7] = 0  # all-zero channel
    v8, vs = tb.quant_v_fp8(v)
    no_timeout()
    c_o, s_o = oracle.quant_v_fp8(f32(v))
    np.testing.assert_array_equal(vs.cpu().numpy(), s_o)
    np.testing.assert_array_equal(v8.cpu().numpy(), c_o)


# ----------------------------------------------------------------------------- attention
def _model_for(q, k, v, causal, smooth, rows=None, heads=None, pv="16bit", sm_scale=None):
    """Oracle quantisation of the same inputs + the exact scheme output (fp64)."""
    qf, kf, vf = f32(q), f32(k), f32(v)
    D = qf.shape[-1]
    km = oracle.k_mean(kf) if smooth else None
    qi, qs = oracle.quant_per_block_int8(qf, 128, oracle.q_multiplier(sm_scale, D))
    ki, ks = oracle.quant_per_block_int8(kf, 64, 1.0, km=km)
    if pv == "fp8":
        codes, vsc = oracle.quant_v_fp8(vf)
        vf = oracle.e4m3_decode(codes) * vsc[:, :, None, :]
    return oracle.sage_model(qi, qs, ki, ks, vf, causal=causal, rows=rows, heads=heads)


@pytest.mark.parametrize("case", ["c1s", "ragged", "bf16", "gqa", "zeroblk"])
def test_attention_golden_noncausal(golden, case):
    dt = dtype_of(golden, case)
    q, k, v = (to_dev(golden(case, n), dt) for n in ("q", "k", "v"))
    o = tb.run(q, k, v, smooth_k=False)
    no_timeout()
    out = f32(o)
    model = _model_for(q, k, v, False, smooth=False)
    tol = 1.6e-2 if dt == torch.bfloat16 else 4e-3
    err_model = np.abs(out - model).max()
    err_tri = np.abs(out - golden(case, "o_triton").astype(np.float32)).max()
    print(f"{case}: vs model {err_model:.2e}, vs reference triton {err_tri:.2e}")
    assert err_model <= tol
    assert err_tri <= tol + 5e-3
    # smoothed (default) path against fp32 exact attention
    o2 = f32(tb.run(q, k, v))
    ref = golden(case, "o_ref")
    e, c = np.abs(o2 - ref).max(), cos(o2, ref)
    print(f"{case}: smoothed vs exact max-abs {e:.3e} cos {c:.6f}")
    assert c >= 0.999 and e <= 2e-2


def test_attention_golden_causal(golden):
    q, k, v = (to_dev(golden("causal", n), torch.float16) for n in ("q", "k", "v"))
    o = f32(tb.run(q, k, v, causal=True))
    no_timeout()
    model = _model_for(q, k, v, True, smooth=True)
    ref = golden("causal", "o_ref")
    e_m, e_r, c = np.abs(o - model).max(), np.abs(o - ref).max(), cos(o, ref)
    print(f"causal: vs model {e_m:.2e}; vs exact max-abs {e_r:.3e} cos {c:.6f}")
    assert e_m <= 4e-3
    assert c >= 0.999 and e_r <= 2.5e-2


@pytest.mark.parametrize("S", [1, 63, 64, 127, 128, 129, 255, 256, 257, 383, 640, 1000])
@pytest.mark.parametrize("D", [64, 128])
def test_attention_ragged_lengths(S, D):
    for causal in (False, True):
        case = dict(batch_size=2, num_heads=3, seq_len=S, head_dim=D, dist="offset", k_offset_std=2.0)
        inp = tb.make_inputs(case, DEV, seed=S + D, dtype="fp16")
        o = f32(tb.run(inp["q"], inp["k"], inp["v"], causal=causal))
        no_timeout()
        model = _model_for(inp["q"], inp["k"], inp["v"], causal, smooth=True)
        err = np.abs(o - model).max()
        assert np.isfinite(o).all() and err <= 4e-3, (S, D, causal, err)


def test_attention_nhd_layout_and_sm_scale():
    case = dict(batch_size=1, num_heads=4, seq_len=300, head_dim=128, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=2, dtype="fp16")
    q, k, v = inp["q"], inp["k"], inp["v"]
    o_hnd = tb.run(q, k, v, sm_scale=0.05)
    qn, kn, vn = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    o_nhd = tb.run(qn, kn, vn, sm_scale=0.05, tensor_layout="NHD")
    assert o_nhd.shape == qn.shape
    assert torch.equal(o_nhd.transpose(1, 2), o_hnd)
    model = _model_for(q, k, v, False, smooth=True, sm_scale=0.05)
    assert np.abs(f32(o_hnd) - model).max() <= 4e-3


def test_attention_gqa_groups():
    case = dict(batch_size=1, num_heads=8, seq_len=520, head_dim=64, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=9, dtype="bf16")
    q = inp["q"]
    k, v = inp["k"][:, :2].contiguous(), inp["v"][:, :2].contiguous()  # Hkv = 2, groups = 4
    o = f32(tb.run(q, k, v, causal=True))
    model = _model_for(q, k, v, True, smooth=True)
    assert np.abs(o - model).max() <= 1.6e-2


@pytest.mark.parametrize("D,dtype", [(64, "bf16"), (128, "fp16"), (64, "fp16"), (128, "bf16")])
def test_attention_fp8_pv(D, dtype):
    case = dict(batch_size=1, num_heads=2, seq_len=777, head_dim=D, dist="vchan", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=4, dtype=dtype)
    q, k, v = inp["q"], inp["k"], inp["v"]
    for causal in (False, True):
        o = f32(tb.run(q, k, v, causal=causal, pv="fp8"))
        no_timeout()
        model = _model_for(q, k, v, causal, smooth=True, pv="fp8")
        vmax = np.abs(f32(v)).max(axis=2, keepdims=True)  # per-channel V magnitude
        err = (np.abs(o - model) / vmax).max()
        ref = oracle.ref_attention(f32(q), f32(k), f32(v), causal=causal)
        print(f"fp8 D={D} {dtype} causal={causal}: |o-model|/|v|max {err:.3e}, cos vs exact {cos(o, ref):.6f}")
        # P in e4m3 (3-bit mantissa) on top of the exact scheme
        assert err <= 2.5e-2
        assert cos(o, ref) >= 0.998


def test_deterministic_and_plan_reuse():
    case = dict(batch_size=2, num_heads=4, seq_len=1024, head_dim=128, dist="offset", k_offset_std=2.0)
    inp = tb.make_inputs(case, DEV, seed=1, dtype="fp16")
    plan = tb.SagePlan(2, 4, 4, 1024, 1024, 128, torch.float16, DEV)
    a = plan.run(inp["q"], inp["k"], inp["v"])
    b = plan.run(inp["q"], inp["k"], inp["v"])
    c = tb.run(inp["q"], inp["k"], inp["v"])
    assert torch.equal(a, b) and torch.equal(a, c)


def test_errors_raise():
    q = torch.randn(1, 1, 64, 96, device=DEV, dtype=torch.float16)
    with pytest.raises(N.SageError) as ei:
        tb.run(q, q, q)
    assert ei.value.code == N.SAGE_ERR_INVALID_ARG
    q = torch.randn(1, 1, 64, 64, device=DEV, dtype=torch.float16)
    with pytest.raises(N.SageError):
        tb.run(q, q[:, :, :32], q[:, :, :32], causal=True)


def test_watchdog_times_out_cleanly_and_context_survives():
    bits = tb.watchdog_selftest(limit_us=2000)
    assert bits == 0x8  # SAGE_DEV_TIMEOUT_EPILOGUE
    assert tb.device_status(DEV) == 0  # cleared
    case = dict(batch_size=1, num_heads=1, seq_len=256, head_dim=64, dist="offset")
    inp = tb.make_inputs(case, DEV, seed=0, dtype="fp16")
    o = f32(tb.run(inp["q"], inp["k"], inp["v"]))
    assert np.isfinite(o).all()
    no_timeout()


# ----------------------------------------------------------------------------- full BASELINE sizes
def _sampled_check(cfg, heads, rows, tol_model, exact_bounds):
    case = dict(tb.CONFIGS[cfg])
    inp = tb.make_inputs(case, DEV, seed=case["seed"], dtype=case["dtype"])
    q, k, v = inp["q"], inp["k"], inp["v"]
    o = tb.run(q, k, v, causal=case["causal"], pv=case["pv"])
    no_timeout()
    H = case["num_heads"]
    worst = (0.0, 1.0, 0.0)
    for (b, h) in heads:
        hk = h  # no GQA in the BASELINE configs
        qh, kh, vh = (t[b:b + 1, hk:hk + 1] for t in (q, k, v))
        model = _model_for(qh, kh, vh, case["causal"], smooth=True, rows=rows, pv=case["pv"])[0, 0]
        out = f32(o[b, h])[rows]
        ref = oracle.ref_attention(f32(qh), f32(kh), f32(vh), causal=case["causal"], rows=rows)[0, 0]
        scale = np.abs(f32(vh)).max(axis=2)[0, 0] if case["pv"] == "fp8" else 1.0
        em = float((np.abs(out - model) / scale).max())
        worst = (max(worst[0], em), min(worst[1], cos(out, ref)), max(worst[2], float(np.abs(out - ref).max())))
    print(f"{cfg}: vs model {worst[0]:.2e}; vs exact cos {worst[1]:.6f} max-abs {worst[2]:.3e}")
    assert worst[0] <= tol_model
    min_cos, max_abs = exact_bounds
    assert worst[1] >= min_cos and worst[2] <= max_abs
    del q, k, v, o
    torch.cuda.empty_cache()


def test_config_c1_full():
    case = dict(tb.CONFIGS["c1"])
    inp = tb.make_inputs(case, DEV, seed=0, dtype="fp16")
    o = f32(tb.run(inp["q"], inp["k"], inp["v"]))
    ref = oracle.ref_attention(f32(inp["q"]), f32(inp["k"]), f32(inp["v"]))
    assert cos(o, ref) >= 0.999 and np.abs(o - ref).max() <= 2e-2


def test_config_c2_full_sampled():
    rows = np.r_[0:256, 2000:2128, 3968:4096]
    _sampled_check("c2", [(0, 0), (3, 31), (2, 17)], rows, 4e-3, (0.999, 2e-2))


def test_config_h8k_full_sampled():
    rows = np.r_[0:128, 4096:4224, 8064:8192]
    _sampled_check("h8k", [(0, 0), (1, 31)], rows, 4e-3, (0.999, 2e-2))


def test_config_c3_causal_full_sampled():
    rows = np.r_[0:256, 8100:8228, 16256:16384]
    # The INT8 block scheme itself (oracle.sage_model, no GPU rounding) reaches ~3.6e-2 on the
    # first causal rows, which average only a few keys; the GPU matches the scheme to < 1e-3.
    _sampled_check("c3", [(0, 0), (1, 31)], rows, 4e-3, (0.999, 5e-2))


def test_config_c4_fp8_causal_full_sampled():
    rows = np.r_[0:128, 4000:4128, 8064:8192]
    # FP8 P.V: error measured relative to each channel's |V| max; e4m3 V/P limit max-abs
    _sampled_check("c4", [(0, 0), (7, 15)], rows, 2.5e-2, (0.998, 0.5))


def test_config_c5_sampled_heads_one_per_shard():
    """C5 (S=32K causal, Student-t Q): one head from each 8-GPU shard of the 1024-head grid,
    generated alone (per-slab seeds give the same values a sharded run sees)."""
    case = dict(tb.CONFIGS["c5"])
    rows = np.r_[0:128, 16000:16128, 32640:32768]
    worst = (0.0, 1.0, 0.0)
    scheme = (1.0, 0.0)  # the INT8 block scheme's own cos / max-abs against exact attention
    for flat in (0, 130, 260, 390, 520, 650, 780, 1023):
        inp = tb.make_inputs(case, DEV, seed=case["seed"], dtype=case["dtype"], heads=(flat, flat + 1))
        q, k, v = inp["q"], inp["k"], inp["v"]
        out = f32(tb.run(q, k, v, causal=True))[0, 0][rows]
        no_timeout()
        model = _model_for(q, k, v, True, smooth=True, rows=rows)[0, 0]
        ref = oracle.ref_attention(f32(q), f32(k), f32(v), causal=True, rows=rows)[0, 0]
        worst = (max(worst[0], float(np.abs(out - model).max())), min(worst[1], cos(out, ref)),
                 max(worst[2], float(np.abs(out - ref).max())))
        scheme = (min(scheme[0], cos(model, ref)), max(scheme[1], float(np.abs(model - ref).max())))
    print(f"c5: vs model {worst[0]:.2e}; vs exact cos {worst[1]:.6f} max-abs {worst[2]:.3e}; "
          f"scheme vs exact cos {scheme[0]:.6f} max-abs {scheme[1]:.3e}")
    # The scheme itself misses cos 0.999 / max-abs 2e-2 on this heavy-tailed Q (INT8 scores of
    # outlier rows lose precision; up to ~0.17 on these heads), so the GPU is held to what it
    # adds: within 4e-3 of the scheme, and no further from exact than the scheme plus 5e-3.
    assert worst[0] <= 4e-3
    assert worst[1] >= scheme[0] - 1e-4 and worst[2] <= scheme[1] + 5e-3


def test_quant_full_size_c2_heads_bit_exact():
    """Full C2 tensors through the pre-pass (smoothing on); sampled heads bit-exact vs the oracle."""
    case = dict(tb.CONFIGS["c2"])
    inp = tb.make_inputs(case, DEV, seed=case["seed"], dtype="fp16")
    q, k = inp["q"], inp["k"]
    qi, qs, ki, ks, km = tb.per_block_int8(q, k, smooth_k=True, return_km=True)
    no_timeout()
    for b, h in [(0, 0), (1, 7), (3, 31)]:
        qf = f32(q[b:b + 1, h:h + 1])
        kf = f32(k[b:b + 1, h:h + 1])
        km_o = oracle.k_mean(kf)
        np.testing.assert_array_equal(km[b:b + 1, h:h + 1].cpu().numpy(), km_o)
        qi_o, qs_o = oracle.quant_per_block_int8(qf, 128, oracle.q_multiplier(None, 128))
        ki_o, ks_o = oracle.quant_per_block_int8(kf, 64, 1.0, km=km_o)
        np.testing.assert_array_equal(qi[b:b + 1, h:h + 1].cpu().numpy(), qi_o)
        np.testing.assert_array_equal(qs[b:b + 1, h:h + 1].cpu().numpy(), qs_o)
        np.testing.assert_array_equal(ki[b:b + 1, h:h + 1].cpu().numpy(), ki_o)
        np.testing.assert_array_equal(ks[b:b + 1, h:h + 1].cpu().numpy(), ks_o)


@pytest.mark.parametrize("Sq,Skv,D", [(300, 777, 128), (1000, 129, 64), (1, 2048, 64)])
def test_attention_cross_lengths(Sq, Skv, D):
    """seq_q != seq_kv (non-causal): every query attends to all seq_kv keys."""
    g = torch.Generator(device=DEV).manual_seed(Sq + Skv)
    q = torch.randn(1, 2, Sq, D, generator=g, device=DEV).half()
    k = (torch.randn(1, 2, Skv, D, generator=g, device=DEV) + 2.0 * torch.randn(1, 1, 1, D, generator=g, device=DEV)).half()
    v = torch.randn(1, 2, Skv, D, generator=g, device=DEV).half()
    o = f32(tb.run(q, k, v))
    no_timeout()
    model = _model_for(q, k, v, False, smooth=True)
    ref = oracle.ref_attention(f32(q), f32(k), f32(v))
    assert o.shape == (1, 2, Sq, D)
    assert np.abs(o - model).max() <= 4e-3
    assert cos(o, ref) >= 0.999
