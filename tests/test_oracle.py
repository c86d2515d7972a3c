"""CPU: the oracle against the reference's own golden vectors (tests/golden/sage_golden.npz).

Bit-exact for the quantisation (the reference's per_block_int8 run under TRITON_INTERPRET=1),
within stated tolerances for attention outputs.
"""
import numpy as np
import pytest

import oracle


def _f32(a):
    return np.asarray(a).astype(np.float32)


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


CASES = ["c1s", "ragged", "bf16", "gqa", "causal", "ties", "zeroblk"]


@pytest.mark.parametrize("case", CASES)
def test_quant_bit_exact_vs_reference(golden, case):
    q, k = _f32(golden(case, "q")), _f32(golden(case, "k"))
    qi, qs = oracle.quant_per_block_int8(q, 128, oracle.q_multiplier(None, q.shape[-1]))
    ki, ks = oracle.quant_per_block_int8(k, 64, 1.0)
    np.testing.assert_array_equal(qi, golden(case, "q_i8"))
    np.testing.assert_array_equal(qs, golden(case, "q_scale"))
    np.testing.assert_array_equal(ki, golden(case, "k_i8"))
    np.testing.assert_array_equal(ks, golden(case, "k_scale"))


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("blkq", [1, 16, 32, 64])
def test_fine_q_blocks_bit_exact_vs_reference(golden, case, blkq):
    """The reference's BLKQ argument (triton_impl.py:35, 57, 63): Q blocks of 64, 32, 16 rows and
    one row (per token) quantised by the reference itself equal the oracle bit for bit."""
    q = _f32(golden(case, "q"))
    qi, qs = oracle.quant_per_block_int8(q, blkq, oracle.q_multiplier(None, q.shape[-1]))
    assert qs.shape[-1] == -(-q.shape[2] // blkq)
    np.testing.assert_array_equal(qi, golden(case, f"q_i8_b{blkq}"))
    np.testing.assert_array_equal(qs, golden(case, f"q_scale_b{blkq}"))


@pytest.mark.parametrize("case", CASES)
def test_smoothed_quant_bit_exact_vs_reference_km(golden, case):
    """The reference's own smoothing path (per_block_int8(..., km=<fp32 km>)) equals the oracle."""
    k = _f32(golden(case, "k"))
    km = oracle.k_mean(k)
    np.testing.assert_array_equal(km, golden(case, "km"))
    ki, ks = oracle.quant_per_block_int8(k, 64, 1.0, km=km)
    np.testing.assert_array_equal(ki, golden(case, "k_i8_sm"))
    np.testing.assert_array_equal(ks, golden(case, "k_scale_sm"))


def test_k_mean_close_to_fp64_mean(golden):
    k = _f32(golden("c1s", "k"))
    km = oracle.k_mean(k)
    exact = k.astype(np.float64).mean(axis=2)
    np.testing.assert_allclose(km, exact, rtol=2 ** -23, atol=1e-7)


def test_k_mean_chunk_order_over_several_chunks():
    rng = np.random.default_rng(0)
    k = (rng.standard_normal((1, 2, 1500, 64)) + 3.0).astype(np.float16).astype(np.float32)
    km = oracle.k_mean(k)
    np.testing.assert_allclose(km, k.astype(np.float64).mean(axis=2), rtol=2 ** -22)


def test_ties_round_half_away_from_zero(golden):
    k = _f32(golden("ties", "k"))[0, 0]
    ks = golden("ties", "k_scale")
    assert ks.ravel()[0] == 1.0
    expect = (np.sign(k) * np.floor(np.abs(k) + 0.5)).astype(np.int8)
    np.testing.assert_array_equal(golden("ties", "k_i8")[0, 0], expect)


def test_zero_block_gives_zero_scale_and_codes(golden):
    assert golden("zeroblk", "q_scale")[0, 0, 0] == 0.0
    assert not golden("zeroblk", "q_i8")[0, 0, :128].any()


@pytest.mark.parametrize("case", CASES)
def test_ref_attention_matches_reference_ref(golden, case):
    q, k, v = (_f32(golden(case, n)) for n in ("q", "k", "v"))
    causal = bool(golden(case, "meta")[1])
    out = oracle.ref_attention(q, k, v, causal=causal)
    tol = 1e-4 if case == "ties" else 5e-6
    np.testing.assert_allclose(out, golden(case, "o_ref"), atol=tol, rtol=0)
    out_t = oracle.ref_attention_torch(q, k, v, causal=causal).numpy()
    np.testing.assert_allclose(out_t, golden(case, "o_ref"), atol=tol, rtol=0)


@pytest.mark.parametrize("case", ["c1s", "ragged", "bf16", "gqa", "zeroblk", "ties"])
def test_sage_model_matches_reference_triton(golden, case):
    """The exact evaluation of the block scheme vs the reference Triton kernel (which adds fp16
    P, per-block fp16 accumulation and, for bf16, a V cast to fp16)."""
    v = _f32(golden(case, "v"))
    m = oracle.sage_model(golden(case, "q_i8"), golden(case, "q_scale"), golden(case, "k_i8"),
                          golden(case, "k_scale"), v)
    tol = 5e-3 if case in ("bf16", "ties") else 1e-3
    np.testing.assert_allclose(m, _f32(golden(case, "o_triton")), atol=tol, rtol=0)


@pytest.mark.parametrize("case", ["c1s", "ragged", "bf16", "gqa", "causal", "zeroblk"])
def test_scheme_accuracy_vs_exact(golden, case):
    """North-star bound on the fixture cases: smoothed INT8 QK^T keeps cos >= 0.999 and
    max-abs <= 2e-2 against fp32 exact attention (C3-like causal rows are the tight one)."""
    q, k, v = (_f32(golden(case, n)) for n in ("q", "k", "v"))
    causal = bool(golden(case, "meta")[1])
    km = oracle.k_mean(k)
    ki, ks = oracle.quant_per_block_int8(k, 64, 1.0, km=km)
    m = oracle.sage_model(golden(case, "q_i8"), golden(case, "q_scale"), ki, ks, v, causal=causal)
    ref = golden(case, "o_ref")
    assert _cos(m, ref) >= 0.999
    assert np.abs(m - ref).max() <= (2.5e-2 if causal else 2e-2)


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    vals = oracle.e4m3_decode(codes)
    finite = ~np.isnan(vals)
    assert finite.sum() == 254  # 0x7F and 0xFF are NaN
    assert vals[0x7E] == 448.0 and vals[0x01] == 2.0 ** -9 and vals[0x08] == 2.0 ** -6
    enc = oracle.e4m3_encode(vals[finite])
    dec = oracle.e4m3_decode(enc)
    np.testing.assert_array_equal(dec, vals[finite])


def test_e4m3_round_to_nearest_even_and_saturate():
    pos = np.sort(oracle.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8)))
    mids = (pos[:-1].astype(np.float64) + pos[1:]) / 2
    enc = oracle.e4m3_encode(mids.astype(np.float32))
    # midpoints go to the neighbour with an even code
    lo = oracle.e4m3_encode(pos[:-1])
    hi = oracle.e4m3_encode(pos[1:])
    expect = np.where(lo % 2 == 0, lo, hi)
    np.testing.assert_array_equal(enc, expect)
    assert oracle.e4m3_encode(np.array([1e6, -500.0, 464.0], np.float32)).tolist() == [0x7E, 0xFE, 0x7E]


def test_quant_v_fp8_scales_and_codes():
    rng = np.random.default_rng(1)
    v = (rng.standard_normal((1, 2, 300, 64)) * rng.uniform(0.5, 4, (1, 2, 1, 64))).astype(np.float32)
    v[0, 1, :, 5] = 0.0  # an all-zero channel: scale 0, codes 0
    codes, sc = oracle.quant_v_fp8(v)
    np.testing.assert_array_equal(sc, (np.abs(v).max(axis=2) / np.float32(448.0)).astype(np.float32))
    assert not codes[0, 1, :, 5].any()
    deq = oracle.e4m3_decode(codes) * sc[:, :, None, :]
    rel = np.abs(deq - v) / np.maximum(np.abs(v), 1e-30)
    big = np.abs(v) > sc[:, :, None, :] * 2 ** -6 * 448  # normal e4m3 range
    assert rel[big].max() <= 2 ** -4 + 1e-6
