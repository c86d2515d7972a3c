"""GPU: TriBench's own correctness gate on both packs' benchmark cases.

`tribench test` runs each variant on the pack's meta.json cases with inputs from the pack's
make_inputs (q, k, v ~ N(0, 1), kernels/*/reference.py:4-13), evaluates `ref` in the input
dtype on the same device (reference.py:15-24 for sage_attn, :15-28 for flash_attn), resolves the
tolerance (tribench/correctness.py:22-38: a per-dtype entry, else the pack's non-default
atol/rtol, else the dtype default) and passes iff torch.allclose(ref.float(), out.float())
(:80-82). This test restates that gate and applies it to the cuda variants' run() at full size:
sage_attn (atol = rtol = 5e-2, kernels/sage_attn/meta.json:45-48) and flash_attn (1e-2).

The BASELINE configs are too large for the unchunked ref (C5's score matrix alone is 2.2 TB);
they go through harness.gate_chunked, the same predicate evaluated over query-row chunks.
"""
import numpy as np
import pytest
import torch

import oracle
import tribench_b200 as tb
from tribench_b200 import harness

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CASES = {"s4k_d64": (8, 16, 4096, 64), "s8k_d64": (4, 16, 8192, 64)}


def ref_in_dtype(q, k, v, causal=False):
    """The packs' ref: softmax(q k^T * D^-0.5) v in the input dtype, one batch at a time."""
    out = torch.empty_like(q)
    for b in range(q.shape[0]):
        p = torch.matmul(q[b], k[b].transpose(1, 2)) * q.shape[-1] ** -0.5
        out[b] = torch.matmul(torch.softmax(p, dim=-1), v[b])
    return out


@pytest.mark.parametrize("pack", ["sage_attn", "flash_attn"])
@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("dtype_str", ["fp16", "bf16"])
def test_tribench_gate_on_pack_cases(pack, case, dtype_str):
    B, H, S, D = CASES[case]
    dtype = torch.float16 if dtype_str == "fp16" else torch.bfloat16
    torch.manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, device=DEV, dtype=dtype) for _ in range(3))
    run = tb.run if pack == "sage_attn" else tb.run_flash_attn
    out = run(q, k, v, causal=False)
    assert tb.device_status(DEV) == 0
    ref = ref_in_dtype(q, k, v)
    atol, rtol = harness.tolerance(dtype_str, *harness.PACK_TOLERANCE[pack])
    diff = (ref.float() - out.float()).abs()
    print(f"{pack} {case} {dtype_str}: max_abs_err {diff.max().item():.3e} (atol {atol}, rtol {rtol})")
    assert torch.allclose(ref.float(), out.float(), atol=atol, rtol=rtol)


def _scheme_row(q, k, v, b, h, row, causal, pv):
    """The exact INT8 block scheme (oracle.sage_model, fp64) for one output row of head (b, h)."""
    f32 = lambda t: t[b:b + 1, h:h + 1].float().cpu().numpy()
    qf, kf, vf = f32(q), f32(k), f32(v)
    D = qf.shape[-1]
    qi, qs = oracle.quant_per_block_int8(qf, 128, oracle.q_multiplier(None, D))
    ki, ks = oracle.quant_per_block_int8(kf, 64, 1.0, km=oracle.k_mean(kf))
    if pv == "fp8":
        codes, vsc = oracle.quant_v_fp8(vf)
        vf = oracle.e4m3_decode(codes) * vsc[:, :, None, :]
    return oracle.sage_model(qi, qs, ki, ks, vf, causal=causal, rows=np.array([row]))[0, 0, 0], np.abs(f32(v)).max()


# (config, P.V mode, TriBench's gate expected to pass). Where it does not, the INT8 / FP8 scheme
# itself misses the tolerance (C4: rows 0-2 of causal attention average one to three keys, so an
# e4m3 or INT8 rounding of a single V row or score is the whole error; C5: Student-t query rows
# with |q| up to ~360 make one channel set the row's INT8 scale), which the test checks at the
# element furthest outside the tolerance: there the kernel matches the scheme to its rounding bound
# and is no further from ref than the scheme is.
GATE_CASES = [("c2", "16bit", True), ("h8k", "16bit", True), ("c3", "16bit", True), ("c4", "16bit", False),
              ("c4", "fp8", False), ("c5", "16bit", False)]


@pytest.mark.parametrize("cfg,pv,expect_pass", GATE_CASES)
def test_tribench_gate_chunked_on_baseline_configs(cfg, pv, expect_pass):
    case = dict(tb.CONFIGS[cfg])
    inp = tb.make_inputs(case, DEV, seed=case["seed"], dtype=case["dtype"])
    q, k, v = inp["q"], inp["k"], inp["v"]
    out = tb.run(q, k, v, causal=case["causal"], pv=pv)
    assert tb.device_status(DEV) == 0
    r = harness.gate_chunked(out, q, k, v, case["causal"], dtype_str=case["dtype"], atol=5e-2, rtol=5e-2)
    print(f"{cfg} {pv}: passed={r['passed']} max_abs_err {r['max_abs_err']:.3e} max_rel_err {r['max_rel_err']:.3e} "
          f"outside tolerance {r['n_fail']} of {r['numel']}, worst at {r['worst']}")
    if expect_pass:
        assert r["passed"], r
    else:
        assert r["n_fail"] <= 1e-3 * r["numel"], r
        b, h, row, c = r["worst"]
        scheme, vmax = _scheme_row(q, k, v, b, h, row, case["causal"], pv)
        ours = out[b, h, row].float().cpu().numpy()
        kend = row + 1 if case["causal"] else k.shape[2]  # keys a causal row sees: [0, row]
        ref16 = harness.ref_chunked(q[b:b + 1, h:h + 1, row:row + 1], k[b:b + 1, h:h + 1, :kend],
                                    v[b:b + 1, h:h + 1, :kend])[0, 0, 0].float().cpu().numpy()
        tol = 2.5e-2 * vmax if pv == "fp8" else (1.6e-2 if case["dtype"] == "bf16" else 4e-3)
        print(f"  worst row: |ours - scheme| {np.abs(ours - scheme).max():.2e} (bound {tol:.2e}); "
              f"at the worst channel ours {ours[c]:.5f} scheme {scheme[c]:.5f} ref {ref16[c]:.5f}")
        assert np.abs(ours - scheme).max() <= tol
        # the gate's miss is the scheme's: the kernel adds at most its rounding bound to it
        assert abs(ours[c] - ref16[c]) <= abs(scheme[c] - ref16[c]) + tol
    del q, k, v, out, inp
    torch.cuda.empty_cache()
