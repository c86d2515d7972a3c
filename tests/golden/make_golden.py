"""Generate tests/golden/sage_golden.npz from the reference implementation itself.

Runs TriBench's own kernels/sage_attn code — ``per_block_int8`` and ``run_sage_attn`` from
triton_impl.py under ``TRITON_INTERPRET=1`` (CPU), and ``ref`` from reference.py in fp32 —
on small seeded inputs, and stores inputs and outputs as fixtures. It needs a TriBench
checkout (its path in $TRIBENCH_REF) and is run by hand where one exists; the tests read the
committed .npz and never import the reference.

    TRIBENCH_REF=/path/to/TriBench python tests/golden/make_golden.py

Cases (all [B, H, S, D], HND layout):
  c1s      B1 H2 S256 D64  fp16, k = N(0,1) + per-channel N(0,2^2) offset (exercises smoothing)
  ragged   B1 H1 S200 D128 fp16, S not a multiple of either block size
  bf16     B1 H2 S192 D64  bf16
  gqa      B1 Hq4 Hkv2 S128 D64 fp16 (num_kv_groups = 2, triton_impl.py:137)
  causal   B1 H1 S256 D64  fp16, causal=True (reference Triton ignores it; only `ref` is kept)
  ties     B1 H1 S64 D64   fp16 K block whose absmax is 127, so x/scale hits .5 exactly
  zeroblk  B1 H1 S192 D64  fp16 with the first 128-row Q block all zero (scale 0)
For every case the fixture holds q/k/v, the reference quantisation without smoothing
(q_i8, q_scale, k_i8, k_scale), the reference's Q quantisation with finer blocks through its
own BLKQ argument (q_i8_b{1,16,32,64}, q_scale_b{1,16,32,64}; triton_impl.py:35, 57, 63), the
smoothed K quantisation through the reference's own
``km`` argument with the oracle's fp32 channel mean (km, k_i8_sm, k_scale_sm), the reference
Triton output (o_triton, non-causal cases) and the fp32 exact output of ``ref`` (o_ref).
"""
from __future__ import annotations

import os
import sys

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("TRIBENCH_REF")
if not REF:
    sys.exit("set TRIBENCH_REF to a TriBench checkout")
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REF, "kernels", "sage_attn"))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import torch  # noqa: E402

import oracle  # noqa: E402
import reference as ref_mod  # noqa: E402  (kernels/sage_attn/reference.py)
import triton_impl  # noqa: E402  (kernels/sage_attn/triton_impl.py)


def offset_inputs(rng, B, Hq, Hkv, S, D, sigma=2.0):
    q = rng.standard_normal((B, Hq, S, D))
    c = rng.normal(0.0, sigma, size=(B, Hkv, 1, D))
    k = rng.standard_normal((B, Hkv, S, D)) + c
    v = rng.standard_normal((B, Hkv, S, D))
    return q, k, v


def run_case(name, q, k, v, dtype, causal=False):
    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16}[dtype]
    qt = torch.tensor(q, dtype=torch.float32).to(tdt)
    kt = torch.tensor(k, dtype=torch.float32).to(tdt)
    vt = torch.tensor(v, dtype=torch.float32).to(tdt)
    q_i8, q_scale, k_i8, k_scale = triton_impl.per_block_int8(qt, kt, BLKQ=128, BLKK=64)
    fine = {}
    for blkq in (1, 16, 32, 64):
        qb, qsb, _, _ = triton_impl.per_block_int8(qt, kt, BLKQ=blkq, BLKK=64)
        fine[f"q_i8_b{blkq}"], fine[f"q_scale_b{blkq}"] = qb.numpy(), qsb.numpy()
    km = oracle.k_mean(kt.float().numpy())  # [B, Hkv, D] fp32
    kmt = torch.tensor(km).unsqueeze(2)  # [B, Hkv, 1, D] fp32 -> k - km evaluated in fp32
    _, _, k_i8_sm, k_scale_sm = triton_impl.per_block_int8(qt, kt, km=kmt, BLKQ=128, BLKK=64)
    out = {
        "q": qt.float().numpy().astype(np.float16 if dtype == "fp16" else np.float32),
        "k": kt.float().numpy().astype(np.float16 if dtype == "fp16" else np.float32),
        "v": vt.float().numpy().astype(np.float16 if dtype == "fp16" else np.float32),
        "q_i8": q_i8.numpy(),
        "q_scale": q_scale.numpy(),
        "k_i8": k_i8.numpy(),
        "k_scale": k_scale.numpy(),
        "km": km,
        "k_i8_sm": k_i8_sm.numpy(),
        "k_scale_sm": k_scale_sm.numpy(),
        "meta": np.array([1 if dtype == "bf16" else 0, 1 if causal else 0], dtype=np.int32),
        **fine,
    }
    if not causal:
        o_tri = triton_impl.run_sage_attn(qt, kt, vt).float().numpy()
        out["o_triton"] = o_tri.astype(np.float16) if dtype == "fp16" else o_tri
    if qt.shape[1] == kt.shape[1]:
        out["o_ref"] = ref_mod.ref(qt.float(), kt.float(), vt.float(), causal=causal).numpy()
    else:
        g = qt.shape[1] // kt.shape[1]
        out["o_ref"] = ref_mod.ref(qt.float(), kt.float().repeat_interleave(g, 1),
                                   vt.float().repeat_interleave(g, 1), causal=causal).numpy()
    return {f"{name}/{k2}": v2 for k2, v2 in out.items()}


def main():
    fixtures = {}
    rng = np.random.default_rng(20261201)
    fixtures.update(run_case("c1s", *offset_inputs(rng, 1, 2, 2, 256, 64), "fp16"))
    fixtures.update(run_case("ragged", *offset_inputs(rng, 1, 1, 1, 200, 128), "fp16"))
    fixtures.update(run_case("bf16", *offset_inputs(rng, 1, 2, 2, 192, 64), "bf16"))
    fixtures.update(run_case("gqa", *offset_inputs(rng, 1, 4, 2, 128, 64), "fp16"))
    fixtures.update(run_case("causal", *offset_inputs(rng, 1, 1, 1, 256, 64), "fp16", causal=True))
    # ties: a K block of half-integers with absmax 127 -> k_scale == 1 and y = x exactly.
    q, _, v = offset_inputs(rng, 1, 1, 1, 64, 64)
    halves = (rng.integers(-127, 127, size=(1, 1, 64, 64)) + 0.5).astype(np.float64)
    halves[0, 0, 0, 0] = 127.0
    fixtures.update(run_case("ties", q, halves, v, "fp16"))
    # zeroblk: first Q block all zero -> reference scale 0 (0/0 -> NaN -> int8 0).
    q, k, v = offset_inputs(rng, 1, 1, 1, 192, 64)
    q[:, :, :128, :] = 0.0
    fixtures.update(run_case("zeroblk", q, k, v, "fp16"))
    path = os.path.join(HERE, "sage_golden.npz")
    np.savez_compressed(path, **fixtures)
    print(f"wrote {path}: {len(fixtures)} arrays, {os.path.getsize(path) / 1e3:.1f} kB")


if __name__ == "__main__":
    main()
