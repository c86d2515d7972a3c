"""The drop-in boundary exercised through TriBench itself.

A copy of an installed TriBench (its ``tribench`` package with the sage_attn and flash_attn packs
beside it, as in a checkout) gets the ``cuda`` variants installed by
kernels/install_into_tribench.py. Then, on the CPU, TriBench's own validation
(tribench/meta.py:92 validate_meta, :152 validate_entrypoints; registry.py:110 validate_all) and
loader (registry.py:92 load_variant) accept them; on the GPU, TriBench's CLI correctness gate
(``tribench test``, tribench/cli.py:205-347: make_inputs, ref in the input dtype, every
implementation, check_correctness with the pack's tolerance) passes for the variants on the
packs' cases and the added BASELINE shapes, fp16 and bf16.

The TriBench copy comes from baseline/_ref (the reference installed with pip --target, its kernel
packs next to the package) or from $TRIBENCH_REF; without either the tests skip.
"""
import importlib.util
import json
import os
import re
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKS = ("sage_attn", "flash_attn")


def _source():
    for cand in (os.environ.get("TRIBENCH_REF"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "tribench")) and all(
                os.path.isfile(os.path.join(cand, "kernels", p, "meta.json")) for p in PACKS):
            return cand
    return None


def _installer():
    spec = importlib.util.spec_from_file_location("install_into_tribench",
                                                  os.path.join(ROOT, "kernels", "install_into_tribench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def tribench_copy(tmp_path_factory):
    src = _source()
    if src is None:
        pytest.skip("no TriBench checkout: baseline/_ref (pip install --target) or $TRIBENCH_REF")
    dst = tmp_path_factory.mktemp("tribench")
    shutil.copytree(os.path.join(src, "tribench"), dst / "tribench")
    for pack in PACKS:
        shutil.copytree(os.path.join(src, "kernels", pack), dst / "kernels" / pack)
    _installer().install(str(dst))
    return dst


def _env(dst):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(dst), ROOT, env.get("PYTHONPATH", "")])
    env["SAGE_B200_ROOT"] = ROOT
    return env


def test_merge_meta_is_idempotent_and_keeps_existing_cases():
    inst = _installer()
    meta = {"entrypoints": {"triton": "t.py:f"}, "cases": [{"name": "s4k_d64", "seq_len": 4096}]}
    patch = {"entrypoints": {"variants": {"cuda": "cuda_impl.py:run"}},
             "cases": [{"name": "s4k_d64", "seq_len": 1}, {"name": "h8k", "seq_len": 8192}]}
    once = inst.merge_meta(json.loads(json.dumps(meta)), patch)
    twice = inst.merge_meta(json.loads(json.dumps(once)), patch)
    assert once == twice
    assert once["entrypoints"] == {"triton": "t.py:f", "variants": {"cuda": "cuda_impl.py:run"}}
    assert [c["name"] for c in once["cases"]] == ["s4k_d64", "h8k"] and once["cases"][0]["seq_len"] == 4096


def test_tribench_validates_and_loads_the_cuda_variants(tribench_copy):
    """TriBench's validate_meta / validate_entrypoints / validate_all report nothing, and its
    registry loads run(q, k, v, causal=False, sm_scale=None) for both packs (CPU only: the
    library is loaded lazily, no device is touched)."""
    code = r"""
import inspect, json, sys
from tribench.meta import load_meta, validate_meta, validate_entrypoints
from tribench.registry import KernelRegistry
kdir = sys.argv[1]
reg = KernelRegistry(kdir)
out = {"validate_all": reg.validate_all(), "packs": {}}
for pack in ("sage_attn", "flash_attn"):
    path = f"{kdir}/{pack}/meta.json"
    raw = json.load(open(path))
    meta = load_meta(path)
    fn = reg.load_variant(pack, "cuda")
    sig = inspect.signature(fn)
    out["packs"][pack] = {
        "errors": validate_meta(raw) + validate_entrypoints(meta),
        "variants": meta.entrypoints.variants,
        "cases": [c.name for c in meta.cases],
        "params": list(sig.parameters),
        "defaults": [repr(p.default) for p in sig.parameters.values()],
        "module": fn.__module__,
    }
print(json.dumps(out))
"""
    r = subprocess.run([sys.executable, "-c", code, str(tribench_copy / "kernels")], env=_env(tribench_copy),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["validate_all"] == {}
    for pack in PACKS:
        p = out["packs"][pack]
        assert p["errors"] == []
        assert p["variants"] == {"cuda": "cuda_impl.py:run"}
        assert p["params"] == ["q", "k", "v", "causal", "sm_scale"]
        assert p["defaults"][3:] == ["False", "None"]
        assert p["module"] == f"tribench.kernels.{pack}.cuda_impl"
    assert out["packs"]["sage_attn"]["cases"] == ["s4k_d64", "s8k_d64", "h8k", "c2", "c3", "c4"]


GATE_CASES = {"sage_attn": ["s4k_d64", "s8k_d64", "h8k", "c2"], "flash_attn": ["s4k_d64", "s8k_d64"]}


@pytest.mark.gpu
@pytest.mark.parametrize("pack", PACKS)
def test_tribench_cli_gate_passes_for_the_cuda_variant(tribench_copy, pack):
    """`tribench test` (tribench/cli.py:205-347) on the variant: every case x dtype PASSes
    TriBench's check_correctness against ref in the input dtype. (c3's and c4's ref would
    materialise 34 GB / 17 GB score matrices per dtype: they are checked by the chunked gate of
    test_gpu_tribench_gate.py instead.) The reference Triton implementation runs in the same
    gate; its lines are printed, not asserted."""
    cases = GATE_CASES[pack]
    cmd = [sys.executable, "-c", "import sys; from tribench.cli import main; sys.exit(main())", "test",
           "--kernel", pack, "--cases", ",".join(cases), "--dtype", "fp16,bf16", "--device", "cuda:0"]
    r = subprocess.run(cmd, env=_env(tribench_copy), cwd=str(tribench_copy), capture_output=True, text=True,
                       timeout=1200)
    print(r.stdout[-6000:])
    ours = re.findall(r"^\s+(PASS|FAIL)\s+(\S+) \[variant:cuda\] dtype=(\w+)", r.stdout, flags=re.M)
    assert len(ours) == 2 * len(cases), r.stdout[-3000:] + r.stderr[-3000:]
    assert all(status == "PASS" for status, _, _ in ours), ours
