"""Register the B200 ``cuda`` variants in a TriBench checkout.

    python kernels/install_into_tribench.py /path/to/TriBench

For each pack here (sage_attn, flash_attn): copies ``cuda_impl.py`` into the checkout's
``kernels/<pack>/`` and merges ``meta_patch.json`` into its ``meta.json`` — the variant goes
under ``entrypoints.variants`` (tribench/meta.py:48, types.py:24-31; the CLI then runs it beside
the Triton implementation, tribench/cli.py:254-258) and the patch's cases are appended unless a
case of that name exists. The sage_attn patch adds the BASELINE shapes (h8k, c2, c3, c4) as
cases; the pack's own make_inputs (reference.py:4-13) draws q, k, v ~ N(0, 1) non-causal for
them, so through TriBench they are these configurations' shapes, not their distributions.
Running the variant needs ``tribench_b200`` importable (installed, or SAGE_B200_ROOT set to
this checkout). Re-running is idempotent.
"""
from __future__ import annotations

import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PACKS = ("sage_attn", "flash_attn")


def merge_meta(meta: dict, patch: dict) -> dict:
    """meta.json with patch's entrypoint variants and new cases merged in (in place)."""
    ep = meta.setdefault("entrypoints", {})
    ep.setdefault("variants", {}).update(patch.get("entrypoints", {}).get("variants", {}))
    names = {c.get("name") for c in meta.setdefault("cases", [])}
    for case in patch.get("cases", []):
        if case["name"] not in names:
            meta["cases"].append(dict(case))
            names.add(case["name"])
    return meta


def install(checkout: str) -> list[str]:
    """Install both packs' variants into `checkout`; returns the meta.json paths written."""
    written = []
    for pack in PACKS:
        dst = os.path.join(checkout, "kernels", pack)
        meta_path = os.path.join(dst, "meta.json")
        if not os.path.exists(meta_path):
            raise FileNotFoundError(f"{meta_path} not found: is {checkout} a TriBench checkout?")
        shutil.copyfile(os.path.join(HERE, pack, "cuda_impl.py"), os.path.join(dst, "cuda_impl.py"))
        with open(meta_path) as f:
            meta = json.load(f)
        with open(os.path.join(HERE, pack, "meta_patch.json")) as f:
            patch = json.load(f)
        with open(meta_path, "w") as f:
            json.dump(merge_meta(meta, patch), f, indent=4)
            f.write("\n")
        written.append(meta_path)
    return written


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    for path in install(sys.argv[1]):
        print("patched", path)
