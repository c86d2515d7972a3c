"""TriBench ``cuda`` variant of the flash_attn kernel pack.

Drop this file into TriBench's kernels/flash_attn/ next to meta.json and register it under
``entrypoints.variants`` (see meta_patch.json):

    "variants": {"cuda": "cuda_impl.py:run"}

TriBench's registry imports it by path (tribench/registry.py:62-75) and calls
``run(q, k, v, causal=False, sm_scale=None)`` with the tensors of the pack's make_inputs —
the signature of run_flash_attn (kernels/flash_attn/triton_impl.py:110) and ref
(kernels/flash_attn/reference.py:15). The work happens in libsage_sm100.so (sm_100a,
sage_flash_attn_fwd); there is no fallback, so a missing build or a non-B200 device raises.

The tribench_b200 package must be importable: install it, or point SAGE_B200_ROOT at its
checkout.
"""
import os
import sys

_root = os.environ.get("SAGE_B200_ROOT")
if _root and _root not in sys.path:
    sys.path.insert(0, _root)

from tribench_b200.flash_attn import run_flash_attn as _run  # noqa: E402


def run(q, k, v, causal=False, sm_scale=None):
    """Same arguments and result as run_flash_attn (triton_impl.py:110-128)."""
    return _run(q, k, v, causal=causal, sm_scale=sm_scale)
