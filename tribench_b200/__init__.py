"""tribench_b200 — B200-native (sm_100a) implementation of TriBench's sage_attn path.

Public API (mirrors kernels/sage_attn/triton_impl.py and reference.py):
  run / run_sage_attn(q, k, v, causal=False, sm_scale=None, *, pv="16bit", smooth_k=True, blkq=128)
  per_block_int8(q, k, km=None, BLKQ=128, BLKK=64, sm_scale=None, tensor_layout="HND")
    (BLKQ / blkq: query rows per Q scale, 128, 64, 32, 16 or 1)
  quant_v_fp8(v), attn_fwd(quant, v, causal), SagePlan (preallocated repeated calls; cuda_graph()
  captures one call for single-launch replay)
  HostPipeline (host q/k/v -> host output, PCIe copies overlapped with the computation)
  make_inputs(case, device, seed, dtype), estimate(case)
  flash_attn.run_flash_attn(q, k, v, causal=False, sm_scale=None): the flash_attn pack (fp16/bf16 QK^T)
  varlen.run_sage_attn_varlen / per_block_int8_varlen / run_flash_attn_varlen: packed
  variable-length batches (q [total_q, H, D] + cu_seqlens)
  harness.ref_chunked / gate_chunked: TriBench's correctness gate for cases too large for ref
"""
from . import flash_attn, harness, varlen
from .flash_attn import run_flash_attn
from .inputs import CONFIGS, estimate, make_inputs, prepass_bytes
from .sage_attn import (HostPipeline, SageGraph, SagePlan, SageQuant, attn_fwd, device_status, per_block_int8,
                        quant_v_fp8, run, run_sage_attn, watchdog_selftest, workspace_bytes)
from .varlen import per_block_int8_varlen, run_flash_attn_varlen, run_sage_attn_varlen

__all__ = [
    "CONFIGS", "estimate", "make_inputs", "prepass_bytes", "HostPipeline", "SageGraph", "SagePlan", "SageQuant", "attn_fwd", "device_status",
    "per_block_int8", "quant_v_fp8", "run", "run_sage_attn", "watchdog_selftest", "workspace_bytes",
    "flash_attn", "run_flash_attn", "harness", "varlen", "per_block_int8_varlen", "run_flash_attn_varlen",
    "run_sage_attn_varlen",
]
