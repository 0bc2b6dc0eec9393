"""alpaca_b200 — B200-native (sm_100a) attention hot path for alpaca.swift.

The product is the C-ABI library ``libalpaca_cuda.so`` (include/alpaca_cuda.h) with three attention paths —
tcgen05 causal flash prefill, split-KV decode + combine, and a general fp32 SIMT kernel — plus the fused RoPE +
KV-cache append that produces their input. This package holds its
sources (``csrc/``), its in-tree build (``build``) and a Python host mirror of alpaca's attention interface
(``ops``) used by the tests and the benchmark.
"""
from ._lib import (EXPORTED_SYMBOLS, FLAG_DEBUG_FORCE_TIMEOUT, FLAG_VARLEN, LIB_PATH, PROJ_ADD, PROJ_NORM, PROJ_SILU,
                   AlpacaCUDAError, AttnDesc, DType, Kernel, ProjDesc, RopeDesc, Status, WeightFormat, load)
from .ops import (KV_PADDING_ROWS, attention, attention_device, decode_project, decode_rope, device_status, launch,
                  make_desc, make_proj_desc, make_rope_desc, make_varlen_desc, prefill_varlen, project_launch, rope,
                  rope_kv_append, rope_launch, select_kernel, workspace_bytes)

__all__ = [
    "EXPORTED_SYMBOLS", "FLAG_DEBUG_FORCE_TIMEOUT", "LIB_PATH", "AlpacaCUDAError", "AttnDesc", "DType", "Kernel",
    "Status", "load", "KV_PADDING_ROWS", "attention", "attention_device", "device_status", "launch", "make_desc",
    "select_kernel", "workspace_bytes", "RopeDesc", "make_rope_desc", "rope", "rope_kv_append", "rope_launch",
    "decode_rope", "FLAG_VARLEN", "make_varlen_desc", "prefill_varlen", "ProjDesc", "WeightFormat", "PROJ_NORM",
    "PROJ_SILU", "PROJ_ADD", "make_proj_desc", "project_launch", "decode_project",
]
