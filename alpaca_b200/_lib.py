"""ctypes bindings of libalpaca_cuda.so (the C ABI declared in include/alpaca_cuda.h).

The shared library is built in-tree by ``alpaca_b200.build``. There is no fallback: if the library is missing or
cannot be loaded, importing the bindings raises.
"""
from __future__ import annotations

import ctypes
from enum import IntEnum
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libalpaca_cuda.so"


class Status(IntEnum):
    OK = 0
    INVALID_ARGUMENT = 1
    UNSUPPORTED = 2
    WORKSPACE_TOO_SMALL = 3
    LAUNCH_FAILED = 4
    DEVICE_TIMEOUT = 5
    CUDA_ERROR = 6


class DType(IntEnum):
    F32 = 0
    F16 = 1


class Kernel(IntEnum):
    AUTO = 0
    DECODE_SPLIT = 1
    PREFILL_TC = 2
    GENERAL = 3


FLAG_DEBUG_FORCE_TIMEOUT = 1 << 31
FLAG_VARLEN = 1 << 0


class AttnDesc(ctypes.Structure):
    """alpaca_attn_desc (include/alpaca_cuda.h)."""
    _fields_ = [
        ("n_seqs", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("start_position", ctypes.c_int32),
        ("ctx_lens", ctypes.c_void_p),
        ("max_ctx_len", ctypes.c_int32),
        ("q_dtype", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("q_token_stride", ctypes.c_int64),
        ("q_seq_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("kv_row_stride", ctypes.c_int64),
        ("kv_seq_stride", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("out_token_stride", ctypes.c_int64),
        ("out_seq_stride", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("block_table", ctypes.c_void_p),
        ("block_rows", ctypes.c_int32),
        ("max_blocks", ctypes.c_int32),
        ("block_stride", ctypes.c_int64),
        ("pool_blocks", ctypes.c_int32),
        ("reserved1", ctypes.c_int32),
        ("q_offsets", ctypes.c_void_p),
        ("start_positions", ctypes.c_void_p),
        ("total_tokens", ctypes.c_int32),
        ("reserved2", ctypes.c_int32),
    ]


class RopeDesc(ctypes.Structure):
    """alpaca_rope_desc (include/alpaca_cuda.h)."""
    _fields_ = [
        ("n_seqs", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("start_position", ctypes.c_int32),
        ("positions", ctypes.c_void_p),
        ("theta", ctypes.c_float),
        ("interleaved", ctypes.c_int32),
        ("q_dtype", ctypes.c_int32),
        ("cache_dtype", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("q_token_stride", ctypes.c_int64),
        ("q_seq_stride", ctypes.c_int64),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("kv_token_stride", ctypes.c_int64),
        ("kv_seq_stride", ctypes.c_int64),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("cache_row_stride", ctypes.c_int64),
        ("cache_seq_stride", ctypes.c_int64),
        ("flags", ctypes.c_uint32),
        ("block_table", ctypes.c_void_p),
        ("block_rows", ctypes.c_int32),
        ("max_blocks", ctypes.c_int32),
        ("block_stride", ctypes.c_int64),
        ("pool_blocks", ctypes.c_int32),
        ("cache_rows", ctypes.c_int32),
    ]


class ProjDesc(ctypes.Structure):
    """alpaca_proj_desc (include/alpaca_cuda.h)."""
    _fields_ = [
        ("n_tokens", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("rows", ctypes.c_int32 * 3),
        ("format", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("eps", ctypes.c_float),
        ("w", ctypes.c_void_p * 3),
        ("x", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64),
        ("norm_weight", ctypes.c_void_p),
        ("y", ctypes.c_void_p * 3),
        ("y_stride", ctypes.c_int64 * 3),
    ]


class WeightFormat(IntEnum):
    F16 = 0
    Q8_0 = 1
    Q4_0 = 2


PROJ_NORM, PROJ_SILU, PROJ_ADD = 1, 2, 4

EXPORTED_SYMBOLS = (
    "alpaca_attention",
    "alpaca_attn_prefill",
    "alpaca_attn_decode",
    "alpaca_attn_decode_noalloc",
    "alpaca_attn_decode_rope",
    "alpaca_attention_workspace_bytes",
    "alpaca_attention_select",
    "alpaca_cuda_device_status",
    "alpaca_cuda_status_string",
    "alpaca_cuda_last_error",
    "alpaca_cuda_version",
    "alpaca_rope_kv_append",
    "alpaca_decode_project",
)

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run `python -m alpaca_b200.build` (needs nvcc)")
    L = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.POINTER(AttnDesc)
    for name in ("alpaca_attn_prefill", "alpaca_attn_decode"):
        f = getattr(L, name)
        f.restype = ctypes.c_int
        f.argtypes = [P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.alpaca_attn_decode_noalloc.restype = ctypes.c_int
    L.alpaca_attn_decode_noalloc.argtypes = [P, ctypes.c_void_p]
    L.alpaca_attention.restype = ctypes.c_int
    L.alpaca_attention.argtypes = [P, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.alpaca_attention_workspace_bytes.restype = ctypes.c_int
    L.alpaca_attention_workspace_bytes.argtypes = [P, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t)]
    L.alpaca_attention_select.restype = ctypes.c_int
    L.alpaca_attention_select.argtypes = [P, ctypes.POINTER(ctypes.c_int)]
    L.alpaca_cuda_device_status.restype = ctypes.c_int
    L.alpaca_cuda_device_status.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.alpaca_cuda_status_string.restype = ctypes.c_char_p
    L.alpaca_cuda_status_string.argtypes = [ctypes.c_int]
    L.alpaca_cuda_last_error.restype = ctypes.c_char_p
    L.alpaca_cuda_last_error.argtypes = []
    L.alpaca_cuda_version.restype = ctypes.c_int
    L.alpaca_cuda_version.argtypes = []
    L.alpaca_rope_kv_append.restype = ctypes.c_int
    L.alpaca_rope_kv_append.argtypes = [ctypes.POINTER(RopeDesc), ctypes.c_void_p]
    L.alpaca_decode_project.restype = ctypes.c_int
    L.alpaca_decode_project.argtypes = [ctypes.POINTER(ProjDesc), ctypes.c_void_p]
    L.alpaca_attn_decode_rope.restype = ctypes.c_int
    L.alpaca_attn_decode_rope.argtypes = [P, ctypes.POINTER(RopeDesc), ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.c_void_p]
    _lib = L
    return L


class AlpacaCUDAError(RuntimeError):
    """A non-OK alpaca_cuda_status, mirroring alpaca.swift's MetalError (MetalContext.swift:7-31)."""

    def __init__(self, status: int, message: str = ""):
        self.status = Status(status)
        L = load()
        text = L.alpaca_cuda_status_string(int(status)).decode()
        super().__init__(f"{text}: {message}" if message else text)


def check(status: int) -> None:
    if status != Status.OK:
        raise AlpacaCUDAError(status, load().alpaca_cuda_last_error().decode())
