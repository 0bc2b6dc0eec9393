"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

ctypes bindings of ``oracle/liboracle.so`` (the C restatement of alpaca.swift's
``CPUOps.attentionScores / softmax / attentionApply``, Sources/AlpacaCore/Operations/CPUOps.swift:162-274, and of
``CPUOps.rope``, CPUOps.swift:184-210, composed into the RoPE + KV-cache append of decode_fused.metal:126-154).
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this module, as the
checker. The product package ``alpaca_b200`` never imports it.

Parity of this oracle is pinned against the reference's own known-answer fixture
(Tests/AlpacaCoreTests/Fixtures/ops.json["attention"] and ["rope"], committed as tests/golden/attention_kat.json
and tests/golden/rope_kat.json).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, no fast-math, no FMA contraction)."""
    srcs = [_HERE / n for n in ("cpu_attention.c", "cpu_attention.h", "cpu_rope.c", "cpu_rope.h", "cpu_proj.c",
                                "cpu_proj.h")]
    if force or not _LIB_PATH.exists() or any(_LIB_PATH.stat().st_mtime < p.stat().st_mtime for p in srcs):
        subprocess.run(["make", "-s", "-C", str(_HERE), "liboracle.so"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        L.oracle_f16_round.restype = ctypes.c_float
        L.oracle_f16_round.argtypes = [ctypes.c_float]
        L.oracle_f16_round_array.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.oracle_attention_scores.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 6 + [_f32p]
        L.oracle_softmax.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int]
        L.oracle_attention_apply.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 5 + [_f32p]
        L.oracle_attention.argtypes = ([_f32p, _f32p, _f32p] + [ctypes.c_int] * 6 +
                                       [ctypes.c_float, _f32p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64])
        L.oracle_attention_strided.argtypes = ([_f32p, ctypes.c_int64, _f32p, _f32p, ctypes.c_int64] +
                                               [ctypes.c_int] * 6 +
                                               [ctypes.c_float, _f32p, ctypes.c_int64, ctypes.c_int,
                                                ctypes.c_int64, ctypes.c_int64])
        L.oracle_attention_rows.argtypes = ([_f32p, ctypes.c_int64, _f32p, _f32p, ctypes.c_int64] +
                                            [ctypes.c_int] * 6 +
                                            [ctypes.c_float, _f32p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64),
                                             ctypes.c_int64, ctypes.c_int])
        L.oracle_error_metrics.argtypes = [_f32p, _f64p, ctypes.c_int64, _f64p]
        L.oracle_error_metrics_f32.argtypes = [_f32p, _f32p, ctypes.c_int64, _f64p]
        L.oracle_splitmix_uniform.argtypes = [ctypes.c_uint64, ctypes.c_float, _f32p, ctypes.c_int64]
        L.oracle_splitmix_normal.argtypes = [ctypes.c_uint64, _f32p, ctypes.c_int64]
        L.oracle_rope.argtypes = [_f32p] + [ctypes.c_int] * 4 + [ctypes.c_double, ctypes.c_int]
        L.oracle_rope_kv_append.argtypes = ([_f32p, _f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 5 +
                                            [ctypes.c_double, ctypes.c_int, ctypes.c_int])
        L.oracle_row_bytes.restype = ctypes.c_int64
        L.oracle_row_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.oracle_row_dot.restype = ctypes.c_float
        L.oracle_row_dot.argtypes = [ctypes.c_int, ctypes.c_void_p, _f32p, ctypes.c_int]
        L.oracle_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, _f32p]
        L.oracle_silu.restype = ctypes.c_float
        L.oracle_silu.argtypes = [ctypes.c_float]
        L.oracle_dequantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, _f32p]
        L.oracle_quantize.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_void_p]
        L.oracle_decode_project.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_uint,
                                            ctypes.c_float, ctypes.POINTER(ctypes.c_void_p), _f32p, ctypes.c_int,
                                            ctypes.c_int64, _f32p, ctypes.POINTER(ctypes.c_void_p),
                                            ctypes.POINTER(ctypes.c_int64)]
        _lib = L
    return _lib


def _p32(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def f16_round(x: np.ndarray) -> np.ndarray:
    """f32 -> binary16 (round to nearest even) -> f32, as Tensor.converted(to: .float16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_f16_round_array(_p32(x), _p32(out), x.size)
    return out


def attention_scores(q, keys, length: int, start: int) -> np.ndarray:
    """CPUOps.attentionScores (CPUOps.swift:222-249): [H, T, length] with -inf where masked."""
    q = np.ascontiguousarray(q, np.float32)
    keys = np.ascontiguousarray(keys, np.float32)
    T, H, d = q.shape
    kvh = keys.shape[1]
    if keys.ndim != 3 or keys.shape[2] != d or H % kvh != 0:
        raise ValueError(f"attentionScores: q {q.shape}, keys {keys.shape}")
    if not (0 <= length <= keys.shape[0] and start + T <= length):
        raise ValueError(f"attention length {length}, start {start}, tokens {T}, capacity {keys.shape[0]}")
    s = np.empty((H, T, length), np.float32)
    lib().oracle_attention_scores(_p32(q), _p32(keys), T, H, kvh, d, length, start, _p32(s))
    return s


def softmax(x) -> np.ndarray:
    """CPUOps.softmax (CPUOps.swift:162-175) over the last dimension."""
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    n = x.shape[-1]
    lib().oracle_softmax(_p32(x), x.size // n, n)
    return x


def attention_apply(probs, values) -> np.ndarray:
    """CPUOps.attentionApply (CPUOps.swift:252-274): [T, H, d]."""
    probs = np.ascontiguousarray(probs, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    H, T, L = probs.shape
    kvh, d = values.shape[1], values.shape[2]
    out = np.empty((T, H, d), np.float32)
    lib().oracle_attention_apply(_p32(probs), _p32(values), H, T, L, kvh, d, _p32(out))
    return out


def attention(q, keys, values, start: int, length: int | None = None, scale: float = 0.0, threads: int = 1,
              rows: tuple[int, int] | None = None, out: np.ndarray | None = None) -> np.ndarray:
    """Fused row-by-row CPU attention, bit-identical to scores -> softmax -> apply.

    q [T,H,d]; keys/values [capacity,Hkv,d] (first `length` rows read, default start+T). `rows` restricts the
    computation to rows h*T+t in [rows[0], rows[1]) (others stay as in `out`, default zeros)."""
    q = np.ascontiguousarray(q, np.float32)
    keys = np.ascontiguousarray(keys, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    T, H, d = q.shape
    kvh = keys.shape[1]
    if length is None:
        length = start + T
    if not (keys.shape == values.shape and keys.shape[2] == d and H % kvh == 0):
        raise ValueError(f"attention shapes q {q.shape} k {keys.shape} v {values.shape}")
    if not (0 <= length <= keys.shape[0] and start + T <= length):
        raise ValueError(f"attention length {length}, start {start}, tokens {T}, capacity {keys.shape[0]}")
    if out is None:
        out = np.zeros((T, H, d), np.float32)
    r0, r1 = rows if rows is not None else (0, H * T)
    lib().oracle_attention(_p32(q), _p32(keys), _p32(values), T, H, kvh, d, length, start, float(scale),
                           _p32(out), int(threads), int(r0), int(r1))
    return out


def attention_rows(q, keys, values, start: int, rows, length: int | None = None, scale: float = 0.0,
                   threads: int | None = None, out: np.ndarray | None = None) -> np.ndarray:
    """oracle attention evaluated only on the listed rows (row = h*T + t), all host threads by default."""
    q = np.ascontiguousarray(q, np.float32)
    keys = np.ascontiguousarray(keys, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    T, H, d = q.shape
    kvh = keys.shape[1]
    if length is None:
        length = start + T
    if not (keys.shape == values.shape and keys.shape[2] == d and H % kvh == 0):
        raise ValueError(f"attention shapes q {q.shape} k {keys.shape} v {values.shape}")
    if not (0 <= length <= keys.shape[0] and start + T <= length):
        raise ValueError(f"attention length {length}, start {start}, tokens {T}, capacity {keys.shape[0]}")
    if out is None:
        out = np.zeros((T, H, d), np.float32)
    r = np.ascontiguousarray(rows, np.int64)
    lib().oracle_attention_rows(_p32(q), H * d, _p32(keys), _p32(values), kvh * d, T, H, kvh, d, length, start,
                                float(scale), _p32(out), H * d, r.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                r.size, int(threads or host_threads()))
    return out


def rope(x, start: int, theta: float, interleaved: bool = True) -> np.ndarray:
    """CPUOps.rope (CPUOps.swift:184-210) of x [tokens, heads, head_dim]; returns a rotated copy. theta is taken
    as a Float first, as the reference's `theta: Float` parameter is."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    T, H, D = y.shape
    lib().oracle_rope(_p32(y), T, H, D, int(start), float(np.float32(theta)), int(bool(interleaved)))
    return y


def rope_kv_append(q, k, v, k_cache, v_cache, start: int, theta: float, interleaved: bool = True,
                   cache_f16: bool = True):
    """One sequence of the fused step (decode_fused.metal:126-154 on the CPU path). q [T, H, d] is returned
    rotated; k_cache / v_cache [rows, Hkv, d] (f32 arrays) are returned with rows start..start+T-1 written
    (rotated k and raw v, binary16-rounded when cache_f16). Inputs are not modified."""
    q = np.ascontiguousarray(q, dtype=np.float32).copy()
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    kc = np.ascontiguousarray(k_cache, dtype=np.float32).copy()
    vc = np.ascontiguousarray(v_cache, dtype=np.float32).copy()
    T, H, D = q.shape
    Hkv = k.shape[1]
    assert kc.shape[0] >= start + T and kc.shape[1:] == (Hkv, D) and vc.shape == kc.shape
    lib().oracle_rope_kv_append(_p32(q), _p32(k), _p32(v), _p32(kc), _p32(vc), T, H, Hkv, D, int(start),
                                float(np.float32(theta)), int(bool(interleaved)), int(bool(cache_f16)))
    return q, kc, vc


# ---------------------------------------------------------------------------------------------- projections

WEIGHT_FORMATS = {"f16": 0, "q8_0": 1, "q4_0": 2, "f32": 3}


def row_bytes(fmt: str, k: int) -> int:
    return int(lib().oracle_row_bytes(WEIGHT_FORMATS[fmt], k))


def quantize(values, fmt: str) -> np.ndarray:
    """quantize() (Quantization.swift:39-73): f32 values (a multiple of 32, row-major [n, k]) -> GGUF blocks (uint8)."""
    v = np.ascontiguousarray(values, np.float32)
    k = v.shape[-1]
    n = v.size // k
    if fmt == "f16":
        return np.frombuffer(f16_round(v).astype(np.float16).tobytes(), np.uint8).reshape(n, 2 * k).copy()
    out = np.zeros(n * row_bytes(fmt, k), np.uint8)
    lib().oracle_quantize(WEIGHT_FORMATS[fmt], _p32(v), v.size, out.ctypes.data)
    return out.reshape(n, row_bytes(fmt, k))


def dequantize(blocks, fmt: str, n: int, k: int) -> np.ndarray:
    """dequantize() (Quantization.swift:9-35) of [n, k] weights stored as `fmt` rows."""
    b = np.ascontiguousarray(blocks, np.uint8)
    out = np.empty(n * k, np.float32)
    lib().oracle_dequantize(WEIGHT_FORMATS[fmt], b.ctypes.data, n * k, _p32(out))
    return out.reshape(n, k)


def linear(x, blocks, fmt: str, n: int) -> np.ndarray:
    """CPUOps.linear (CPUOps.swift:77-105): y[m, n] = x[m, k] . W[n, k]^T with CPUOps.dot per row."""
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    b = np.ascontiguousarray(blocks, np.uint8).reshape(n, -1)
    y = np.empty((m, n), np.float32)
    L = lib()
    for i in range(m):
        xi = np.ascontiguousarray(x[i])
        for r in range(n):
            y[i, r] = L.oracle_row_dot(WEIGHT_FORMATS[fmt], b[r].ctypes.data, _p32(xi), k)
    return y


def rmsnorm(x, w, eps: float) -> np.ndarray:
    """CPUOps.rmsNorm (CPUOps.swift:144-158) over the last dimension."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    d = x.shape[-1]
    out = np.empty_like(x)
    lib().oracle_rmsnorm(_p32(x), _p32(w), x.size // d, d, float(eps), _p32(out))
    return out


def silu(x) -> np.ndarray:
    """CPUOps.silu (CPUOps.swift:49-53)."""
    f = lib().oracle_silu
    return np.array([f(float(v)) for v in np.asarray(x, np.float32).reshape(-1)], np.float32).reshape(np.shape(x))


def decode_project(fmt: str, weights, x, *, norm_weight=None, eps: float = 1e-5, silu_gate: bool = False,
                   add_to=None) -> list[np.ndarray]:
    """The fused projection of the dec_* kernels (decode_fused.metal:32-122) on the CPU path: x [tokens, k] f32,
    optionally RMS-normalised (norm_weight [k]), then each weight matrix (GGUF rows, list of up to 3 [n_i, row
    bytes] uint8 arrays) applied; silu_gate: [silu(W0 xn) * (W1 xn)]; add_to: list of [tokens, n_i] arrays the
    results are added to (residual). Returns the outputs."""
    x = np.ascontiguousarray(x, np.float32)
    T, k = x.shape
    mats = [np.ascontiguousarray(w, np.uint8) for w in weights]
    rows = [m.shape[0] for m in mats] + [0] * (3 - len(mats))
    if silu_gate:
        rows = [rows[0], 0, 0]
    outs = [np.array(add_to[i], np.float32, copy=True) if add_to is not None else np.zeros((T, rows[i]), np.float32)
            for i in range(1 if silu_gate else len(mats))]
    flags = (1 if norm_weight is not None else 0) | (2 if silu_gate else 0) | (4 if add_to is not None else 0)
    wp = (ctypes.c_void_p * 3)(*[mats[min(i, len(mats) - 1)].ctypes.data for i in range(3)])
    yp = (ctypes.c_void_p * 3)(*[outs[min(i, len(outs) - 1)].ctypes.data for i in range(3)])
    ys = (ctypes.c_int64 * 3)(*[outs[min(i, len(outs) - 1)].shape[1] for i in range(3)])
    g = np.ascontiguousarray(norm_weight if norm_weight is not None else np.zeros(k), np.float32)
    lib().oracle_decode_project(WEIGHT_FORMATS[fmt], k, (ctypes.c_int * 3)(*rows), flags, float(eps), wp, _p32(x), T,
                                k, _p32(g), yp, ys)
    return outs


def rows_mask(rows, T: int, H: int) -> np.ndarray:
    """[T, H] boolean mask of the rows (row = h*T + t)."""
    m = np.zeros((T, H), bool)
    r = np.asarray(rows, np.int64)
    m[r % T, r // T] = True
    return m


def error_metrics(actual, expected) -> dict:
    """ErrorMetrics (ErrorMetrics.swift:15-27)."""
    a = np.ascontiguousarray(actual, np.float32).reshape(-1)
    e = np.ascontiguousarray(expected, np.float64).reshape(-1)
    if a.size != e.size:
        raise ValueError("length mismatch")
    o = np.zeros(4, np.float64)
    lib().oracle_error_metrics(_p32(a), e.ctypes.data_as(_f64p), a.size, o.ctypes.data_as(_f64p))
    return {"n": int(a.size), "maxAbs": float(o[0]), "meanAbs": float(o[1]), "rms": float(o[2]),
            "maxRelPeak": float(o[3])}


def format_metrics(m: dict) -> str:
    return (f"n={m['n']} maxAbs={m['maxAbs']:.3e} meanAbs={m['meanAbs']:.3e} rms={m['rms']:.3e} "
            f"maxRel(peak)={m['maxRelPeak']:.3e}")


def splitmix_uniform(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """SplitMix.nextFloat() draws of KernelTests.swift:102-114 (uniform [-1,1)), in row-major order."""
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    lib().oracle_splitmix_uniform(ctypes.c_uint64(seed & (2**64 - 1)), float(scale), _p32(out), n)
    return out.reshape(shape)


def splitmix_normal(seed: int, shape) -> np.ndarray:
    """SplitMix64 + Box-Muller N(0,1) draws, row-major."""
    n = int(np.prod(shape))
    out = np.empty(max(n, 1), np.float32)
    lib().oracle_splitmix_normal(ctypes.c_uint64(seed & (2**64 - 1)), _p32(out), n)
    return out[:n].reshape(shape)


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
