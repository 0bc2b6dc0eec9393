"""Host-side attention interface over libalpaca_cuda.so.

``attention`` mirrors alpaca.swift's test-level boundary ``MetalOps.attention(q:keys:values:startPosition:kv:
precision:) -> Tensor`` (Sources/AlpacaMetal/Backend/MetalOps.swift:177-206): f32 host arrays in, the KV cache
rounded to f16 with 32 zero pad rows when ``kv == "f16"`` (MetalOps.swift:182-189), the kernel chosen by the
dispatch policy of ``KernelEncoder.attention`` (KernelEncoder.swift:306-343), f32 [tokens, heads, head_dim] out.

``attention_device`` is the model-path form (``KernelEncoder.attention`` / ``attentionTensor``): torch CUDA
tensors already resident in HBM, enqueued on the current stream, no host round trip. PyTorch only supplies device
memory and streams here; all attention arithmetic runs in the library's own sm_100a kernels.

``rope_kv_append`` is the step upstream of attention, ``KernelEncoder.ropeQKVStore`` (KernelEncoder.swift:401-411):
q rotated in place, rotated k and raw v appended to the cache. ``rope`` mirrors ``MetalOps.rope(_:startPosition:
theta:)`` (MetalOps.swift:165-171): a host f32 [tokens, heads, head_dim] array rotated through the same kernel.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import (FLAG_VARLEN, PROJ_ADD, PROJ_NORM, PROJ_SILU, AlpacaCUDAError, AttnDesc, DType, Kernel,
                   ProjDesc, RopeDesc, Status, WeightFormat, check, load)

KV_PADDING_ROWS = 32  # KernelEncoder.kvPaddingRows (KernelEncoder.swift:73)

_DT = {torch.float32: DType.F32, torch.float16: DType.F16}


def _dtype(t: torch.Tensor) -> DType:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"unsupported dtype {t.dtype}") from None


def _as4(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() == 3:
        t = t.unsqueeze(0)
    if t.dim() != 4:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"{name} must be [seqs, rows, heads, head_dim] or 3-D")
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"{name}: [heads, head_dim] must be contiguous")
    return t


def make_desc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *, start_position: int = 0,
              ctx_lens: torch.Tensor | None = None, max_ctx_len: int | None = None, scale: float = 0.0,
              flags: int = 0, block_table: torch.Tensor | None = None) -> AttnDesc:
    """Descriptor for q [S,T,H,d], k/v [S,rows,Hkv,d], out [S,T,H,d] (3-D tensors mean S = 1). With
    `block_table` (CUDA int32 [S, max_blocks]) k and v are block pools [pool_blocks, block_rows, Hkv, d] and row r
    of sequence s is row r % block_rows of block block_table[s, r // block_rows]."""
    q4, k4, v4, o4 = _as4(q, "q"), _as4(k, "k"), _as4(v, "v"), _as4(out, "out")
    if k4.stride() != v4.stride() or k4.shape != v4.shape or k4.dtype != v4.dtype:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "k and v must share shape, dtype and strides")
    S, T, H, d = q4.shape
    d_ = AttnDesc()
    d_.n_seqs, d_.n_heads, d_.n_kv_heads, d_.head_dim = S, H, k4.shape[2], d
    d_.tokens, d_.start_position = T, int(start_position)
    if ctx_lens is not None:
        if ctx_lens.dtype != torch.int32 or not ctx_lens.is_cuda:
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "ctx_lens must be a CUDA int32 tensor")
        d_.ctx_lens = ctx_lens.data_ptr()
        d_.max_ctx_len = int(max_ctx_len if max_ctx_len is not None else k4.shape[1])
    d_.q_dtype, d_.kv_dtype, d_.out_dtype = _dtype(q4), _dtype(k4), _dtype(o4)
    d_.q, d_.q_token_stride, d_.q_seq_stride = q4.data_ptr(), q4.stride(1), q4.stride(0) if S > 1 else 0
    d_.k, d_.v = k4.data_ptr(), v4.data_ptr()
    d_.kv_row_stride, d_.kv_seq_stride = k4.stride(1), k4.stride(0) if S > 1 else 0
    if block_table is not None:
        if block_table.dtype != torch.int32 or not block_table.is_cuda or block_table.dim() != 2 or \
                block_table.shape[0] != S or not block_table.is_contiguous():
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "block_table must be a contiguous CUDA int32 [seqs, blocks]")
        d_.block_table = block_table.data_ptr()
        d_.max_blocks = block_table.shape[1]
        d_.block_rows, d_.pool_blocks, d_.block_stride = k4.shape[1], k4.shape[0], k4.stride(0)
        d_.kv_seq_stride = 0
    d_.out, d_.out_token_stride, d_.out_seq_stride = o4.data_ptr(), o4.stride(1), o4.stride(0) if S > 1 else 0
    d_.scale, d_.flags = float(scale), int(flags) & 0xFFFFFFFF
    return d_


def make_varlen_desc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, q_offsets: torch.Tensor,
                     start_positions: torch.Tensor, *, max_tokens: int, max_ctx_len: int, scale: float = 0.0,
                     flags: int = 0, block_table: torch.Tensor | None = None) -> AttnDesc:
    """Descriptor of a ragged prefill (ALPACA_ATTN_FLAG_VARLEN): several sequences' query chunks in one call.

    q [total_tokens, H, d] and out [total_tokens, H, d] are packed: sequence s owns rows q_offsets[s] ..
    q_offsets[s+1]-1 (q_offsets: CUDA int32 [S + 1]) and its query t sits at absolute position start_positions[s] + t
    (CUDA int32 [S]) of its own cache, k/v [S, rows >= max_ctx_len, Hkv, d], or pools with `block_table` as for
    make_desc. `max_tokens` bounds every sequence's query count and `max_ctx_len` every start + count."""
    for name, t, n in (("q_offsets", q_offsets, None), ("start_positions", start_positions, None)):
        if t.dtype != torch.int32 or not t.is_cuda or t.dim() != 1 or not t.is_contiguous():
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"{name} must be a contiguous CUDA int32 vector")
    S = start_positions.numel()
    if q_offsets.numel() != S + 1:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "q_offsets must hold n_seqs + 1 entries")
    if q.dim() != 3 or out.dim() != 3 or out.shape[:1] != q.shape[:1]:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "ragged q and out must be packed [total_tokens, heads, head_dim]")
    k4 = _as4(k, "k")
    if block_table is None and k4.shape[0] != S:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "k / v must hold one cache per sequence")
    # the per-sequence cache layout, with a stand-in q / out of S sequences (their strides are ignored)
    d_ = make_desc(q.unsqueeze(0).expand(S, *q.shape), k, v, out.unsqueeze(0).expand(S, *out.shape),
                   scale=scale, flags=flags, block_table=block_table)
    d_.flags = (int(flags) | FLAG_VARLEN) & 0xFFFFFFFF
    d_.q_seq_stride = d_.out_seq_stride = 0
    d_.tokens = int(max_tokens)
    d_.start_position = 0
    d_.max_ctx_len = int(max_ctx_len)
    d_.q_offsets, d_.start_positions = q_offsets.data_ptr(), start_positions.data_ptr()
    d_.total_tokens = q.shape[0]
    return d_


def prefill_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, q_offsets: torch.Tensor,
                   start_positions: torch.Tensor, *, max_tokens: int, max_ctx_len: int, scale: float = 0.0,
                   flags: int = 0, workspace: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
                   block_table: torch.Tensor | None = None) -> AttnDesc:
    """Enqueue a ragged prefill (make_varlen_desc) on the tensor-core kernel; allocates the workspace (work list,
    f16 staging of f32 queries and, for a call with fewer work items than SMs, the split-KV records) with torch
    when none is given or the one given is smaller than the library asks for."""
    desc = make_varlen_desc(q, k, v, out, q_offsets, start_positions, max_tokens=max_tokens, max_ctx_len=max_ctx_len,
                            scale=scale, flags=flags, block_table=block_table)
    need = workspace_bytes(desc, Kernel.PREFILL_TC)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    launch(desc, Kernel.PREFILL_TC, workspace, stream)
    return desc


def workspace_bytes(desc: AttnDesc, kind: Kernel = Kernel.AUTO) -> int:
    n = ctypes.c_size_t(0)
    check(load().alpaca_attention_workspace_bytes(ctypes.byref(desc), int(kind), ctypes.byref(n)))
    return int(n.value)


def select_kernel(desc: AttnDesc) -> Kernel:
    k = ctypes.c_int(0)
    check(load().alpaca_attention_select(ctypes.byref(desc), ctypes.byref(k)))
    return Kernel(k.value)


def launch(desc: AttnDesc, kind: Kernel = Kernel.AUTO, workspace: torch.Tensor | None = None,
           stream: torch.cuda.Stream | None = None) -> None:
    """Enqueue one call of alpaca_attention on `stream` (default: torch's current stream)."""
    s = stream if stream is not None else torch.cuda.current_stream()
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(load().alpaca_attention(ctypes.byref(desc), int(kind), ws_ptr, ws_len, s.cuda_stream))


def attention_device(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *, start_position: int = 0,
                     kind: Kernel = Kernel.AUTO, ctx_lens: torch.Tensor | None = None,
                     max_ctx_len: int | None = None, scale: float = 0.0, flags: int = 0,
                     workspace: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
                     block_table: torch.Tensor | None = None) -> AttnDesc:
    """Enqueue attention on device tensors (KernelEncoder.attention / attentionTensor). Allocates the workspace
    with torch when none is given (callers on a hot loop pass their own). `block_table`: paged cache (make_desc)."""
    desc = make_desc(q, k, v, out, start_position=start_position, ctx_lens=ctx_lens, max_ctx_len=max_ctx_len,
                     scale=scale, flags=flags, block_table=block_table)
    need = workspace_bytes(desc, kind)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    launch(desc, kind, workspace, stream)
    return desc


def device_status(stream: torch.cuda.Stream | None = None, clear: bool = True) -> None:
    """Synchronise and raise AlpacaCUDAError(DEVICE_TIMEOUT) if a bounded device-side wait gave up."""
    s = stream if stream is not None else torch.cuda.current_stream()
    check(load().alpaca_cuda_device_status(s.cuda_stream, int(clear)))


def to_cache(x: np.ndarray, kv: str, device) -> torch.Tensor:
    """Upload keys/values [capacity, kvHeads, d] as the GPU cache: f32, or f16 with 32 zero pad rows."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if kv == "f32":
        return torch.from_numpy(x).to(device)
    buf = torch.zeros((x.shape[0] + KV_PADDING_ROWS,) + x.shape[1:], dtype=torch.float16, device=device)
    buf[: x.shape[0]] = torch.from_numpy(x).to(device).half()
    return buf


def attention(q: np.ndarray, keys: np.ndarray, values: np.ndarray, start_position: int, kv: str = "f16",
              precision: str = "fast", *, kind: Kernel = Kernel.AUTO, device: str | int = "cuda") -> np.ndarray:
    """MetalOps.attention (MetalOps.swift:177-206).

    q [tokens, heads, d], keys/values [capacity, kvHeads, d], all f32; the query token t sits at absolute
    position start_position + t. `kv` is "f16" (cache rounded to half, as the model path stores it) or "f32".
    `precision` is accepted for signature compatibility: every f16-KV prefill kernel here uses f16 MMA operands
    and f32 accumulation, as both of the reference's prefill paths do. Returns f32 [tokens, heads, d]."""
    q = np.asarray(q, dtype=np.float32)
    keys = np.asarray(keys, dtype=np.float32)
    values = np.asarray(values, dtype=np.float32)
    if not (q.ndim == 3 and keys.ndim == 3 and keys.shape == values.shape and keys.shape[2] == q.shape[2]
            and q.shape[1] % keys.shape[1] == 0 and q.shape[2] % 32 == 0 and q.shape[2] <= 256
            and start_position + q.shape[0] <= keys.shape[0] and start_position >= 0):
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"attention shapes q {q.shape} k {keys.shape}")
    if kv not in ("f16", "f32"):
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"kv precision {kv!r}")
    if precision not in ("fast", "exact"):
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"precision {precision!r}")
    dev = torch.device(device)
    kb, vb = to_cache(keys, kv, dev), to_cache(values, kv, dev)
    qb = torch.from_numpy(np.ascontiguousarray(q)).to(dev)
    out = torch.empty(q.shape, dtype=torch.float32, device=dev)
    attention_device(qb, kb, vb, out, start_position=start_position, kind=kind)
    device_status()
    return out.cpu().numpy()


# ---------------------------------------------------------------------------------------------- RoPE + KV append

def make_rope_desc(q: torch.Tensor | None, k: torch.Tensor | None, v: torch.Tensor | None,
                   k_cache: torch.Tensor | None, v_cache: torch.Tensor | None, *, theta: float,
                   start_position: int = 0, positions: torch.Tensor | None = None,
                   interleaved: bool = True, block_table: torch.Tensor | None = None) -> RopeDesc:
    """Descriptor for q [S,T,H,d] (rotated in place), k/v [S,T,Hkv,d] f32 and caches [S,rows,Hkv,d] (3-D tensors
    mean S = 1). q or (k, v, caches) may be None. With `block_table` (CUDA int32 [S, max_blocks]) the caches are
    block pools [pool_blocks, block_rows, Hkv, d], laid out as for the attention call (make_desc)."""
    d_ = RopeDesc()
    ref = q if q is not None else k
    if ref is None:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "rope: neither q nor k given")
    r4 = _as4(ref, "q" if q is not None else "k")
    S, T, _, D = r4.shape
    d_.n_seqs, d_.tokens, d_.head_dim = S, T, D
    d_.start_position = int(start_position)
    if positions is not None:
        if positions.dtype != torch.int32 or not positions.is_cuda:
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "positions must be a CUDA int32 tensor")
        d_.positions = positions.data_ptr()
    d_.theta = float(theta)
    d_.interleaved = 1 if interleaved else 0
    if q is not None:
        q4 = _as4(q, "q")
        d_.n_heads, d_.q_dtype = q4.shape[2], _dtype(q4)
        d_.q, d_.q_token_stride, d_.q_seq_stride = q4.data_ptr(), q4.stride(1), q4.stride(0) if S > 1 else 0
    if k is not None:
        k4, v4, kc4, vc4 = _as4(k, "k"), _as4(v, "v"), _as4(k_cache, "k_cache"), _as4(v_cache, "v_cache")
        if k4.dtype != torch.float32 or v4.dtype != torch.float32 or k4.stride() != v4.stride():
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "rope: k and v must be f32 with equal strides")
        if kc4.stride() != vc4.stride() or kc4.dtype != vc4.dtype:
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "rope: caches must share dtype and strides")
        d_.n_kv_heads, d_.cache_dtype = k4.shape[2], _dtype(kc4)
        d_.k, d_.v, d_.kv_token_stride = k4.data_ptr(), v4.data_ptr(), k4.stride(1)
        d_.kv_seq_stride = k4.stride(0) if S > 1 else 0
        d_.k_cache, d_.v_cache, d_.cache_row_stride = kc4.data_ptr(), vc4.data_ptr(), kc4.stride(1)
        d_.cache_seq_stride = kc4.stride(0) if S > 1 else 0
        d_.cache_rows = kc4.shape[1]  # contiguous caches: positions past the cache are reported, not written
        if block_table is not None:
            if block_table.dtype != torch.int32 or not block_table.is_cuda or block_table.dim() != 2 or \
                    block_table.shape[0] != S or not block_table.is_contiguous():
                raise AlpacaCUDAError(Status.INVALID_ARGUMENT,
                                      "block_table must be a contiguous CUDA int32 [seqs, blocks]")
            d_.block_table, d_.max_blocks = block_table.data_ptr(), block_table.shape[1]
            d_.block_rows, d_.pool_blocks, d_.block_stride = kc4.shape[1], kc4.shape[0], kc4.stride(0)
            d_.cache_seq_stride = 0
            d_.cache_rows = 0
    return d_


def rope_launch(desc: RopeDesc, stream: torch.cuda.Stream | None = None) -> None:
    s = stream if stream is not None else torch.cuda.current_stream()
    check(load().alpaca_rope_kv_append(ctypes.byref(desc), ctypes.c_void_p(s.cuda_stream)))


def rope_kv_append(q: torch.Tensor | None, k: torch.Tensor | None, v: torch.Tensor | None,
                   k_cache: torch.Tensor | None, v_cache: torch.Tensor | None, *, theta: float,
                   start_position: int = 0, positions: torch.Tensor | None = None, interleaved: bool = True,
                   stream: torch.cuda.Stream | None = None, block_table: torch.Tensor | None = None) -> RopeDesc:
    """Enqueue RoPE + KV append on device tensors (KernelEncoder.ropeQKVStore, KernelEncoder.swift:401-411)."""
    d_ = make_rope_desc(q, k, v, k_cache, v_cache, theta=theta, start_position=start_position, positions=positions,
                        interleaved=interleaved, block_table=block_table)
    rope_launch(d_, stream)
    return d_


def decode_rope(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor, out: torch.Tensor, *, theta: float, start_position: int = 0,
                ctx_lens: torch.Tensor | None = None, max_ctx_len: int | None = None, interleaved: bool = True,
                block_table: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> None:
    """One decode step with the RoPE + KV append fused into the attention launch (alpaca_attn_decode_rope): the
    results of rope_kv_append(q, k_new, v_new, caches, positions = context length - 1) followed by the split decode
    over the caches, except that q is not rotated in place. q [S,1,H,d], k_new / v_new f32 [S,1,Hkv,d], caches as
    for attention_device (contiguous [S,rows,Hkv,d] f16, or pools with `block_table`), out [S,1,H,d]."""
    ad = make_desc(q, k_cache, v_cache, out, start_position=start_position, ctx_lens=ctx_lens,
                   max_ctx_len=max_ctx_len, block_table=block_table)
    rd = make_rope_desc(q, k_new, v_new, k_cache, v_cache, theta=theta, start_position=start_position,
                        interleaved=interleaved, block_table=block_table)
    if workspace is None:
        n = workspace_bytes(ad, Kernel.DECODE_SPLIT)
        workspace = torch.empty(max(n, 16), dtype=torch.uint8, device=q.device)
    s = stream if stream is not None else torch.cuda.current_stream()
    check(load().alpaca_attn_decode_rope(ctypes.byref(ad), ctypes.byref(rd), workspace.data_ptr(),
                                         workspace.numel() * workspace.element_size(), s.cuda_stream))


def rope(x: np.ndarray, start_position: int, theta: float, interleaved: bool = True) -> np.ndarray:
    """MetalOps.rope(_:startPosition:theta:) (MetalOps.swift:165-171): f32 [tokens, heads, head_dim] in and out."""
    x = np.asarray(x, dtype=np.float32)
    if x.ndim != 3 or x.shape[2] % 2:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, f"rope shape {x.shape}")
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    rope_kv_append(t, None, None, None, None, theta=theta, start_position=start_position, interleaved=interleaved)
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ---------------------------------------------------------------------------------------------- decode projections

_WF = {"f16": WeightFormat.F16, "q8_0": WeightFormat.Q8_0, "q4_0": WeightFormat.Q4_0}


def make_proj_desc(weights: list[torch.Tensor], fmt: str, k: int, x: torch.Tensor, outs: list[torch.Tensor], *,
                   norm_weight: torch.Tensor | None = None, eps: float = 1e-5, silu_gate: bool = False,
                   add: bool = False) -> ProjDesc:
    """Descriptor of alpaca_decode_project: weights are CUDA uint8 [rows, row bytes] tensors in `fmt` ("f16", "q8_0",
    "q4_0"; f16 may also be given as float16 [rows, k]), x f32 [tokens, >= k], outs f32 [tokens, >= rows_i] (one
    per matrix; one for silu_gate, which takes the gate and up matrices)."""
    if fmt not in _WF:
        raise AlpacaCUDAError(Status.UNSUPPORTED, f"weight format {fmt!r}")
    if not 1 <= len(weights) <= (2 if silu_gate else 3) or len(outs) != (1 if silu_gate else len(weights)):
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "project: 1-3 matrices with one output each (silu: 2 and 1)")
    x2 = x if x.dim() == 2 else x.reshape(1, -1)
    d = ProjDesc()
    d.n_tokens, d.k, d.format = x2.shape[0], int(k), int(_WF[fmt])
    d.flags = (PROJ_NORM if norm_weight is not None else 0) | (PROJ_SILU if silu_gate else 0) | (PROJ_ADD if add else 0)
    d.eps = float(eps)
    for i, w in enumerate(weights):
        if not w.is_cuda or not w.is_contiguous():
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "project: weights must be contiguous CUDA tensors")
        d.w[i] = w.data_ptr()
        if i == 0 or not silu_gate:
            d.rows[i] = w.shape[0]
    if silu_gate:
        d.rows[1] = 0
    for i, o in enumerate(outs):
        o2 = o if o.dim() == 2 else o.reshape(1, -1)
        if o2.dtype != torch.float32 or o2.stride(-1) != 1:
            raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "project: outputs must be f32 rows")
        d.y[i], d.y_stride[i] = o2.data_ptr(), o2.stride(0)
    if x2.dtype != torch.float32 or x2.stride(-1) != 1:
        raise AlpacaCUDAError(Status.INVALID_ARGUMENT, "project: x must be f32 rows")
    d.x, d.x_stride = x2.data_ptr(), x2.stride(0)
    if norm_weight is not None:
        d.norm_weight = norm_weight.data_ptr()
    return d


def project_launch(desc: ProjDesc, stream: torch.cuda.Stream | None = None) -> None:
    s = stream if stream is not None else torch.cuda.current_stream()
    check(load().alpaca_decode_project(ctypes.byref(desc), ctypes.c_void_p(s.cuda_stream)))


def decode_project(weights: list[torch.Tensor], fmt: str, k: int, x: torch.Tensor, outs: list[torch.Tensor], *,
                   norm_weight: torch.Tensor | None = None, eps: float = 1e-5, silu_gate: bool = False,
                   add: bool = False, stream: torch.cuda.Stream | None = None) -> ProjDesc:
    """Enqueue the fused decode projection (KernelEncoder.decodeQKV / decodeProjection / decodeGateUp,
    KernelEncoder.swift:386-400) on device tensors; see make_proj_desc."""
    d = make_proj_desc(weights, fmt, k, x, outs, norm_weight=norm_weight, eps=eps, silu_gate=silu_gate, add=add)
    project_launch(d, stream)
    return d
