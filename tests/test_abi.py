"""The C ABI without a GPU: the library loads, exports every symbol include/alpaca_cuda.h declares, and its
host-only entry points (validation, dispatch policy, workspace sizing, status strings) behave as specified.
No call here launches a kernel."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "alpaca_cuda.h"


@pytest.fixture(scope="module")
def lib():
    from alpaca_b200 import build
    try:
        build.build()
    except (RuntimeError, OSError) as e:  # pragma: no cover - toolchain missing
        pytest.fail(f"cannot build libalpaca_cuda.so: {e}")
    import alpaca_b200
    return alpaca_b200.load()


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_]+\s*\*?\s*(alpaca_[a-z_0-9]+)\s*\(", text, re.M)))


def test_header_declarations_match_bindings():
    import alpaca_b200
    assert declared_functions() == sorted(alpaca_b200.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.alpaca_cuda_version() == 10100


def test_status_strings(lib):
    from alpaca_b200 import Status
    for s in Status:
        assert lib.alpaca_cuda_status_string(int(s))
    assert lib.alpaca_cuda_status_string(99) == b"unknown status"


FAKE = 1 << 20  # a 16-byte aligned fake device address: validation never dereferences pointers


def desc(**kw):
    from alpaca_b200 import AttnDesc, DType
    d = AttnDesc()
    d.n_seqs, d.n_heads, d.n_kv_heads, d.head_dim = 1, 9, 3, 64
    d.tokens, d.start_position = 128, 0
    d.q_dtype = d.kv_dtype = int(DType.F16)
    d.out_dtype = int(DType.F32)
    d.q = d.k = d.v = d.out = FAKE
    d.q_token_stride = d.out_token_stride = 9 * 64
    d.kv_row_stride = 3 * 64
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def select(lib, d):
    k = ctypes.c_int(-1)
    st = lib.alpaca_attention_select(ctypes.byref(d), ctypes.byref(k))
    return st, k.value


def ws(lib, d, kind=0):
    n = ctypes.c_size_t(0)
    st = lib.alpaca_attention_workspace_bytes(ctypes.byref(d), kind, ctypes.byref(n))
    return st, n.value


def test_dispatch_policy_mirrors_kernel_encoder(lib):
    """KernelEncoder.attention (KernelEncoder.swift:309-343): decode split for one f16-KV token with context >= 64,
    head_dim 64/128 and G <= 8; tensor prefill for f16 KV and >= 8 tokens; the general kernel otherwise."""
    from alpaca_b200 import DType, Kernel, Status
    assert select(lib, desc()) == (Status.OK, Kernel.PREFILL_TC)
    assert select(lib, desc(tokens=7)) == (Status.OK, Kernel.GENERAL)
    assert select(lib, desc(tokens=8)) == (Status.OK, Kernel.PREFILL_TC)
    assert select(lib, desc(tokens=1, start_position=63)) == (Status.OK, Kernel.DECODE_SPLIT)
    assert select(lib, desc(tokens=1, start_position=62)) == (Status.OK, Kernel.GENERAL)
    assert select(lib, desc(kv_dtype=int(DType.F32))) == (Status.OK, Kernel.GENERAL)
    assert select(lib, desc(tokens=1, start_position=100, kv_dtype=int(DType.F32))) == (Status.OK, Kernel.GENERAL)
    assert select(lib, desc(tokens=1, start_position=100, n_heads=18, n_kv_heads=2,
                            q_token_stride=18 * 64, out_token_stride=18 * 64, kv_row_stride=128)) == \
        (Status.OK, Kernel.GENERAL)  # G = 9 > 8
    assert select(lib, desc(head_dim=96, q_token_stride=9 * 96, out_token_stride=9 * 96, kv_row_stride=3 * 96)) == \
        (Status.OK, Kernel.GENERAL)


def test_decode_workspace_matches_split_layout(lib):
    """Partial state [seq][kvHead][split][G][d+2] f32 with 128-row splits at d=64 (one split needs none)."""
    from alpaca_b200 import Kernel, Status
    assert ws(lib, desc(tokens=1, start_position=127), Kernel.DECODE_SPLIT) == (Status.OK, 0)
    st, n = ws(lib, desc(tokens=1, start_position=128), Kernel.DECODE_SPLIT)
    assert st == Status.OK and n == 4 * 1 * 9 * 2 * 66
    st, n = ws(lib, desc(tokens=1, start_position=4095, n_seqs=64, q_seq_stride=576, kv_seq_stride=4128 * 192,
                         out_seq_stride=576), Kernel.DECODE_SPLIT)
    assert st == Status.OK and n == 4 * 64 * 9 * 32 * 66
    assert ws(lib, desc(), Kernel.PREFILL_TC) == (Status.OK, 0)             # f16 Q needs no staging
    from alpaca_b200 import DType
    assert ws(lib, desc(q_dtype=int(DType.F32), q_token_stride=576), Kernel.PREFILL_TC) == (Status.OK, 128 * 576 * 2)


@pytest.mark.parametrize("bad", [
    dict(n_heads=10),                 # not a multiple of kv heads
    dict(head_dim=48),                # not a multiple of 32
    dict(head_dim=288),               # above 256
    dict(tokens=0),
    dict(start_position=-1),
    dict(q=0),
    dict(k=FAKE + 8),                 # misaligned
    dict(kv_row_stride=100),          # smaller than a row
    dict(q_token_stride=9 * 64 + 4),  # not a multiple of 16 bytes for f16
    dict(q_dtype=7),
    dict(scale=-1.0),
    dict(n_seqs=2),                   # several sequences with zero sequence strides
])
def test_invalid_arguments_rejected(lib, bad):
    from alpaca_b200 import Status
    d = desc(**bad)
    st, _ = select(lib, d)
    assert st == Status.INVALID_ARGUMENT
    assert lib.alpaca_cuda_last_error()
    # the launching entry point refuses before touching the device
    assert lib.alpaca_attention(ctypes.byref(d), 0, None, 0, None) == Status.INVALID_ARGUMENT


def test_unsupported_kernel_requests(lib):
    from alpaca_b200 import DType, Kernel, Status
    d = desc(kv_dtype=int(DType.F32))
    assert lib.alpaca_attn_prefill(ctypes.byref(d), None, 0, None) == Status.UNSUPPORTED
    d = desc(tokens=4)
    assert lib.alpaca_attn_decode(ctypes.byref(d), None, 0, None) == Status.UNSUPPORTED
    assert ws(lib, desc(tokens=4), Kernel.DECODE_SPLIT)[0] == Status.UNSUPPORTED


def test_workspace_too_small_is_reported(lib):
    from alpaca_b200 import Kernel, Status
    d = desc(tokens=1, start_position=1000)
    assert lib.alpaca_attn_decode(ctypes.byref(d), None, 0, None) == Status.WORKSPACE_TOO_SMALL
    assert b"needed" in lib.alpaca_cuda_last_error()
    _ = Kernel


def test_ctx_lens_rules(lib):
    from alpaca_b200 import Kernel, Status
    d = desc(tokens=2, ctx_lens=FAKE, max_ctx_len=10)
    assert select(lib, d)[0] == Status.INVALID_ARGUMENT       # ragged lengths are decode-only
    d = desc(tokens=1, ctx_lens=FAKE, max_ctx_len=0)
    assert select(lib, d)[0] == Status.INVALID_ARGUMENT       # needs an upper bound
    d = desc(tokens=1, ctx_lens=FAKE, max_ctx_len=10)
    assert select(lib, d) == (Status.OK, Kernel.DECODE_SPLIT)  # ragged decode always splits


def test_python_mirror_rejects_like_metalops():
    """MetalOps.attention's guard (MetalOps.swift:179-181) raises invalidArgument before any device work."""
    import numpy as np
    from alpaca_b200 import AlpacaCUDAError, Status, attention
    q = np.zeros((4, 9, 64), np.float32)
    with pytest.raises(AlpacaCUDAError) as e:
        attention(q, np.zeros((3, 3, 64), np.float32), np.zeros((3, 3, 64), np.float32), 0)  # capacity < T
    assert e.value.status == Status.INVALID_ARGUMENT
    with pytest.raises(AlpacaCUDAError):
        attention(q, np.zeros((8, 2, 64), np.float32), np.zeros((8, 2, 64), np.float32), 0)  # 9 % 2
    with pytest.raises(AlpacaCUDAError):
        attention(np.zeros((4, 9, 48), np.float32), np.zeros((8, 3, 48), np.float32),
                  np.zeros((8, 3, 48), np.float32), 0)  # head dim % 32


# ---------------------------------------------------------------------------------------------- struct layouts

def test_descriptor_layouts_match_the_c_compiler(tmp_path):
    """The ctypes mirrors have the C structs' size and field offsets (gcc on the header)."""
    import shutil
    import subprocess

    from alpaca_b200 import AttnDesc, ProjDesc, RopeDesc
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "alpaca_cuda.h"', 'int main(void) {']
    structs = (("alpaca_attn_desc", AttnDesc), ("alpaca_rope_desc", RopeDesc), ("alpaca_proj_desc", ProjDesc))
    for cname, cls in structs:
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = dict((" ".join(l.split()[:2]), int(l.split()[2])) for l in subprocess.run([str(exe)], capture_output=True,
                                                                                      text=True, check=True).stdout.splitlines())
    for cname, cls in structs:
        assert out[f"{cname} size"] == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert out[f"{cname} {f}"] == getattr(cls, f).offset, (cname, f)


# ---------------------------------------------------------------------------------------------- RoPE + KV append

def rope_desc(**kw):
    from alpaca_b200 import DType, RopeDesc
    d = RopeDesc()
    d.n_seqs, d.n_heads, d.n_kv_heads, d.head_dim, d.tokens, d.start_position = 1, 9, 3, 64, 4, 10
    d.theta, d.interleaved = 1e5, 1
    d.q_dtype, d.cache_dtype = int(DType.F32), int(DType.F16)
    d.q = d.k = d.v = d.k_cache = d.v_cache = FAKE
    d.q_token_stride, d.kv_token_stride, d.cache_row_stride = 9 * 64, 3 * 64, 3 * 64
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("bad", [
    dict(head_dim=63),                # odd (CPUOps.rope's guard, CPUOps.swift:188)
    dict(head_dim=258),               # above the kernel's 256
    dict(theta=0.0),                  # CPUOps.swift:191
    dict(theta=float("nan")),
    dict(start_position=-1),          # CPUOps.swift:191
    dict(tokens=0),
    dict(n_heads=0, n_kv_heads=0),    # nothing to do
    dict(interleaved=2),
    dict(q=0),
    dict(k_cache=FAKE + 4),           # not 8-byte aligned
    dict(q_token_stride=9 * 64 - 2),  # smaller than a token
    dict(cache_row_stride=3 * 64 + 1),  # odd
    dict(n_seqs=2),                   # several sequences with zero sequence strides
    dict(n_seqs=70000),
    dict(cache_dtype=5),
    dict(flags=1),
])
def test_rope_invalid_arguments_rejected(lib, bad):
    from alpaca_b200 import Status
    d = rope_desc(**bad)
    assert lib.alpaca_rope_kv_append(ctypes.byref(d), None) == Status.INVALID_ARGUMENT
    assert lib.alpaca_cuda_last_error().startswith(b"rope")


# ---------------------------------------------------------------------------------------------- paged KV cache

def paged(**kw):
    base = dict(block_table=FAKE, block_rows=256, max_blocks=4, block_stride=256 * 3 * 64, pool_blocks=64,
                kv_seq_stride=0)
    base.update(kw)
    return base


def test_paged_cache_policy(lib):
    """A paged cache goes to the split decode at any context and to the tensor-core prefill at any length; the
    general kernel has no paged form."""
    from alpaca_b200 import DType, Kernel, Status
    assert select(lib, desc(tokens=1, start_position=10, **paged())) == (Status.OK, Kernel.DECODE_SPLIT)
    assert select(lib, desc(tokens=4, start_position=10, **paged())) == (Status.OK, Kernel.PREFILL_TC)
    assert select(lib, desc(tokens=2, n_seqs=2, q_seq_stride=576, out_seq_stride=576, **paged())) == \
        (Status.OK, Kernel.PREFILL_TC)  # no sequence stride needed for a paged cache
    assert select(lib, desc(tokens=4, kv_dtype=int(DType.F32), **paged()))[0] == Status.UNSUPPORTED
    d = desc(tokens=4, **paged())
    assert lib.alpaca_attention(ctypes.byref(d), int(Kernel.GENERAL), None, 0, None) == Status.UNSUPPORTED


@pytest.mark.parametrize("bad", [
    dict(block_rows=100),                    # not a multiple of 128
    dict(block_rows=0),
    dict(max_blocks=0),
    dict(pool_blocks=0),
    dict(max_blocks=1, start_position=200),  # 328 rows > 1 block of 256
    dict(block_stride=256 * 3 * 64 - 64),    # smaller than a block
    dict(block_stride=256 * 3 * 64 + 4),     # not a multiple of 16 bytes for f16
])
def test_paged_cache_invalid(lib, bad):
    from alpaca_b200 import Status
    d = desc(**paged(**bad))
    assert select(lib, d)[0] == Status.INVALID_ARGUMENT
    assert lib.alpaca_attention(ctypes.byref(d), 0, None, 0, None) == Status.INVALID_ARGUMENT


def rope_paged(**kw):
    base = dict(block_table=FAKE, block_rows=128, max_blocks=2, block_stride=128 * 3 * 64, pool_blocks=8)
    base.update(kw)
    return base


@pytest.mark.parametrize("bad", [
    dict(block_rows=100),                    # not a multiple of 128 (the attention kernels' block granularity)
    dict(max_blocks=0),
    dict(pool_blocks=0),
    dict(block_stride=127 * 3 * 64),         # smaller than a block
    dict(block_stride=128 * 3 * 64 + 1),     # odd
    dict(max_blocks=1, start_position=126),  # rows 126..129 need a second block
])
def test_rope_paged_invalid_arguments_rejected(lib, bad):
    from alpaca_b200 import Status
    d = rope_desc(**rope_paged(**bad))
    assert lib.alpaca_rope_kv_append(ctypes.byref(d), None) == Status.INVALID_ARGUMENT
    assert lib.alpaca_cuda_last_error().startswith(b"rope")


def test_rope_paged_cache_needs_no_sequence_stride(lib):
    """Several sequences appending into one pool: the cache sequence stride is unused (0) and the descriptor passes
    validation (without a GPU the call then fails at the device query, not on its arguments)."""
    from alpaca_b200 import Status
    d = rope_desc(**rope_paged(n_seqs=3, q_seq_stride=4 * 9 * 64, kv_seq_stride=4 * 3 * 64))
    assert lib.alpaca_rope_kv_append(ctypes.byref(d), None) != Status.INVALID_ARGUMENT
    d = rope_desc(**rope_paged(n_seqs=3, q_seq_stride=4 * 9 * 64, kv_seq_stride=4 * 3 * 64, block_table=0))
    assert lib.alpaca_rope_kv_append(ctypes.byref(d), None) == Status.INVALID_ARGUMENT


# ---------------------------------------------------------------------------------------------- fused RoPE + decode

def test_decode_rope_validation(lib):
    """alpaca_attn_decode_rope takes the new token's position from the attention descriptor and needs the RoPE
    descriptor to describe that one token of the same sequences, heads, q and f16 caches; anything else is an
    invalid argument before any device work (a valid pair fails only at the device query without a GPU)."""
    from alpaca_b200 import DType, Status

    def attn(**kw):
        base = dict(tokens=1, start_position=300, q_dtype=int(DType.F32), q_token_stride=576)
        base.update(kw)
        return desc(**base)

    def call(a, r):
        return lib.alpaca_attn_decode_rope(ctypes.byref(a), ctypes.byref(r), FAKE, 1 << 20, None)

    st = call(attn(), rope_desc(tokens=1, start_position=300))
    assert st not in (Status.OK, Status.INVALID_ARGUMENT, Status.UNSUPPORTED, Status.WORKSPACE_TOO_SMALL)
    for bad in (dict(positions=FAKE), dict(tokens=2), dict(start_position=299), dict(k_cache=FAKE + 4096),
                dict(cache_dtype=int(DType.F32)), dict(n_heads=8), dict(interleaved=2)):
        kw = dict(tokens=1, start_position=300)
        kw.update(bad)
        assert call(attn(), rope_desc(**kw)) == Status.INVALID_ARGUMENT, bad
        msg = lib.alpaca_cuda_last_error()
        assert msg.startswith(b"decode_rope") or msg.startswith(b"rope"), msg
    assert call(attn(tokens=2), rope_desc(tokens=1, start_position=300)) == Status.UNSUPPORTED
    assert lib.alpaca_attn_decode_rope(ctypes.byref(attn()), ctypes.byref(rope_desc(tokens=1, start_position=300)),
                                       FAKE, 16, None) == Status.WORKSPACE_TOO_SMALL


@pytest.mark.parametrize("bad", [
    dict(cache_rows=-1),
    dict(cache_rows=12, start_position=10, tokens=4),  # rows 10..13 past a 12-row cache
])
def test_rope_cache_rows_checked(lib, bad):
    from alpaca_b200 import Status
    d = rope_desc(**bad)
    assert lib.alpaca_rope_kv_append(ctypes.byref(d), None) == Status.INVALID_ARGUMENT
    assert lib.alpaca_cuda_last_error().startswith(b"rope")


def test_prefill_split_kv_workspace_policy(lib):
    """A uniform prefill with fewer work items (sequences x heads x pairs of 128-query tiles) than a B200's 148 SMs
    asks for split-KV records: parts = min(8, floor(148 / items), KV blocks / 4), so all parts run in one wave and
    each has at least 4 blocks; records of items x parts x 2 tiles x 128 rows x (d + 2) f32 follow the f32 queries'
    staging. A call that cannot use two parts asks for none."""
    from alpaca_b200 import DType, Kernel, Status
    pf = int(Kernel.PREFILL_TC)

    def rec(items, parts, d=64):
        return items * parts * 2 * 128 * (d + 2) * 4

    # alpaca's last 512-token chunk of a 4096-token prompt: 18 items, 32 KV blocks of 128 rows, 8 parts
    assert ws(lib, desc(tokens=512, start_position=3584), pf) == (Status.OK, rec(18, 8))
    # the second chunk (8 blocks): 2 parts; the first (4 blocks): too few for two parts of 4
    assert ws(lib, desc(tokens=512, start_position=512), pf) == (Status.OK, rec(18, 2))
    assert ws(lib, desc(tokens=512, start_position=0), pf) == (Status.OK, 0)
    # f32 queries: their f16 staging comes first
    assert ws(lib, desc(tokens=512, start_position=3584, q_dtype=int(DType.F32)), pf) == \
        (Status.OK, 512 * 9 * 64 * 2 + rec(18, 8))
    # three 256-token sequences at 3000 (26 blocks): 27 items, floor(148 / 27) = 5 parts; 6 would need a second wave
    three = dict(n_seqs=3, tokens=256, start_position=3000, q_seq_stride=256 * 9 * 64, out_seq_stride=256 * 9 * 64,
                 kv_seq_stride=3256 * 3 * 64)
    assert ws(lib, desc(**three), pf) == (Status.OK, rec(27, 5))
    # head_dim 128 (64-row KV blocks): 16 items, 38 blocks, 8 parts
    d128 = dict(head_dim=128, n_heads=8, n_kv_heads=2, tokens=384, start_position=2000, q_token_stride=8 * 128,
                out_token_stride=8 * 128, kv_row_stride=2 * 128)
    assert ws(lib, desc(**d128), pf) == (Status.OK, rec(16, 8, 128))
    # a whole 4096-token prompt: 144 items, floor(148 / 144) = 1, no split
    assert ws(lib, desc(tokens=4096), pf) == (Status.OK, 0)


def test_varlen_prefill_host_checks(lib):
    """The ragged prefill flag: AUTO picks the tensor-core prefill, the other kernels refuse it, the workspace holds
    the heaviest-first work list (16 bytes + 32 per unit of two 128-row tiles), the f16 staging of f32 queries and,
    for a call with fewer work items than SMs at its bounds, the split-KV records, and the descriptor's own
    contradictions are refused before anything is enqueued."""
    from alpaca_b200 import FLAG_VARLEN, DType, Kernel, Status
    base = dict(flags=FLAG_VARLEN, n_seqs=3, tokens=600, max_ctx_len=2000, total_tokens=900, q_offsets=FAKE,
                start_positions=FAKE + 256, kv_seq_stride=2000 * 3 * 64)
    st, k = select(lib, desc(**base))
    assert (st, k) == (Status.OK, Kernel.PREFILL_TC)
    units = 3 * 3  # ceil(600 / 256) units per sequence
    # 81 items (units x heads): two parts each would need 162 > 148 SMs, so the call runs unsplit
    assert ws(lib, desc(**base)) == (Status.OK, 16 + 32 * units)
    assert ws(lib, desc(**base, q_dtype=int(DType.F32), q_token_stride=9 * 64)) == \
        (Status.OK, 900 * 9 * 64 * 2 + 16 + 32 * units)
    # one sequence: 3 units x 9 heads = 27 items, floor(148 / 27) = 5 parts, capped at ceil(2000 / 128) / 4 = 4
    one = {**base, "n_seqs": 1, "total_tokens": 600}
    records = 27 * 4 * 2 * 128 * (64 + 2) * 4
    assert ws(lib, desc(**one)) == (Status.OK, 16 + 32 * 3 + records)
    # 3 x 16 units x 9 heads = 432 items: no split, the work list alone
    big = {**base, "tokens": 4096, "max_ctx_len": 8192, "total_tokens": 9000, "kv_seq_stride": 8192 * 3 * 64}
    assert ws(lib, desc(**big)) == (Status.OK, 16 + 32 * 3 * 16)
    assert ws(lib, desc(**base), int(Kernel.GENERAL))[0] == Status.UNSUPPORTED
    assert ws(lib, desc(**base), int(Kernel.DECODE_SPLIT))[0] == Status.UNSUPPORTED
    # q / out sequence strides are ignored (packed rows); the per-sequence caches still need theirs
    assert select(lib, desc(**{**base, "kv_seq_stride": 0}))[0] == Status.INVALID_ARGUMENT
    for bad in (dict(q_offsets=0), dict(start_positions=0), dict(total_tokens=0), dict(max_ctx_len=0),
                dict(ctx_lens=FAKE)):
        assert select(lib, desc(**{**base, **bad}))[0] == Status.INVALID_ARGUMENT, bad
    # a paged ragged call: the block table must cover max_ctx_len rows
    paged = {**base, "kv_seq_stride": 0, "block_table": FAKE, "block_rows": 256, "pool_blocks": 64,
             "block_stride": 256 * 3 * 64}
    assert select(lib, desc(**paged, max_blocks=8))[0] == Status.OK
    assert select(lib, desc(**paged, max_blocks=7))[0] == Status.INVALID_ARGUMENT


# ---------------------------------------------------------------------------------------------- decode projections

def proj_desc(**kw):
    from alpaca_b200 import ProjDesc, WeightFormat
    d = ProjDesc()
    d.n_tokens, d.k, d.format, d.eps = 1, 576, int(WeightFormat.Q8_0), 1e-5
    d.rows[0], d.rows[1], d.rows[2] = 576, 192, 192
    for i in range(3):
        d.w[i] = FAKE + 4096 * i
        d.y[i] = FAKE + 65536 + 4096 * i
        d.y_stride[i] = 576
    d.x, d.x_stride, d.norm_weight = FAKE + 8192, 576, FAKE + 12288
    for key, v in kw.items():
        setattr(d, key, v)
    return d


def test_decode_project_host_checks(lib):
    """alpaca_decode_project refuses what the kernels cannot serve before enqueueing anything (no GPU needed): formats,
    flags, k (a multiple of 32 up to 16384), row counts, SILU's pairing rules, pointer alignment, strides, eps."""
    from alpaca_b200 import PROJ_ADD, PROJ_NORM, PROJ_SILU, Status

    def st(d):
        return lib.alpaca_decode_project(ctypes.byref(d), None)

    assert st(proj_desc(format=7)) == Status.UNSUPPORTED
    for bad in (dict(flags=8), dict(k=100), dict(k=0), dict(k=32768), dict(n_tokens=0),
                dict(flags=PROJ_NORM, eps=0.0), dict(flags=PROJ_NORM, norm_weight=0), dict(flags=PROJ_SILU | PROJ_ADD),
                dict(x=FAKE + 2), dict(n_tokens=2, x_stride=100)):
        assert st(proj_desc(**bad)) == Status.INVALID_ARGUMENT, bad
    d = proj_desc()
    d.w[1] = FAKE + 8  # not 16-byte aligned
    assert st(d) == Status.INVALID_ARGUMENT
    d = proj_desc(flags=PROJ_SILU)  # SILU: rows[1] and rows[2] must be 0 (W1 has rows[0] rows)
    assert st(d) == Status.INVALID_ARGUMENT
    d = proj_desc()
    d.rows[0] = d.rows[1] = d.rows[2] = 0
    assert st(d) == Status.INVALID_ARGUMENT
    d = proj_desc(n_tokens=2)
    d.y_stride[2] = 100  # smaller than rows[2] = 192
    assert st(d) == Status.INVALID_ARGUMENT
