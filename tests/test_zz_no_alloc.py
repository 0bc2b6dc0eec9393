"""alpaca_attn_decode_noalloc: the decode entry point that allocates nothing.

Some callers cannot call cudaMalloc or hand the library a scratch buffer — a host runtime that owns every device
allocation through a fixed memory plan, or code running where allocation is not allowed. For them the library
keeps the split-decode scratch in a built-in device array. This test calls that entry point through the C ABI
twice in a row (different inputs and context lengths each time, so stale scratch from the first call would show)
and checks each result against the existing workspace entry point, alpaca_attn_decode, within the decode
tolerance the other tests use. It also checks that a call needing more split scratch than the built-in 8 MiB is
rejected before anything is enqueued.

The file name makes pytest collect it last; it passes alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DECODE_TOL = 1e-5  # max-abs bound of the decode parity tests (tests/test_gpu_parity.py, config 3)


def _case(seed: int, S: int, cap: int, H: int = 9, kvh: int = 3, d: int = 64):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((S, 1, H, d), generator=g, device="cuda")
    k = torch.randn((S, cap, kvh, d), generator=g, device="cuda").half()
    v = torch.randn((S, cap, kvh, d), generator=g, device="cuda").half()
    gl = torch.Generator()
    gl.manual_seed(seed)
    lens = torch.randint(1, cap + 1, (S,), generator=gl, dtype=torch.int32).cuda()
    return q, k, v, lens


def test_decode_noalloc_matches_workspace_entry_point(cuda_lib):
    import alpaca_b200 as ab
    lib = cuda_lib
    stream = torch.cuda.current_stream()
    for call, (seed, S, cap) in enumerate([(101, 64, 4096), (202, 37, 1500)]):
        q, k, v, lens = _case(seed, S, cap)
        ref = torch.empty((S, 1, 9, 64), dtype=torch.float32, device="cuda")
        got = torch.full((S, 1, 9, 64), float("nan"), dtype=torch.float32, device="cuda")

        # existing entry point, with a caller workspace
        dref = ab.make_desc(q, k, v, ref, ctx_lens=lens, max_ctx_len=cap)
        need = ab.workspace_bytes(dref, ab.Kernel.DECODE_SPLIT)
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
        st = lib.alpaca_attn_decode(ctypes.byref(dref), ctypes.c_void_p(ws.data_ptr()), need,
                                    ctypes.c_void_p(stream.cuda_stream))
        assert st == ab.Status.OK, lib.alpaca_cuda_last_error()

        # the no-allocation entry point
        dnew = ab.make_desc(q, k, v, got, ctx_lens=lens, max_ctx_len=cap)
        st = lib.alpaca_attn_decode_noalloc(ctypes.byref(dnew), ctypes.c_void_p(stream.cuda_stream))
        assert st == ab.Status.OK, lib.alpaca_cuda_last_error()
        ab.device_status()

        diff = float((got - ref).abs().max().item())
        print(f"[metrics] decode_noalloc call {call}: seqs={S} max ctx={cap} max-abs vs alpaca_attn_decode {diff:.3e}")
        assert np.isfinite(diff) and diff <= DECODE_TOL


def test_decode_noalloc_rejects_oversized_scratch(cuda_lib):
    import alpaca_b200 as ab
    lib = cuda_lib
    # 512 sequences of up to 8192 positions at 32/32 heads: 512*32*64*66*4 bytes of split state > 8 MiB
    S, cap, H, d = 512, 8192, 32, 64
    q = torch.zeros((S, 1, H, d), dtype=torch.float32, device="cuda")
    kv = torch.zeros((S, 16, H, d), dtype=torch.float16, device="cuda")  # never read: the call is refused first
    out = torch.zeros((S, 1, H, d), dtype=torch.float32, device="cuda")
    lens = torch.ones((S,), dtype=torch.int32, device="cuda")
    desc = ab.make_desc(q, kv, kv, out, ctx_lens=lens, max_ctx_len=cap)
    st = lib.alpaca_attn_decode_noalloc(ctypes.byref(desc), None)
    assert st == ab.Status.WORKSPACE_TOO_SMALL
    assert b"8388608" in lib.alpaca_cuda_last_error()
