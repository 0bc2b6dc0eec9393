"""alpaca_attn_decode_noalloc: the decode entry point that allocates nothing.

Some callers cannot call cudaMalloc or hand the library a scratch buffer — a host runtime that owns every device
allocation through a fixed memory plan, or code running where allocation is not allowed. For them the library
keeps the split-decode scratch in a built-in device array. This test first fills that array's split records with NaN
(a call whose queries are NaN), then enqueues two such calls back to back on one stream with no synchronisation in
between (different sequences, context lengths and split counts, so the second call runs over split records the first
one left in the shared array): a record read before the call wrote it would show as NaN. It checks each output
against the existing workspace entry point, alpaca_attn_decode, and every sequence against the CPU oracle, within
the decode tolerance the other tests use. It also checks that a call needing more split scratch than the built-in 8 MiB is rejected
before anything is enqueued.

The file name makes pytest collect it last; it passes alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from tests._util import max_abs_check

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DECODE_TOL = 1e-5  # max-abs bound of the decode parity tests (tests/test_gpu_parity.py, config 3)
H, KVH, D = 9, 3, 64


def _case(seed: int, S: int, cap: int):
    """Host f32 inputs (f16-representable K/V) and ragged context lengths in [1, cap]."""
    q = oracle.splitmix_normal(seed, (S, 1, H, D))
    k = oracle.f16_round(oracle.splitmix_normal(seed + 1, (S, cap, KVH, D)))
    v = oracle.f16_round(oracle.splitmix_normal(seed + 2, (S, cap, KVH, D)))
    lens = np.random.default_rng(seed).integers(1, cap + 1, size=S).astype(np.int32)
    lens[0] = cap  # one sequence uses every split
    return q, k, v, lens


def test_decode_noalloc_matches_workspace_entry_point(cuda_lib):
    import alpaca_b200 as ab
    lib = cuda_lib
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    cases = []
    for seed, S, cap in [(101, 64, 4096), (202, 37, 1500)]:
        q, k, v, lens = _case(seed, S, cap)
        dev = dict(q=torch.from_numpy(q).cuda(), k=torch.from_numpy(k).cuda().half(),
                   v=torch.from_numpy(v).cuda().half(), lens=torch.from_numpy(lens).cuda())
        ref = torch.empty((S, 1, H, D), dtype=torch.float32, device="cuda")
        got = torch.full((S, 1, H, D), float("nan"), dtype=torch.float32, device="cuda")
        # the existing entry point, with a caller workspace
        dref = ab.make_desc(dev["q"], dev["k"], dev["v"], ref, ctx_lens=dev["lens"], max_ctx_len=cap)
        need = ab.workspace_bytes(dref, ab.Kernel.DECODE_SPLIT)
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
        st = lib.alpaca_attn_decode(ctypes.byref(dref), ctypes.c_void_p(ws.data_ptr()), need, sp)
        assert st == ab.Status.OK, lib.alpaca_cuda_last_error()
        ab.device_status()
        dnew = ab.make_desc(dev["q"], dev["k"], dev["v"], got, ctx_lens=dev["lens"], max_ctx_len=cap)
        cases.append((q, k, v, lens, dev, ref, got, dnew))

    # A first call with NaN queries fills the split records of the built-in array (64 sequences x 4096 rows covers
    # every record the two calls below use) with NaN, so a record that either call read without writing it first
    # would turn its output into NaN.
    S0, cap0 = 64, 4096
    pq = torch.full((S0, 1, H, D), float("nan"), dtype=torch.float32, device="cuda")
    pkv = torch.zeros((S0, cap0, KVH, D), dtype=torch.float16, device="cuda")
    pout = torch.empty((S0, 1, H, D), dtype=torch.float32, device="cuda")
    plens = torch.full((S0,), cap0, dtype=torch.int32, device="cuda")
    dpoison = ab.make_desc(pq, pkv, pkv, pout, ctx_lens=plens, max_ctx_len=cap0)
    assert lib.alpaca_attn_decode_noalloc(ctypes.byref(dpoison), sp) == ab.Status.OK, lib.alpaca_cuda_last_error()

    # the no-allocation entry point: both calls enqueued back to back, one synchronisation
    for c in cases:
        st = lib.alpaca_attn_decode_noalloc(ctypes.byref(c[-1]), sp)
        assert st == ab.Status.OK, lib.alpaca_cuda_last_error()
    ab.device_status()

    for call, (q, k, v, lens, _, ref, got, _) in enumerate(cases):
        diff = float((got - ref).abs().max().item())
        print(f"[metrics] decode_noalloc call {call}: seqs={lens.size} max ctx={int(lens.max())} "
              f"max-abs vs alpaca_attn_decode {diff:.3e}")
        assert np.isfinite(diff) and diff <= DECODE_TOL
        g = got.cpu().numpy()
        for s in range(lens.size):
            L = int(lens[s])
            cpu = oracle.attention(q[s], k[s], v[s], L - 1, length=L)
            max_abs_check(g[s], cpu, DECODE_TOL, f"decode_noalloc call {call} seq {s} ctx={L} vs oracle")


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
