"""Paged KV cache (block tables) on the GPU through the C ABI.

The cache rows of each sequence live in shuffled blocks of a shared pool whose every other row holds NaN. The split
decode and the tensor-core prefill must give exactly the results of the same call on contiguous caches (same
arithmetic, same order) and match the CPU oracle at the decode / f16 bounds; rows past a context are never read
(the NaNs never reach an output); the RoPE append writes exactly the rows of the contiguous call into the pool; a
block index outside the pool is reported through alpaca_cuda_device_status,
with the rows it names read as zero.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests._util import max_abs_check, pool as _pool

pytestmark = pytest.mark.gpu

DECODE_TOL = 1e-5
F16_BOUND = 2e-3


@pytest.mark.parametrize("d,G,block_rows", [(64, 3, 256), (64, 3, 128), (128, 4, 384)])
def test_paged_decode_matches_contiguous_and_oracle(cuda_lib, d, G, block_rows):
    from alpaca_b200 import Kernel, attention_device, device_status
    S, Hkv, cap = 16, 3 if G == 3 else 2, 1500
    H = G * Hkv
    rng = np.random.default_rng(7 + d + block_rows)
    lens = rng.integers(1, cap + 1, size=S).astype(np.int32)
    q = oracle.splitmix_normal(201, (S, 1, H, d))
    k = oracle.f16_round(oracle.splitmix_normal(202, (S, cap, Hkv, d)))
    v = oracle.f16_round(oracle.splitmix_normal(203, (S, cap, Hkv, d)))
    # the same block assignment for K and V: both pools from identically seeded generators
    kp, table = _pool([k[s, :lens[s]] for s in range(S)], block_rows, np.random.default_rng(17 + d), cap)
    vp, table_v = _pool([v[s, :lens[s]] for s in range(S)], block_rows, np.random.default_rng(17 + d), cap)
    assert np.array_equal(table, table_v)
    dev = torch.device("cuda")
    qd = torch.from_numpy(q).to(dev)
    ld = torch.from_numpy(lens).to(dev)
    out_c = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
    attention_device(qd, torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half(), out_c,
                     ctx_lens=ld, max_ctx_len=cap, kind=Kernel.DECODE_SPLIT)
    out_p = torch.empty_like(out_c)
    attention_device(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out_p,
                     ctx_lens=ld, max_ctx_len=cap, block_table=torch.from_numpy(table).to(dev))
    device_status()
    gp, gc = out_p.cpu().numpy(), out_c.cpu().numpy()
    assert np.array_equal(gp, gc), float(np.abs(gp - gc).max())
    for s in range(S):
        L = int(lens[s])
        ref = oracle.attention(q[s], k[s], v[s], L - 1, length=L)
        max_abs_check(gp[s], ref, DECODE_TOL, f"paged decode d={d} rows/block={block_rows} seq {s} ctx={L}")


@pytest.mark.parametrize("d,block_rows", [(64, 128), (64, 384), (128, 256)])
def test_paged_prefill_matches_contiguous_and_oracle(cuda_lib, d, block_rows):
    """3 sequences, 300 new tokens at position 150 (450 visible rows): the last block of each sequence is partial
    and the pool rows after it are NaN."""
    from alpaca_b200 import Kernel, attention_device, device_status
    S, T, start, H, Hkv = 3, 300, 150, 8, 2
    L = start + T
    rng = np.random.default_rng(11 + d + block_rows)
    q = oracle.f16_round(oracle.splitmix_normal(211, (S, T, H, d)))
    k = oracle.f16_round(oracle.splitmix_normal(212, (S, L, Hkv, d)))
    v = oracle.f16_round(oracle.splitmix_normal(213, (S, L, Hkv, d)))
    kp, table = _pool([k[s] for s in range(S)], block_rows, rng, L)
    vp, table_v = _pool([v[s] for s in range(S)], block_rows, np.random.default_rng(11 + d + block_rows), L)
    assert np.array_equal(table, table_v)
    dev = torch.device("cuda")
    qd = torch.from_numpy(q).to(dev).half()
    out_c = torch.empty((S, T, H, d), dtype=torch.float32, device=dev)
    attention_device(qd, torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half(), out_c,
                     start_position=start, kind=Kernel.PREFILL_TC)
    out_p = torch.empty_like(out_c)
    attention_device(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out_p,
                     start_position=start, block_table=torch.from_numpy(table).to(dev))
    device_status()
    gp, gc = out_p.cpu().numpy(), out_c.cpu().numpy()
    assert np.isfinite(gp).all()
    assert np.array_equal(gp, gc), float(np.abs(gp - gc).max())
    for s in range(S):
        ref = oracle.attention(q[s], k[s], v[s], start)
        max_abs_check(gp[s], ref, F16_BOUND, f"paged prefill d={d} rows/block={block_rows} seq {s}")


@pytest.mark.parametrize("tokens", [1, 64])
def test_block_index_outside_pool_is_reported(cuda_lib, tokens):
    """A table entry past the pool is caught by the kernels' own bounds check: its rows read as zero and
    alpaca_cuda_device_status reports INVALID_ARGUMENT; the next call is unaffected."""
    from alpaca_b200 import AlpacaCUDAError, Status, attention_device, device_status
    S, H, Hkv, d, rows = 2, 4, 2, 64, 128
    dev = torch.device("cuda")
    pool = torch.zeros((4, rows, Hkv, d), dtype=torch.float16, device=dev)
    table = torch.tensor([[0, 1], [2, 4 + 5]], dtype=torch.int32, device=dev)  # sequence 1, block 1: outside
    L = 200
    q = torch.zeros((S, tokens, H, d), dtype=torch.float16, device=dev)
    out = torch.empty((S, tokens, H, d), dtype=torch.float32, device=dev)
    device_status()  # start from a clear error word
    attention_device(q, pool, pool, out, start_position=L - tokens, block_table=table)
    with pytest.raises(AlpacaCUDAError) as e:
        device_status()
    assert e.value.status == Status.INVALID_ARGUMENT
    assert torch.isfinite(out).all()
    table[1, 1] = 3
    attention_device(q, pool, pool, out, start_position=L - tokens, block_table=table)
    device_status()


def _ulps(a: np.ndarray, b: np.ndarray, dt) -> int:
    """Largest distance in units in the last place of dt (float16 or float32)."""
    it, lo = (np.int16, -2 ** 15) if dt == np.float16 else (np.int32, -2 ** 31)
    ai = a.astype(dt).view(it).astype(np.int64)
    bi = b.astype(dt).view(it).astype(np.int64)
    ai = np.where(ai < 0, lo - ai, ai)
    bi = np.where(bi < 0, lo - bi, bi)
    return int(np.abs(ai - bi).max()) if a.size else 0


def _gather(pool: np.ndarray, table: np.ndarray, s: int, rows: int) -> np.ndarray:
    R = pool.shape[1]
    return np.concatenate([pool[table[s, b]] for b in range(-(-rows // R))])[:rows]


@pytest.mark.parametrize("d,cache_f16,block_rows,positions", [
    (64, True, 128, False),    # a 300-token prefill chunk over three blocks, vector kernel
    (64, False, 256, True),    # one new token per sequence at its own position (device positions)
    (12, True, 128, False),    # head_dim % 8 != 0: the scalar kernel
])
def test_paged_rope_append_matches_contiguous(cuda_lib, d, cache_f16, block_rows, positions):
    """RoPE + append into a block pool writes exactly the rows the contiguous call writes (bit-exact), and no pool
    block outside the table changes."""
    from alpaca_b200 import device_status, rope_kv_append
    S, H, Hkv, cap, theta = 4, 6, 2, 640, 1e5
    T = 1 if positions else 300
    rng = np.random.default_rng(31 + d + block_rows)
    pos = rng.integers(0, cap, size=S).astype(np.int32)
    start = 150
    q = oracle.splitmix_normal(301, (S, T, H, d))
    k = oracle.splitmix_normal(302, (S, T, Hkv, d))
    v = oracle.splitmix_normal(303, (S, T, Hkv, d))
    init = oracle.f16_round(oracle.splitmix_normal(304, (S, cap, Hkv, d)))
    kp, table = _pool([init[s] for s in range(S)], block_rows, np.random.default_rng(5 + d), cap)
    vp, _ = _pool([-init[s] for s in range(S)], block_rows, np.random.default_rng(5 + d), cap)
    dev = torch.device("cuda")
    cdt = torch.float16 if cache_f16 else torch.float32
    kd, vd = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
    pd = torch.from_numpy(pos).to(dev) if positions else None
    qc = torch.from_numpy(q).to(dev)
    kc, vc = torch.from_numpy(init).to(dev).to(cdt), torch.from_numpy(-init).to(dev).to(cdt)
    rope_kv_append(qc, kd, vd, kc, vc, theta=theta, start_position=start, positions=pd)
    qp = torch.from_numpy(q).to(dev)
    kpd, vpd = torch.from_numpy(kp).to(dev).to(cdt), torch.from_numpy(vp).to(dev).to(cdt)
    rope_kv_append(qp, kd, vd, kpd, vpd, theta=theta, start_position=start, positions=pd,
                   block_table=torch.from_numpy(table).to(dev))
    device_status()
    assert torch.equal(qp, qc)
    kg, vg = kpd.float().cpu().numpy(), vpd.float().cpu().numpy()
    kcg, vcg = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    for s in range(S):
        assert np.array_equal(_gather(kg, table, s, cap), kcg[s]), f"k seq {s}"
        assert np.array_equal(_gather(vg, table, s, cap), vcg[s]), f"v seq {s}"
    unused = np.setdiff1d(np.arange(kp.shape[0]), table[:, :-(-cap // block_rows)])
    assert np.isnan(kg[unused]).all() and np.isnan(vg[unused]).all()
    if not positions:  # the chunk against the oracle: V exact, K within one ulp (device vs host double cos / sin)
        _, kcr, vcr = oracle.rope_kv_append(q[0].copy(), k[0], v[0], init[0].copy(), -init[0], start, theta, True,
                                            cache_f16)
        assert np.array_equal(_gather(vg, table, 0, cap), vcr)
        assert _ulps(_gather(kg, table, 0, cap), kcr, np.float16 if cache_f16 else np.float32) <= 1


def test_paged_rope_append_then_paged_decode(cuda_lib):
    """The decode step on a paged cache: append the newest token of each sequence into its block, then split-KV
    decode over the pool equals the same two calls on contiguous caches, bit for bit."""
    from alpaca_b200 import Kernel, attention_device, device_status, rope_kv_append
    S, H, Hkv, d, cap, R, theta = 6, 9, 3, 64, 1024, 128, 1e5
    rng = np.random.default_rng(99)
    lens = rng.integers(1, cap + 1, size=S).astype(np.int32)
    init_k = oracle.f16_round(oracle.splitmix_normal(311, (S, cap, Hkv, d)))
    init_v = oracle.f16_round(oracle.splitmix_normal(312, (S, cap, Hkv, d)))
    q = oracle.splitmix_normal(313, (S, 1, H, d))
    k = oracle.splitmix_normal(314, (S, 1, Hkv, d))
    v = oracle.splitmix_normal(315, (S, 1, Hkv, d))
    kp, table = _pool([init_k[s] for s in range(S)], R, np.random.default_rng(3), cap)
    vp, _ = _pool([init_v[s] for s in range(S)], R, np.random.default_rng(3), cap)
    dev = torch.device("cuda")
    pos = torch.from_numpy(lens - 1).to(dev)
    ld = torch.from_numpy(lens).to(dev)
    tab = torch.from_numpy(table).to(dev)
    kd, vd = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
    outs = []
    for paged in (False, True):
        qd = torch.from_numpy(q).to(dev)
        kc = torch.from_numpy(kp if paged else init_k).to(dev).half()
        vc = torch.from_numpy(vp if paged else init_v).to(dev).half()
        rope_kv_append(qd, kd, vd, kc, vc, theta=theta, positions=pos, block_table=tab if paged else None)
        out = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
        attention_device(qd, kc, vc, out, ctx_lens=ld, max_ctx_len=cap, kind=Kernel.DECODE_SPLIT,
                         block_table=tab if paged else None)
        device_status()
        outs.append(out.cpu().numpy())
    assert np.isfinite(outs[1]).all()
    assert np.array_equal(outs[0], outs[1]), float(np.abs(outs[0] - outs[1]).max())


def test_paged_rope_block_outside_pool_is_reported(cuda_lib):
    """A table entry past the pool: the rows it names are not written, q is still rotated, and
    alpaca_cuda_device_status reports INVALID_ARGUMENT; a corrected table then appends normally."""
    from alpaca_b200 import AlpacaCUDAError, Status, device_status, rope_kv_append
    S, H, Hkv, d, R, T = 2, 4, 2, 64, 128, 200
    dev = torch.device("cuda")
    kp = torch.zeros((4, R, Hkv, d), dtype=torch.float16, device=dev)
    vp = torch.zeros_like(kp)
    table = torch.tensor([[0, 1], [2, 4 + 7]], dtype=torch.int32, device=dev)  # sequence 1, block 1: outside
    q = torch.ones((S, T, H, d), device=dev)
    k = torch.ones((S, T, Hkv, d), device=dev)
    v = torch.ones((S, T, Hkv, d), device=dev)
    device_status()
    rope_kv_append(q, k, v, kp, vp, theta=1e4, block_table=table)
    with pytest.raises(AlpacaCUDAError) as e:
        device_status()
    assert e.value.status == Status.INVALID_ARGUMENT
    assert not torch.equal(q, torch.ones_like(q))
    assert torch.all(vp[3] == 0)  # block 3 is in no table row
    assert torch.all(vp[2] == 1) and torch.all(vp[0] == 1) and torch.all(vp[1, :T - R] == 1)
    table[1, 1] = 3
    rope_kv_append(q, k, v, kp, vp, theta=1e4, block_table=table)
    device_status()
    assert torch.all(vp[3, :T - R] == 1)


def test_ctx_len_past_max_is_reported_and_clamped(cuda_lib):
    """A ctx_lens entry above max_ctx_len breaks the caller's contract (the grid and the workspace are sized for
    max_ctx_len): the kernels clamp it, so nothing is read or written past the sequence's records, and
    alpaca_cuda_device_status reports INVALID_ARGUMENT; the other sequences are unaffected. The caches hold the
    longer context, so even an unclamped read would stay inside them."""
    from alpaca_b200 import AlpacaCUDAError, Kernel, Status, attention_device, device_status
    S, H, Hkv, d, cap, mx = 3, 9, 3, 64, 600, 300
    lens = np.array([100, 550, 200], np.int32)
    q = oracle.splitmix_normal(701, (S, 1, H, d))
    k = oracle.f16_round(oracle.splitmix_normal(702, (S, cap, Hkv, d)))
    v = oracle.f16_round(oracle.splitmix_normal(703, (S, cap, Hkv, d)))
    dev = torch.device("cuda")
    out = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
    device_status()
    attention_device(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev).half(),
                     torch.from_numpy(v).to(dev).half(), out, ctx_lens=torch.from_numpy(lens).to(dev),
                     max_ctx_len=mx, kind=Kernel.DECODE_SPLIT)
    with pytest.raises(AlpacaCUDAError) as e:
        device_status()
    assert e.value.status == Status.INVALID_ARGUMENT
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    for s in (0, 2):
        L = int(lens[s])
        ref = oracle.attention(q[s], k[s], v[s], L - 1, length=L)
        max_abs_check(got[s], ref, DECODE_TOL, f"ctx_len clamp, unaffected seq {s}")
    ref1 = oracle.attention(q[1], k[1], v[1], mx - 1, length=mx)  # the offending sequence: clamped to max_ctx_len
    max_abs_check(got[1], ref1, DECODE_TOL, "ctx_len clamp, clamped seq")


def test_rope_position_past_cache_is_reported(cuda_lib):
    """A device position at or past the contiguous cache's rows writes no cache row and is reported; the rows of the
    in-range sequence are written. The caches are 16-row views of 64-row buffers, so the row an unchecked kernel
    would write exists and can be checked untouched."""
    from alpaca_b200 import AlpacaCUDAError, Status, device_status, rope_kv_append
    S, H, Hkv, d = 2, 4, 2, 64
    dev = torch.device("cuda")
    kb = torch.full((S, 64, Hkv, d), 7.0, dtype=torch.float16, device=dev)
    vb = torch.full_like(kb, 7.0)
    kc, vc = kb[:, :16], vb[:, :16]
    q = torch.ones((S, 1, H, d), device=dev)
    k = torch.ones((S, 1, Hkv, d), device=dev)
    v = torch.ones((S, 1, Hkv, d), device=dev)
    pos = torch.tensor([3, 40], dtype=torch.int32, device=dev)
    device_status()
    rope_kv_append(q, k, v, kc, vc, theta=1e4, positions=pos)
    with pytest.raises(AlpacaCUDAError) as e:
        device_status()
    assert e.value.status == Status.INVALID_ARGUMENT
    assert torch.all(vb[0, 3] == 1) and torch.all(vb[1, 40] == 7) and torch.all(kb[1, 40] == 7)
    assert not torch.equal(q[1], torch.ones_like(q[1]))  # q is rotated regardless
