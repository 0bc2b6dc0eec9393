"""Paged KV cache (block tables) on the GPU through the C ABI.

The cache rows of each sequence live in shuffled blocks of a shared pool whose every other row holds NaN. The split
decode and the tensor-core prefill must give exactly the results of the same call on contiguous caches (same
arithmetic, same order) and match the CPU oracle at the decode / f16 bounds; rows past a context are never read
(the NaNs never reach an output); a block index outside the pool is reported through alpaca_cuda_device_status,
with the rows it names read as zero.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests._util import max_abs_check

pytestmark = pytest.mark.gpu

DECODE_TOL = 1e-5
F16_BOUND = 2e-3


def _pool(caches, block_rows, rng, max_rows, extra_blocks=3):
    """Scatter per-sequence caches [S][rows][Hkv][d] (rows may differ) into a NaN pool of shuffled blocks; the table
    has room for max_rows rows per sequence. Returns (pool, block_table [S, max_blocks] int32 numpy)."""
    S = len(caches)
    Hkv, d = caches[0].shape[1:]
    nblk = [-(-c.shape[0] // block_rows) for c in caches]
    max_blocks = -(-max_rows // block_rows)
    total = sum(nblk) + extra_blocks
    order = rng.permutation(total)
    pool = np.full((total, block_rows, Hkv, d), np.nan, np.float32)
    table = np.full((S, max_blocks), -1, np.int32)
    nxt = 0
    for s, c in enumerate(caches):
        for b in range(nblk[s]):
            blk = int(order[nxt])
            nxt += 1
            table[s, b] = blk
            rows = c[b * block_rows:(b + 1) * block_rows]
            pool[blk, :rows.shape[0]] = rows
    table[table < 0] = int(order[-1])  # unused entries point at a valid (NaN) block
    return pool, table


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
