"""Shared test helpers: the reference's element-wise comparison and metric printing."""
from __future__ import annotations

import numpy as np

import oracle


def compare(actual, expected, atol: float, rtol: float, label: str) -> dict:
    """KernelTests.compare (Tests/AlpacaMetalTests/KernelTests.swift:30-36): every element must satisfy
    |a - e| <= atol + rtol * |e|. Prints the [metrics] line and returns the ErrorMetrics."""
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    m = oracle.error_metrics(a, e)
    print(f"[metrics] {label}: {oracle.format_metrics(m)}")
    assert np.all(np.isfinite(a)), f"{label}: non-finite output"
    bad = np.abs(a.astype(np.float64) - e) > atol + rtol * np.abs(e)
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"{label}[{i}] gpu {a[i]} cpu {e[i]} (atol {atol}, rtol {rtol}); {oracle.format_metrics(m)}")
    return m


def max_abs_check(actual, expected, bound: float, label: str) -> dict:
    a = np.asarray(actual, np.float32).reshape(-1)
    m = oracle.error_metrics(a, np.asarray(expected, np.float64).reshape(-1))
    print(f"[metrics] {label}: {oracle.format_metrics(m)}")
    assert np.all(np.isfinite(a)), f"{label}: non-finite output"
    assert m["maxAbs"] < bound, f"{label}: maxAbs {m['maxAbs']:.3e} >= {bound:.1e}"
    return m


def pool(caches, block_rows, rng, max_rows, extra_blocks=3):
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


def prefill_unsplit(q, k, v, out, start_position: int = 0):
    """A uniform tensor-core prefill given only its minimum workspace (the f32 queries' staging), so the library runs
    it unsplit: one work item per (sequence, head, pair of query tiles) over the whole KV range, the arithmetic the
    ragged form shares bit for bit (a split-KV call sums its parts in another order)."""
    import torch

    import alpaca_b200 as ab
    desc = ab.make_desc(q, k, v, out, start_position=start_position)
    n = 1
    for x in q.shape[:-1]:
        n *= x
    minimum = (n * q.shape[-1] * 2 + 15) // 16 * 16 if q.dtype == torch.float32 else 0
    ws = torch.empty(minimum, dtype=torch.uint8, device=q.device) if minimum else None
    ab.launch(desc, ab.Kernel.PREFILL_TC, ws)


def varlen_unsplit(q, k, v, out, q_offsets, start_positions, *, max_tokens: int, max_ctx_len: int):
    """A ragged prefill given only its minimum workspace (the f32 queries' staging and the work list), so the library
    runs it unsplit (see prefill_unsplit)."""
    import torch

    import alpaca_b200 as ab
    desc = ab.make_varlen_desc(q, k, v, out, q_offsets, start_positions, max_tokens=max_tokens,
                               max_ctx_len=max_ctx_len)
    units = (q_offsets.numel() - 1) * -(-max_tokens // 256)
    stage = (q.shape[0] * q.shape[1] * q.shape[2] * 2 + 15) // 16 * 16 if q.dtype == torch.float32 else 0
    ws = torch.empty(stage + 16 * (1 + 2 * units), dtype=torch.uint8, device=q.device)
    ab.launch(desc, ab.Kernel.PREFILL_TC, ws)
