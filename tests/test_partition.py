"""Multi-GPU split of the attention path, on CPU.

Host logic: every (sequence, KV-head) unit is assigned exactly once, deterministically, with the LPT load balance.
Two `gloo` ranks then run their units with the CPU oracle (standing in for the per-GPU kernel) and all-gather the
results; the gathered output must equal a one-process run bit for bit, which is the property the GPU scaling run
relies on (no exchange step, results independent of the split).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from alpaca_b200.partition import Unit, head_ranges, partition, units_for_batch


def test_every_unit_assigned_once_and_deterministic():
    rng = np.random.default_rng(0)
    toks = [int(x) for x in np.round(np.exp(rng.uniform(np.log(128), np.log(8192), 256)))] + [1] * 512
    starts = [0] * 256 + [int(x) for x in rng.integers(0, 8192, 512)]
    units = units_for_batch(toks, starts, 32, 32)
    for n in (1, 2, 4, 8):
        p1, p2 = partition(units, n), partition(units, n)
        assert [[(u.seq, u.kv_head) for u in r] for r in p1.ranks] == [[(u.seq, u.kv_head) for u in r] for r in p2.ranks]
        flat = sorted((u.seq, u.kv_head) for r in p1.ranks for u in r)
        assert flat == sorted((u.seq, u.kv_head) for u in units)
        assert p1.imbalance < 1.02, (n, p1.imbalance)


def test_lpt_bound_and_uniform_batches():
    # 8 equal sequences x 5 KV heads over 1/2/4/8 ranks (config 4 shape): perfect balance when units divide evenly
    units = units_for_batch([4096] * 8, [0] * 8, 15, 5)
    for n in (1, 2, 4, 8):
        p = partition(units, n)
        assert max(len(r) for r in p.ranks) == len(units) // n
        assert p.imbalance == pytest.approx(1.0)
    # LPT guarantee: max load <= 4/3 of the optimum lower bound (max(mean, largest unit)) + one unit
    rng = np.random.default_rng(1)
    units = [Unit(i, 0, int(t), 0, 1) for i, t in enumerate(rng.integers(1, 4096, 37))]
    p = partition(units, 8)
    lb = max(sum(u.cost() for u in units) / 8, max(u.cost() for u in units))
    assert max(p.loads) <= 4 / 3 * lb + 1e-12


def test_unit_cost_model():
    u = Unit(0, 0, tokens=4096, start=0, group=3)
    assert u.flops == pytest.approx(3 * 2 * 64 * 4096 * 4097)  # 2*G*d*T*(T+1)
    d = Unit(0, 0, tokens=1, start=2047, group=3)
    assert d.kv_bytes == 2048 * 64 * 4
    assert d.cost() == pytest.approx(d.kv_bytes / 6000e9)       # decode is HBM-bound


def test_head_ranges_collapse_consecutive_heads():
    units = [Unit(0, h, 8, 0, 2) for h in (0, 1, 2, 5)] + [Unit(3, 1, 8, 0, 2)]
    assert head_ranges(units) == [(0, 0, 3), (0, 5, 1), (3, 1, 1)]


# ------------------------------------------------------------------------------------------- gloo world size 2

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q, k, v, starts, H, kvh, out_path):
    import torch
    import torch.distributed as dist

    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    S, T, _, d = q.shape
    units = units_for_batch([T] * S, starts, H, kvh)
    plan = partition(units, world)
    G = H // kvh
    mine = np.zeros_like(q)
    mask = np.zeros(q.shape[:3], bool)
    for s, h0, n in head_ranges(plan.ranks[rank]):
        hs = slice(h0 * G, (h0 + n) * G)
        L = starts[s] + T
        res = oracle.attention(np.ascontiguousarray(q[s][:, hs]), np.ascontiguousarray(k[s][:L, h0:h0 + n]),
                               np.ascontiguousarray(v[s][:L, h0:h0 + n]), starts[s])
        mine[s][:, hs] = res
        mask[s][:, hs] = True
    t_out, t_mask = torch.from_numpy(mine), torch.from_numpy(mask)
    outs = [torch.zeros_like(t_out) for _ in range(world)]
    masks = [torch.zeros_like(t_mask) for _ in range(world)]
    dist.all_gather(outs, t_out)
    dist.all_gather(masks, t_mask)
    if rank == 0:
        total = np.zeros_like(q)
        cover = np.zeros(q.shape[:3], np.int32)
        for o, m in zip(outs, masks):
            total[m.numpy()] = o.numpy()[m.numpy()]
            cover += m.numpy().astype(np.int32)
        np.savez(out_path, out=total, cover=cover)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_single_process(tmp_path):
    import torch.multiprocessing as mp

    import oracle
    S, T, H, kvh, d = 3, 20, 6, 3, 32
    starts = [0, 5, 11]
    q = oracle.splitmix_normal(1, (S, T, H, d))
    k = oracle.splitmix_normal(2, (S, T + 11, kvh, d))
    v = oracle.splitmix_normal(3, (S, T + 11, kvh, d))
    out_path = str(tmp_path / "gathered.npz")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, k, v, starts, H, kvh, out_path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    res = np.load(out_path)
    assert np.all(res["cover"] == 1)  # every (seq, token, head) produced by exactly one rank
    ref = np.stack([oracle.attention(q[s], k[s], v[s], starts[s], length=starts[s] + T) for s in range(S)])
    assert np.array_equal(res["out"], ref)


def test_head_group_units_cost_and_balance():
    """Config-5-shaped batch split into units of 8 KV heads: every (sequence, head group) once, costs 8 heads' worth,
    and the LPT split over 8 ranks stays within 1% of the mean."""
    from alpaca_b200.partition import head_group_units
    rng = np.random.default_rng(20260105)
    toks = [int(x) for x in np.round(np.exp(rng.uniform(np.log(128), np.log(8192), 256)))]
    units = head_group_units(toks, [0] * 256, 32, 8) + \
        head_group_units([1] * 512, [int(x) for x in rng.integers(0, 8192, 512)], 32, 8, first_seq=256)
    assert len(units) == (256 + 512) * 4
    one = Unit(0, 0, toks[0], 0, 1)
    assert units[0].flops == pytest.approx(8 * one.flops) and units[0].kv_bytes == pytest.approx(8 * one.kv_bytes)
    for n in (1, 2, 4, 8):
        p = partition(units, n)
        assert sorted((u.seq, u.kv_head) for r in p.ranks for u in r) == sorted((u.seq, u.kv_head) for u in units)
        assert p.imbalance < 1.01, (n, p.imbalance)
    with pytest.raises(ValueError):
        head_group_units([8], [0], 32, 5)


def test_head_ranges_of_head_group_units():
    from alpaca_b200.partition import head_group_units
    units = [u for u in head_group_units([8, 8], [0, 0], 32, 8) if (u.seq, u.kv_head) != (0, 16)]
    assert head_ranges(units) == [(0, 0, 16), (0, 24, 8), (1, 0, 32)]
