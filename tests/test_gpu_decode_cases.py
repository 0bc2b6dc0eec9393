"""Split-KV decode edge cases against the CPU oracle, through the C ABI.

Batches that stress the split grid's corners beyond config 3 / config 5: one long sequence whose many splits all
meet in the combine, many 1-40 row sequences (finished by the split kernel itself) next to long ones, every GQA
ratio 1..8 with lengths on the 128-row split boundaries, f16 queries and f16 output, a shuffled paged pool with NaN
rows past every context, and 1100 sequences in one call.

Bounds: f32 queries over the f16 cache within max-abs 1e-5 of the oracle (config 3's bound; the split-decode
cases of KernelTests.swift:124-144 keep their 2e-6 in tests/test_gpu_parity.py); f16 queries are rounded the same
way for the oracle; f16 output within 2e-3 (one f16 rounding of values of magnitude < 4).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests._util import max_abs_check, pool

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

D = 64


def _caches(seed: int, lens, hkv: int):
    ks = [oracle.f16_round(oracle.splitmix_normal(seed + 2 * s, (int(L), hkv, D))) for s, L in enumerate(lens)]
    vs = [oracle.f16_round(oracle.splitmix_normal(seed + 2 * s + 1, (int(L), hkv, D))) for s, L in enumerate(lens)]
    return ks, vs


def _run(lens, heads, hkv, seed, *, q_f16=False, out_f16=False, paged=False, uniform=False, cap=None):
    from alpaca_b200 import Kernel, attention_device, device_status
    lens = np.asarray(lens, np.int32)
    S = lens.size
    cap = int(cap or lens.max())
    q = oracle.splitmix_normal(seed, (S, 1, heads, D))
    if q_f16:
        q = oracle.f16_round(q)
    ks, vs = _caches(seed + 100, lens, hkv)
    dev = torch.device("cuda")
    qd = torch.from_numpy(q).to(dev)
    if q_f16:
        qd = qd.half()
    out = torch.full((S, 1, heads, D), float("nan"), dtype=torch.float16 if out_f16 else torch.float32, device=dev)
    kw = {} if uniform else {"ctx_lens": torch.from_numpy(lens).to(dev), "max_ctx_len": cap}
    if paged:
        kp, table = pool(ks, 256, np.random.default_rng(seed), cap)
        vp, table_v = pool(vs, 256, np.random.default_rng(seed), cap)
        assert np.array_equal(table, table_v)
        attention_device(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out,
                         kind=Kernel.DECODE_SPLIT, block_table=torch.from_numpy(table).to(dev), **kw)
    else:
        kd = torch.full((S, cap, hkv, D), float("nan"), dtype=torch.float16, device=dev)
        vd = torch.full((S, cap, hkv, D), float("nan"), dtype=torch.float16, device=dev)
        for s, L in enumerate(lens):
            kd[s, :L] = torch.from_numpy(ks[s]).to(dev).half()
            vd[s, :L] = torch.from_numpy(vs[s]).to(dev).half()
        if uniform:
            attention_device(qd, kd, vd, out, start_position=cap - 1, kind=Kernel.DECODE_SPLIT)
        else:
            attention_device(qd, kd, vd, out, kind=Kernel.DECODE_SPLIT, **kw)
    device_status()
    got = out.float().cpu().numpy()
    bound = 2e-3 if out_f16 else 1e-5
    for s, L in enumerate(lens):
        L = int(L)
        ref = oracle.attention(q[s], ks[s], vs[s], L - 1, length=L)
        max_abs_check(got[s], ref, bound, f"decode H={heads}/{hkv} seq {s} ctx={L}"
                      f"{' q16' if q_f16 else ''}{' o16' if out_f16 else ''}{' paged' if paged else ''}")


def test_one_long_sequence_many_splits(cuda_lib):
    """One 16384-row sequence at 9/3 heads, same length for the call (no ctx_lens): 128 splits per KV head meet in
    the combine (more than one staging round of split states)."""
    _run([16384], 9, 3, 11, uniform=True)


def test_uniform_batch_32_heads(cuda_lib):
    """Eight sequences of 3001 rows, uniform length (ctx_lens absent), 32/32 heads (G = 1)."""
    _run([3001] * 8, 32, 32, 21, uniform=True)


@pytest.mark.parametrize("heads,hkv", [(4, 4), (8, 4), (9, 3), (12, 3), (10, 2), (12, 2), (14, 2), (8, 1)],
                         ids=lambda x: str(x))
def test_gqa_ratios_mixed_lengths(cuda_lib, heads, hkv):
    """GQA 1..8 over a ragged batch mixing 1-row, split-boundary and long contexts."""
    rng = np.random.default_rng(heads * 10 + hkv)
    lens = [1, 2, 127, 128, 129, 255, 256, 257] + list(rng.integers(1, 4097, 8))
    _run(lens, heads, hkv, 31 + heads)


def test_many_short_sequences_beside_long_ones(cuda_lib):
    """600 sequences of 1-40 rows (one split each, finished in the split kernel) around three long ones at the
    start, middle and end of the batch."""
    rng = np.random.default_rng(7)
    lens = list(rng.integers(1, 41, 600))
    lens[0], lens[300], lens[599] = 5000, 2049, 8192
    _run(lens, 9, 3, 41)


@pytest.mark.parametrize("q_f16,out_f16", [(True, False), (False, True), (True, True)], ids=["q16", "o16", "q16o16"])
def test_f16_query_and_output(cuda_lib, q_f16, out_f16):
    rng = np.random.default_rng(3)
    _run(list(rng.integers(1, 3000, 24)) + [4096], 9, 3, 51, q_f16=q_f16, out_f16=out_f16)


def test_paged_pool_with_nan_tails(cuda_lib):
    """Shuffled 256-row blocks whose rows past each context (and unused blocks) are NaN, 15/5 heads."""
    rng = np.random.default_rng(9)
    lens = [1, 129, 256, 257, 4096] + list(rng.integers(1, 4097, 20))
    _run(lens, 15, 5, 61, paged=True, cap=4096)


def test_eleven_hundred_sequences(cuda_lib):
    """1100 sequences in one call (grid y extent and per-sequence records well past config 5's 512)."""
    rng = np.random.default_rng(13)
    lens = list(rng.integers(1, 300, 1100))
    _run(lens, 4, 2, 71)
