"""BASELINE config 5's shape on the GPU: SmolLM2-1.7B attention (32 query heads over 32 KV heads, so G = 1,
head_dim 64), prefill sequences up to 8192 tokens and a ragged decode batch over caches of up to 8192 rows, each in
contiguous caches and in a shuffled pool of 256-row blocks (the serving layout the config-5 bench runs on).

Bounds as in the other parity tests: f16 Q/K/V prefill within max-abs 2e-3 of the oracle fed the same f16-rounded
inputs, f32-query decode over the f16 cache within 1e-5. Prefill rows are checked on a sample (rows are independent,
so each sampled row is an exact check) that always includes the first and last token of every head. The shape matrix
follows the reference's own choice of covering every GQA ratio and split boundary
(Tests/AlpacaMetalTests/KernelTests.swift:124-170): the decode lengths sit on the 128-row split boundaries and span
one to 64 splits.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests._util import max_abs_check, pool

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H = HKV = 32
D = 64
F16_BOUND = 2e-3
DECODE_TOL = 1e-5
BLOCK_ROWS = 256
PREFILL_T = (128, 3000, 8192)
DECODE_LENS = (1, 127, 128, 129, 4097, 8192)


def _sample_rows(T: int, step: int) -> np.ndarray:
    """(head, token) rows h*T + t: every `step`-th one plus tokens 0 and T-1 of every head."""
    ends = np.concatenate([np.arange(H) * T, np.arange(H) * T + T - 1])
    return np.unique(np.concatenate([np.arange(0, H * T, step), ends]))


def _prefill_inputs(T: int, seed: int):
    q = oracle.f16_round(oracle.splitmix_normal(seed, (T, H, D)))
    k = oracle.f16_round(oracle.splitmix_normal(seed + 1, (T, HKV, D)))
    v = oracle.f16_round(oracle.splitmix_normal(seed + 2, (T, HKV, D)))
    return q, k, v


@pytest.mark.parametrize("paged", [False, True], ids=["contiguous", "paged"])
def test_config5_prefill_32_heads(cuda_lib, paged):
    """Prefill of 128, 3000 and 8192 tokens at 32/32 heads through the tensor-core kernel; the paged form reads K/V
    from shuffled 256-row blocks of a pool whose unused rows are NaN, and equals the contiguous call bit for bit."""
    from alpaca_b200 import Kernel, attention_device, device_status
    dev = torch.device("cuda")
    for i, T in enumerate(PREFILL_T):
        q, k, v = _prefill_inputs(T, 500 + 10 * i)
        qd = torch.from_numpy(q).to(dev).half()
        kd, vd = torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half()
        out = torch.empty((T, H, D), dtype=torch.float32, device=dev)
        attention_device(qd, kd, vd, out, kind=Kernel.PREFILL_TC)
        if paged:
            kp, table = pool([k], BLOCK_ROWS, np.random.default_rng(T), T)
            vp, table_v = pool([v], BLOCK_ROWS, np.random.default_rng(T), T)
            assert np.array_equal(table, table_v)
            out_p = torch.empty_like(out)
            attention_device(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out_p,
                             kind=Kernel.PREFILL_TC, block_table=torch.from_numpy(table).to(dev))
            device_status()
            assert torch.equal(out_p, out)
            out = out_p
        device_status()
        rows = _sample_rows(T, 97 if T > 4096 else 23)
        cpu = oracle.attention_rows(q, k, v, 0, rows)
        sel = oracle.rows_mask(rows, T, H)
        got = out.cpu().numpy()
        max_abs_check(got[sel], cpu[sel], F16_BOUND, f"config 5 prefill T={T} {'paged' if paged else 'contiguous'}")
        last = oracle.attention_rows(q, k, v, 0, [h * T + T - 1 for h in range(H)])
        max_abs_check(got[T - 1], last[T - 1], F16_BOUND, f"config 5 prefill T={T} last token, every head")


@pytest.mark.parametrize("paged", [False, True], ids=["contiguous", "paged"])
def test_config5_decode_ragged_32_heads(cuda_lib, paged):
    """Ragged one-token decode at 32/32 heads over caches of up to 8192 rows: 18 sequences, lengths on the split
    boundaries (1, 127, 128, 129, 4097, 8192) plus 12 drawn from U[1, 8192]; rows past each context are NaN."""
    from alpaca_b200 import Kernel, attention_device, device_status
    cap = 8192
    rng = np.random.default_rng(20260105)
    lens = np.array(list(DECODE_LENS) + list(rng.integers(1, cap + 1, 12)), np.int32)
    S = lens.size
    q = oracle.splitmix_normal(601, (S, 1, H, D))
    ks = [oracle.f16_round(oracle.splitmix_normal(700 + s, (int(L), HKV, D))) for s, L in enumerate(lens)]
    vs = [oracle.f16_round(oracle.splitmix_normal(800 + s, (int(L), HKV, D))) for s, L in enumerate(lens)]
    dev = torch.device("cuda")
    ld = torch.from_numpy(lens).to(dev)
    qd = torch.from_numpy(q).to(dev)
    out = torch.empty((S, 1, H, D), dtype=torch.float32, device=dev)
    if paged:
        kp, table = pool(ks, BLOCK_ROWS, np.random.default_rng(5), cap)
        vp, table_v = pool(vs, BLOCK_ROWS, np.random.default_rng(5), cap)
        assert np.array_equal(table, table_v)
        kd, vd = torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half()
        del kp, vp
        attention_device(qd, kd, vd, out, ctx_lens=ld, max_ctx_len=cap, block_table=torch.from_numpy(table).to(dev))
    else:
        kd = torch.full((S, cap, HKV, D), float("nan"), dtype=torch.float16, device=dev)
        vd = torch.full((S, cap, HKV, D), float("nan"), dtype=torch.float16, device=dev)
        for s, L in enumerate(lens):
            kd[s, :L] = torch.from_numpy(ks[s]).to(dev).half()
            vd[s, :L] = torch.from_numpy(vs[s]).to(dev).half()
        attention_device(qd, kd, vd, out, ctx_lens=ld, max_ctx_len=cap, kind=Kernel.DECODE_SPLIT)
    device_status()
    got = out.cpu().numpy()
    for s, L in enumerate(lens):
        L = int(L)
        ref = oracle.attention(q[s], ks[s], vs[s], L - 1, length=L)
        max_abs_check(got[s], ref, DECODE_TOL,
                      f"config 5 decode seq {s} ctx={L} {'paged' if paged else 'contiguous'}")


def test_config5_dispatch_policy(cuda_lib):
    """The AUTO policy at config 5's shape: G = 1 is within the split decode's group limit, so one-token calls take
    the split decode and multi-token calls the tensor-core prefill (KernelEncoder.swift:306-343)."""
    import alpaca_b200 as ab
    dev = torch.device("cuda")
    q1 = torch.zeros((4, 1, H, D), dtype=torch.float32, device=dev)
    qT = torch.zeros((1, 300, H, D), dtype=torch.float16, device=dev)
    kv = torch.zeros((4, 512, HKV, D), dtype=torch.float16, device=dev)
    lens = torch.full((4,), 300, dtype=torch.int32, device=dev)
    assert ab.select_kernel(ab.make_desc(q1, kv, kv, q1, ctx_lens=lens, max_ctx_len=512)) == ab.Kernel.DECODE_SPLIT
    assert ab.select_kernel(ab.make_desc(qT, kv[:1], kv[:1], qT.float())) == ab.Kernel.PREFILL_TC


@pytest.mark.parametrize("paged", [False, True], ids=["contiguous", "paged"])
def test_config5_prefill_one_ragged_call(cuda_lib, paged):
    """The three prefill sequences (128, 3000 and 8192 tokens) in one ragged launch: packed queries, one cache (or
    block table) per sequence. Every output row equals the per-sequence uniform call bit for bit, and sampled rows,
    the last token of every head included, match the oracle."""
    from alpaca_b200 import Kernel, attention_device, device_status, prefill_varlen
    dev = torch.device("cuda")
    ins = [_prefill_inputs(T, 500 + 10 * i) for i, T in enumerate(PREFILL_T)]
    lens = np.array(PREFILL_T, np.int32)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    cap = int(lens.max())
    qd = torch.from_numpy(np.concatenate([x[0] for x in ins])).to(dev).half()
    out = torch.empty((int(offs[-1]), H, D), dtype=torch.float32, device=dev)
    starts = torch.zeros(len(PREFILL_T), dtype=torch.int32, device=dev)
    if paged:
        kp, table = pool([x[1] for x in ins], BLOCK_ROWS, np.random.default_rng(77), cap)
        vp, _ = pool([x[2] for x in ins], BLOCK_ROWS, np.random.default_rng(77), cap)
        prefill_varlen(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out,
                       torch.from_numpy(offs).to(dev), starts, max_tokens=cap, max_ctx_len=cap,
                       block_table=torch.from_numpy(table).to(dev))
    else:
        kd = torch.full((len(ins), cap, HKV, D), float("nan"), dtype=torch.float16, device=dev)
        vd = torch.full_like(kd, float("nan"))
        for s, x in enumerate(ins):
            kd[s, :x[1].shape[0]] = torch.from_numpy(x[1]).to(dev).half()
            vd[s, :x[2].shape[0]] = torch.from_numpy(x[2]).to(dev).half()
        prefill_varlen(qd, kd, vd, out, torch.from_numpy(offs).to(dev), starts, max_tokens=cap, max_ctx_len=cap)
    device_status()
    for s, (T, (q, k, v)) in enumerate(zip(PREFILL_T, ins)):
        o0 = int(offs[s])
        uni = torch.empty((T, H, D), dtype=torch.float32, device=dev)
        attention_device(qd[o0:o0 + T], torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half(), uni,
                         kind=Kernel.PREFILL_TC)
        device_status()
        assert torch.equal(uni, out[o0:o0 + T]), f"T={T}: ragged call differs from the uniform call"
        rows = _sample_rows(T, 997 if T > 4096 else 101)
        cpu = oracle.attention_rows(q, k, v, 0, rows)
        sel = oracle.rows_mask(rows, T, H)
        max_abs_check(out[o0:o0 + T].cpu().numpy()[sel], cpu[sel], F16_BOUND,
                      f"config 5 ragged prefill T={T} {'paged' if paged else 'contiguous'}")
