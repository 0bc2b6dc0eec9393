"""Split-KV prefill: a uniform call with fewer work items than one per SM cuts each item's KV blocks into parts that
run on their own SMs, then merges them. The case is alpaca.swift's prefill loop: one session's 512-token chunk per
call at a moving start position (MetalLlamaModel.swift:293-298), 18 work items at SmolLM2-135M's 9 heads.

Each case runs with the workspace size the library asks for (split) and with a workspace of the minimum size
(unsplit). Both are checked against the CPU oracle on sampled rows, including every head's last token, at the f16
bound. The two outputs are compared with each other, which holds whole tensors to the same bound; they are not bit for
bit equal, since the parts sum in a different order. Cases: head_dim 64 and 128, f32 and f16 output, f32 queries
(staged in the same workspace), a multi-sequence batch, a paged cache, one 128-row tile per item, and parts that
start past some of a tile's rows (rows that see no key in that part).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from tests._util import max_abs_check

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F16_BOUND = 2e-3   # f16 inputs, fp32 accumulate
F16_OUT = 1e-3     # extra allowance for an f16 output


def _normal(seed, shape):
    return oracle.f16_round(oracle.splitmix_normal(seed, shape))


def _rows(T, H, seed):
    """Sampled rows (row = h*T + t): every head's first and last token plus random ones."""
    rng = np.random.default_rng(seed)
    rows = set()
    for h in range(H):
        rows.update({h * T, h * T + T - 1})
    rows.update(rng.integers(0, T * H, size=min(T * H, 96)).tolist())
    return sorted(rows)


def _run(desc_args, ws_bytes):
    import alpaca_b200 as ab
    lib = ab.load()
    desc = ab.make_desc(*desc_args[0], **desc_args[1])
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    st = lib.alpaca_attention(ctypes.byref(desc), int(ab.Kernel.PREFILL_TC), ctypes.c_void_p(ws.data_ptr()),
                              ws_bytes, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == ab.Status.OK, lib.alpaca_cuda_last_error()
    ab.device_status()


@pytest.mark.parametrize("d,H,kvh,T,start,odt,qdt", [
    (64, 9, 3, 512, 3584, torch.float32, torch.float16),   # alpaca's last chunk of a 4096-token prompt
    (64, 9, 3, 512, 1536, torch.float16, torch.float16),
    (64, 9, 3, 300, 3000, torch.float32, torch.float32),   # f32 queries staged in the same workspace
    (64, 9, 3, 100, 4000, torch.float32, torch.float16),   # one 128-row tile per item
    (128, 8, 2, 384, 2000, torch.float32, torch.float16),
    (128, 8, 2, 512, 3584, torch.float16, torch.float16),
    # the first group's second part starts at position 256, past its first rows (positions 150-255), which see no
    # key there; in the warp holding rows 96-127 some rows see keys and some none
    (64, 8, 2, 1000, 150, torch.float32, torch.float16),
    (128, 8, 2, 1000, 150, torch.float16, torch.float16),
])
def test_split_kv_matches_oracle_and_unsplit(cuda_lib, d, H, kvh, T, start, odt, qdt):
    import alpaca_b200 as ab
    dev = torch.device("cuda")
    q = _normal(500 + T, (1, T, H, d))
    k = _normal(501 + T, (1, start + T, kvh, d))
    v = _normal(502 + T, (1, start + T, kvh, d))
    qd = torch.from_numpy(q).to(dev).to(qdt)
    kd, vd = torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half()
    outs = []
    for split in (True, False):
        out = torch.full((1, T, H, d), float("nan"), dtype=odt, device=dev)
        args = ((qd, kd, vd, out), {"start_position": start})
        need = ab.workspace_bytes(ab.make_desc(qd, kd, vd, out, start_position=start), ab.Kernel.PREFILL_TC)
        # the minimum: the f32 queries' staging only
        minimum = T * H * d * 2 if qdt == torch.float32 else 0
        minimum = (minimum + 15) // 16 * 16
        if split:
            assert need > minimum, "the call should ask for split-KV records"
        _run(args, need if split else minimum)
        outs.append(out.float().cpu().numpy())
    rows = _rows(T, H, T + start)
    cpu = oracle.attention_rows(q[0], k[0], v[0], start, rows)
    sel = oracle.rows_mask(rows, T, H)
    bound = F16_BOUND + (F16_OUT if odt == torch.float16 else 0.0)
    for name, g in zip(("split", "unsplit"), outs):
        assert np.isfinite(g).all(), name
        max_abs_check(g[0][sel], cpu[sel], bound, f"split-KV d={d} T={T} start={start} out={odt} q={qdt} {name}")
    diff = float(np.abs(outs[0] - outs[1]).max())
    print(f"[metrics] split-KV d={d} T={T} start={start}: split vs unsplit max-abs {diff:.3e}")
    assert diff <= bound


def test_split_kv_batch_and_paged_pool(cuda_lib):
    """Three sequences in one call (27 items), contiguous and from a shuffled pool of 256-row blocks with a NaN
    filler, split against the oracle."""
    import alpaca_b200 as ab
    from tests._util import pool
    dev = torch.device("cuda")
    S, T, start, H, kvh, d = 3, 256, 2600, 9, 3, 64
    q = _normal(601, (S, T, H, d))
    k = _normal(602, (S, start + T, kvh, d))
    v = _normal(603, (S, start + T, kvh, d))
    qd = torch.from_numpy(q).to(dev).half()
    kd, vd = torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half()
    rng = np.random.default_rng(604)
    kp, table = pool([k[s] for s in range(S)], 256, rng, start + T)
    vp, _ = pool([v[s] for s in range(S)], 256, np.random.default_rng(604), start + T)
    kpd, vpd = torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half()
    tabd = torch.from_numpy(table).to(dev)
    results = {}
    for name in ("contiguous", "paged"):
        out = torch.full((S, T, H, d), float("nan"), dtype=torch.float32, device=dev)
        if name == "contiguous":
            desc = ab.make_desc(qd, kd, vd, out, start_position=start)
        else:
            desc = ab.make_desc(qd, kpd, vpd, out, start_position=start, block_table=tabd)
        need = ab.workspace_bytes(desc, ab.Kernel.PREFILL_TC)
        assert need > 0
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        ab.launch(desc, ab.Kernel.PREFILL_TC, ws)
        ab.device_status()
        results[name] = out.cpu().numpy()
    rows = _rows(T, H, 605)
    sel = oracle.rows_mask(rows, T, H)
    for s in range(S):
        cpu = oracle.attention_rows(q[s], k[s], v[s], start, rows)
        for name, g in results.items():
            max_abs_check(g[s][sel], cpu[sel], F16_BOUND, f"split-KV batch seq {s} {name}")
    assert np.array_equal(results["contiguous"], results["paged"])


@pytest.mark.parametrize("d,H,kvh,odt", [(64, 9, 3, torch.float32), (128, 8, 2, torch.float16)])
def test_split_kv_ragged_call(cuda_lib, d, H, kvh, odt):
    """A ragged call of four sessions' chunks (8 units x heads: fewer items than SMs) splits too. Each unit uses as
    many parts as its own KV blocks allow, so the chunk at position 0 stays whole and writes its output directly.
    Each cache holds NaN past its context; rows of a sequence's last KV block past its context are zeroed inside
    whichever part holds that block. Checked against the oracle on sampled rows and against the same call given only
    the minimum workspace (unsplit); the split call over shuffled 256-row blocks of a NaN pool equals the contiguous
    split call bit for bit."""
    import alpaca_b200 as ab
    from tests._util import pool, varlen_unsplit
    dev = torch.device("cuda")
    seqs = [(512, 3584), (300, 2000), (100, 4000), (512, 0)]
    cap = 4200
    lens = [t for t, _ in seqs]
    offs_np = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q = _normal(700, (int(offs_np[-1]), H, d))
    ks, vs = [], []
    kc = np.full((len(seqs), cap, kvh, d), np.nan, np.float32)
    vc = np.full((len(seqs), cap, kvh, d), np.nan, np.float32)
    for s, (T, start) in enumerate(seqs):
        ks.append(_normal(710 + s, (start + T, kvh, d)))
        vs.append(_normal(720 + s, (start + T, kvh, d)))
        kc[s, :start + T], vc[s, :start + T] = ks[-1], vs[-1]
    qd = torch.from_numpy(q).to(dev).half()
    kd, vd = torch.from_numpy(kc).to(dev).half(), torch.from_numpy(vc).to(dev).half()
    offs = torch.from_numpy(offs_np).to(dev)
    starts = torch.tensor([st for _, st in seqs], dtype=torch.int32, device=dev)
    outs = []
    for split in (True, False):
        out = torch.full((int(offs_np[-1]), H, d), float("nan"), dtype=odt, device=dev)
        if split:
            desc = ab.make_varlen_desc(qd, kd, vd, out, offs, starts, max_tokens=512, max_ctx_len=cap)
            need = ab.workspace_bytes(desc, ab.Kernel.PREFILL_TC)
            minimum = 16 * (1 + 2 * len(seqs) * 2)
            assert need > minimum, "the ragged call should ask for split-KV records"
            ab.launch(desc, ab.Kernel.PREFILL_TC, torch.empty(need, dtype=torch.uint8, device=dev))
        else:
            varlen_unsplit(qd, kd, vd, out, offs, starts, max_tokens=512, max_ctx_len=cap)
        ab.device_status()
        outs.append(out.float().cpu().numpy())
    bound = F16_BOUND + (F16_OUT if odt == torch.float16 else 0.0)
    for s, (T, start) in enumerate(seqs):
        o0 = int(offs_np[s])
        rows = _rows(T, H, 730 + s)
        cpu = oracle.attention_rows(q[o0:o0 + T], ks[s], vs[s], start, rows)
        sel = oracle.rows_mask(rows, T, H)
        for name, g in zip(("split", "unsplit"), outs):
            assert np.isfinite(g[o0:o0 + T]).all(), f"{name} seq {s}"
            max_abs_check(g[o0:o0 + T][sel], cpu[sel], bound, f"ragged split-KV d={d} seq {s} {name}")
    diff = float(np.abs(outs[0] - outs[1]).max())
    print(f"[metrics] ragged split-KV d={d}: split vs unsplit max-abs {diff:.3e}")
    assert diff <= bound
    kp, table = pool(ks, 256, np.random.default_rng(740), cap)
    vp, _ = pool(vs, 256, np.random.default_rng(740), cap)
    out_p = torch.full((int(offs_np[-1]), H, d), float("nan"), dtype=odt, device=dev)
    ab.prefill_varlen(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out_p, offs,
                      starts, max_tokens=512, max_ctx_len=cap, block_table=torch.from_numpy(table).to(dev))
    ab.device_status()
    got = out_p.float().cpu().numpy()
    differ = []
    for s in range(len(seqs)):
        a, b = got[offs_np[s]:offs_np[s + 1]], outs[0][offs_np[s]:offs_np[s + 1]]
        bad = np.nonzero(~((a == b) | (np.isnan(a) & np.isnan(b))).all(axis=(1, 2)))[0]
        if bad.size:
            differ.append(f"seq {s}: {bad.size} rows ({bad.min()}-{bad.max()}), "
                          f"{int((~np.isfinite(a[bad])).any(axis=(1, 2)).sum())} of them non-finite")
    assert not differ, "paged split call differs from the contiguous one: " + "; ".join(differ)
