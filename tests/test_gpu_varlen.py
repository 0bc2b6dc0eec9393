"""Ragged (varlen) prefill on the GPU through the C ABI: several sequences with their own query counts and start
positions in one tensor-core prefill launch, queries and outputs packed back to back.

A serving loop prefills the chunks of several sessions at their own positions (alpaca.swift runs one session's
512-token chunks per call at a moving startPosition, Sources/AlpacaMetal/Backend/MetalLlamaModel.swift:293-298);
the ragged call takes them together. Checked here: every row against the CPU oracle at the f16 bound; bit-exact
equality with one uniform call per sequence (same tiles, same KV blocks, same arithmetic); cache rows past each
sequence's context filled with NaN never reach an output; a paged pool gives the same bits as contiguous caches;
packed rows that belong to no sequence are never written; a sequence that breaks the call's bounds is reported and
skipped while the others are computed; a multi-session chunked prefill equals each session's one-shot prefill.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests._util import max_abs_check, pool, prefill_unsplit, varlen_unsplit

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F16_BOUND = 2e-3
SENTINEL = 7.0

# (query tokens, start position): single-token, empty, tile-boundary, partial-tile and multi-group sequences
SEQS = [(300, 0), (1, 517), (0, 50), (128, 128), (129, 1000), (700, 33), (512, 1536), (37, 0)]


def _inputs(seqs, H, Hkv, d, seed):
    """Packed f16-representable queries, per-sequence caches with NaN past each context, offsets and starts."""
    lens = np.array([t for t, _ in seqs], np.int32)
    starts = np.array([s for _, s in seqs], np.int32)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    total = int(offs[-1])
    max_ctx = int((lens + starts).max())
    q = oracle.f16_round(oracle.splitmix_normal(seed, (total, H, d)))
    ks = [oracle.f16_round(oracle.splitmix_normal(seed + 1 + s, (int(starts[s] + lens[s]), Hkv, d)))
          for s in range(len(seqs))]
    vs = [oracle.f16_round(oracle.splitmix_normal(seed + 101 + s, (int(starts[s] + lens[s]), Hkv, d)))
          for s in range(len(seqs))]
    return q, ks, vs, lens, starts, offs, max_ctx


def _caches(ks, vs, cap, dev):
    S = len(ks)
    Hkv, d = ks[0].shape[1:]
    kd = torch.full((S, cap, Hkv, d), float("nan"), dtype=torch.float16, device=dev)
    vd = torch.full((S, cap, Hkv, d), float("nan"), dtype=torch.float16, device=dev)
    for s in range(S):
        n = ks[s].shape[0]
        kd[s, :n] = torch.from_numpy(ks[s]).to(dev).half()
        vd[s, :n] = torch.from_numpy(vs[s]).to(dev).half()
    return kd, vd


@pytest.mark.parametrize("d,H,Hkv", [(64, 9, 3), (128, 8, 2)])
@pytest.mark.parametrize("q_dtype,out_dtype", [(torch.float16, torch.float32), (torch.float32, torch.float16)])
def test_varlen_prefill_matches_oracle_and_uniform_calls(cuda_lib, d, H, Hkv, q_dtype, out_dtype):
    from alpaca_b200 import device_status, prefill_varlen
    q, ks, vs, lens, starts, offs, max_ctx = _inputs(SEQS, H, Hkv, d, 900 + d)
    dev = torch.device("cuda")
    total, pad = q.shape[0], 5
    kd, vd = _caches(ks, vs, max_ctx + 40, dev)
    qd = torch.zeros((total + pad, H, d), dtype=q_dtype, device=dev)
    qd[:total] = torch.from_numpy(q).to(dev).to(q_dtype)
    out = torch.full((total + pad, H, d), SENTINEL, dtype=out_dtype, device=dev)
    prefill_varlen(qd, kd, vd, out, torch.from_numpy(offs).to(dev), torch.from_numpy(starts).to(dev),
                   max_tokens=int(lens.max()), max_ctx_len=max_ctx + 40)
    device_status()
    got = out.float().cpu().numpy()
    assert np.all(got[total:] == SENTINEL), "rows past the last sequence were written"
    bound = F16_BOUND + (1e-3 if out_dtype == torch.float16 else 0.0)
    for s, (T, start) in enumerate(SEQS):
        if T == 0:
            continue
        o0 = int(offs[s])
        ref = oracle.attention(q[o0:o0 + T], ks[s], vs[s], start)
        max_abs_check(got[o0:o0 + T], ref, bound, f"varlen d={d} seq {s} T={T} start={start} q={q_dtype} out={out_dtype}")
        # the same sequence as its own (unsplit) uniform call: identical bits
        uni = torch.empty((T, H, d), dtype=out_dtype, device=dev)
        prefill_unsplit(qd[o0:o0 + T], kd[s, :start + T], vd[s, :start + T], uni, start_position=start)
        device_status()
        assert torch.equal(uni, out[o0:o0 + T]), f"seq {s}: ragged and uniform calls differ"


@pytest.mark.parametrize("block_rows", [128, 256])
def test_varlen_prefill_paged_equals_contiguous(cuda_lib, block_rows):
    """The same ragged call over shuffled blocks of a NaN pool: bit for bit the contiguous result."""
    from alpaca_b200 import device_status, prefill_varlen
    H, Hkv, d = 9, 3, 64
    q, ks, vs, lens, starts, offs, max_ctx = _inputs(SEQS, H, Hkv, d, 950)
    dev = torch.device("cuda")
    kd, vd = _caches(ks, vs, max_ctx, dev)
    qd = torch.from_numpy(q).to(dev).half()
    od, ld = torch.from_numpy(offs).to(dev), torch.from_numpy(starts).to(dev)
    out_c = torch.empty((q.shape[0], H, d), dtype=torch.float32, device=dev)
    prefill_varlen(qd, kd, vd, out_c, od, ld, max_tokens=int(lens.max()), max_ctx_len=max_ctx)
    kp, table = pool(ks, block_rows, np.random.default_rng(block_rows), max_ctx)
    vp, table_v = pool(vs, block_rows, np.random.default_rng(block_rows), max_ctx)
    assert np.array_equal(table, table_v)
    out_p = torch.empty_like(out_c)
    prefill_varlen(qd, torch.from_numpy(kp).to(dev).half(), torch.from_numpy(vp).to(dev).half(), out_p, od, ld,
                   max_tokens=int(lens.max()), max_ctx_len=max_ctx, block_table=torch.from_numpy(table).to(dev))
    device_status()
    assert torch.isfinite(out_p).all()
    assert torch.equal(out_p, out_c)


def test_varlen_prefill_bad_sequence_is_reported_and_skipped(cuda_lib):
    """A sequence whose start + tokens passes max_ctx_len breaks the call's bounds: it is reported
    (INVALID_ARGUMENT) and its rows are not written; the other sequences are computed."""
    from alpaca_b200 import AlpacaCUDAError, Status, device_status, prefill_varlen
    H, Hkv, d = 9, 3, 64
    seqs = [(200, 0), (100, 450), (150, 10)]  # sequence 1 reaches row 550 > max_ctx_len 500
    q, ks, vs, lens, starts, offs, _ = _inputs(seqs, H, Hkv, d, 970)
    dev = torch.device("cuda")
    kd, vd = _caches(ks, vs, 600, dev)
    out = torch.full((q.shape[0], H, d), SENTINEL, dtype=torch.float32, device=dev)
    device_status()
    prefill_varlen(torch.from_numpy(q).to(dev).half(), kd, vd, out, torch.from_numpy(offs).to(dev),
                   torch.from_numpy(starts).to(dev), max_tokens=200, max_ctx_len=500)
    with pytest.raises(AlpacaCUDAError) as e:
        device_status()
    assert e.value.status == Status.INVALID_ARGUMENT
    got = out.cpu().numpy()
    assert np.all(got[offs[1]:offs[2]] == SENTINEL)
    for s in (0, 2):
        o0, T = int(offs[s]), int(lens[s])
        ref = oracle.attention(q[o0:o0 + T], ks[s], vs[s], int(starts[s]))
        max_abs_check(got[o0:o0 + T], ref, F16_BOUND, f"varlen bounds check, unaffected seq {s}")


def test_chunked_prefill_of_several_sessions(cuda_lib):
    """Three sessions' prompts prefilled in 512-token chunks, every active session's next chunk in one ragged call
    per step (each at its own moving start, as MetalLlamaModel.swift:293-298 moves startPosition), equal each
    session's one-shot prefill bit for bit. A step has 54 work items at most, so with the workspace the library asks
    for, its later steps split their KV range over the SMs; that loop is checked against the one-shot prefill at the
    f16 bound (the parts sum in another order), and the loop given only the minimum workspace (unsplit) bit for
    bit."""
    from alpaca_b200 import device_status, prefill_varlen
    H, Hkv, d, chunk = 9, 3, 64, 512
    prompts = [1300, 512, 2000]
    dev = torch.device("cuda")
    qs = [torch.from_numpy(oracle.f16_round(oracle.splitmix_normal(990 + i, (n, H, d)))).to(dev).half()
          for i, n in enumerate(prompts)]
    kc = torch.from_numpy(oracle.f16_round(oracle.splitmix_normal(995, (3, 2048, Hkv, d)))).to(dev).half()
    vc = torch.from_numpy(oracle.f16_round(oracle.splitmix_normal(996, (3, 2048, Hkv, d)))).to(dev).half()
    results = {}
    for split in (False, True):
        outs = [torch.empty((n, H, d), dtype=torch.float32, device=dev) for n in prompts]
        done = [0, 0, 0]
        while any(done[i] < prompts[i] for i in range(3)):
            # sessions with no tokens left take part with an empty chunk
            take = [min(chunk, prompts[i] - done[i]) for i in range(3)]
            offs = torch.from_numpy(np.concatenate([[0], np.cumsum(take)]).astype(np.int32)).to(dev)
            starts = torch.tensor(done, dtype=torch.int32, device=dev)
            qpack = torch.cat([qs[i][done[i]:done[i] + take[i]] for i in range(3)])
            opack = torch.empty((int(offs[-1]), H, d), dtype=torch.float32, device=dev)
            if split:
                prefill_varlen(qpack, kc, vc, opack, offs, starts, max_tokens=chunk, max_ctx_len=2048)
            else:
                varlen_unsplit(qpack, kc, vc, opack, offs, starts, max_tokens=chunk, max_ctx_len=2048)
            for i in range(3):
                outs[i][done[i]:done[i] + take[i]] = opack[int(offs[i]):int(offs[i + 1])]
                done[i] += take[i]
        device_status()
        results[split] = outs
    for i, n in enumerate(prompts):
        one = torch.empty((n, H, d), dtype=torch.float32, device=dev)
        prefill_unsplit(qs[i], kc[i, :n], vc[i, :n], one)
        device_status()
        assert torch.equal(one, results[False][i]), f"session {i}: chunked and one-shot prefill differ"
        diff = float((one - results[True][i]).abs().max())
        print(f"[metrics] session {i}: split-KV chunk loop vs one-shot max-abs {diff:.3e}")
        assert np.isfinite(diff) and diff <= 2e-3, f"session {i}: split-KV chunk loop differs by {diff:.3e}"
