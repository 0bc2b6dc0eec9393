"""The decode step with the RoPE + KV append fused into the attention launch (alpaca_attn_decode_rope).

Its contract is the two calls it replaces: alpaca_rope_kv_append of each sequence's new token at position
ctx_len - 1, then the split decode over the caches. The tests compare the fused call with those two calls on
copies of the same tensors and require identical bits: the attention output, every cache row (the new row included,
which starts out as NaN so that a stale read would show), and an unmodified q (the fused call rotates q as it reads
it). Covered: head_dim 64 (tensor-core unit compute) and 128 (packed-FMA form), both pair conventions, f32 and f16
queries, ragged contexts from 1 to past several splits, a uniform start_position, a paged pool, and one check
against the CPU oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

THETA = 1e5


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16 if t.element_size() == 2 else torch.int32).numpy()


def _case(d, G, Hkv, lens, q_f16, seed):
    S, cap = len(lens), int(max(lens))
    H = G * Hkv
    dev = torch.device("cuda")
    q = torch.from_numpy(oracle.splitmix_normal(seed, (S, 1, H, d))).to(dev)
    if q_f16:
        q = q.half()
    kn = torch.from_numpy(oracle.splitmix_normal(seed + 1, (S, 1, Hkv, d))).to(dev)
    vn = torch.from_numpy(oracle.splitmix_normal(seed + 2, (S, 1, Hkv, d))).to(dev)
    kc = torch.from_numpy(oracle.splitmix_normal(seed + 3, (S, cap, Hkv, d))).to(dev).half()
    vc = torch.from_numpy(oracle.splitmix_normal(seed + 4, (S, cap, Hkv, d))).to(dev).half()
    for s, L in enumerate(lens):  # the new token's row and everything after it: NaN until written
        kc[s, L - 1:] = float("nan")
        vc[s, L - 1:] = float("nan")
    return q, kn, vn, kc, vc


@pytest.mark.parametrize("d,G,inter,q_f16", [
    (64, 3, True, False),    # the SmolLM2 decode shape, GGUF pairs, f32 q
    (64, 3, False, False),   # split halves
    (64, 4, True, True),     # f16 q (rotated, then rounded to f16 as the in-place rotation stores it)
    (128, 4, True, False),   # head_dim 128: the packed-FMA unit compute
    (128, 2, False, True),
])
def test_fused_equals_rope_then_decode(cuda_lib, d, G, inter, q_f16):
    from alpaca_b200 import Kernel, attention_device, decode_rope, device_status, rope_kv_append
    Hkv = 3 if G == 3 else 2
    lens = [1, 2, 127, 128, 129, 257, 700, 1500]
    q, kn, vn, kc, vc = _case(d, G, Hkv, lens, q_f16, 400 + d + G)
    S, H = len(lens), G * Hkv
    dev = q.device
    ld = torch.tensor(lens, dtype=torch.int32, device=dev)
    cap = int(max(lens))
    # the two calls on copies
    q2, kc2, vc2 = q.clone(), kc.clone(), vc.clone()
    rope_kv_append(q2, kn, vn, kc2, vc2, theta=THETA, positions=ld - 1, interleaved=inter)
    out2 = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
    attention_device(q2, kc2, vc2, out2, ctx_lens=ld, max_ctx_len=cap, kind=Kernel.DECODE_SPLIT)
    # the fused call
    q0 = q.clone()
    out = torch.empty_like(out2)
    decode_rope(q, kn, vn, kc, vc, out, theta=THETA, ctx_lens=ld, max_ctx_len=cap, interleaved=inter)
    device_status()
    assert np.array_equal(_bits(out), _bits(out2)), float((out - out2).abs().max())
    assert np.array_equal(_bits(kc), _bits(kc2)) and np.array_equal(_bits(vc), _bits(vc2))
    assert np.array_equal(_bits(q), _bits(q0))  # q is read, not rotated in place
    assert torch.isfinite(out).all()


def test_fused_uniform_position_matches_oracle(cuda_lib):
    """ctx_lens NULL: every sequence's new token at start_position; against the CPU oracle's rope + attention."""
    from alpaca_b200 import decode_rope, device_status
    S, H, Hkv, d, pos = 3, 9, 3, 64, 700
    q, kn, vn, kc, vc = _case(d, 3, Hkv, [pos + 1] * S, False, 500)
    out = torch.empty((S, 1, H, d), dtype=torch.float32, device=q.device)
    k_prev = kc.float().cpu().numpy()
    v_prev = vc.float().cpu().numpy()
    decode_rope(q, kn, vn, kc, vc, out, theta=THETA, start_position=pos)
    device_status()
    got = out.cpu().numpy()
    for s in range(S):
        qr, kcr, vcr = oracle.rope_kv_append(q[s].cpu().numpy(), kn[s].cpu().numpy(), vn[s].cpu().numpy(),
                                             k_prev[s].copy(), v_prev[s].copy(), pos, THETA, True, True)
        ref = oracle.attention(qr, kcr, vcr, pos, length=pos + 1)
        err = float(np.abs(got[s] - ref).max())
        print(f"[metrics] fused rope + decode vs oracle, seq {s}: max-abs {err:.2e}")
        assert err <= 1e-5


def test_fused_on_paged_pool(cuda_lib):
    """Block-table caches: the fused call writes the new rows into the pool blocks the two calls write."""
    from alpaca_b200 import Kernel, attention_device, decode_rope, device_status, rope_kv_append
    S, G, Hkv, d, R = 6, 3, 3, 64, 128
    H = G * Hkv
    lens = [1, 128, 129, 300, 640, 1000]
    dev = torch.device("cuda")
    nb = [-(-L // R) for L in lens]
    total = sum(nb) + 2
    order = np.random.default_rng(9).permutation(total).astype(np.int32)
    table = np.zeros((S, max(nb)), np.int32)
    nxt = 0
    for s, n in enumerate(nb):
        table[s, :n] = order[nxt:nxt + n]
        nxt += n
    tab = torch.from_numpy(table).to(dev)
    kp = torch.from_numpy(oracle.splitmix_normal(601, (total, R, Hkv, d))).to(dev).half()
    vp = torch.from_numpy(oracle.splitmix_normal(602, (total, R, Hkv, d))).to(dev).half()
    q = torch.from_numpy(oracle.splitmix_normal(603, (S, 1, H, d))).to(dev)
    kn = torch.from_numpy(oracle.splitmix_normal(604, (S, 1, Hkv, d))).to(dev)
    vn = torch.from_numpy(oracle.splitmix_normal(605, (S, 1, Hkv, d))).to(dev)
    ld = torch.tensor(lens, dtype=torch.int32, device=dev)
    cap = max(lens)
    q2, kp2, vp2 = q.clone(), kp.clone(), vp.clone()
    rope_kv_append(q2, kn, vn, kp2, vp2, theta=THETA, positions=ld - 1, block_table=tab)
    out2 = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
    attention_device(q2, kp2, vp2, out2, ctx_lens=ld, max_ctx_len=cap, kind=Kernel.DECODE_SPLIT, block_table=tab)
    out = torch.empty_like(out2)
    decode_rope(q, kn, vn, kp, vp, out, theta=THETA, ctx_lens=ld, max_ctx_len=cap, block_table=tab)
    device_status()
    assert np.array_equal(_bits(out), _bits(out2))
    assert np.array_equal(_bits(kp), _bits(kp2)) and np.array_equal(_bits(vp), _bits(vp2))
