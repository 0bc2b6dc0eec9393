"""RoPE + KV-cache append on the GPU through the C ABI, against the CPU oracle (CPUOps.rope restated).

Covers the reference's own RoPE fixture through MetalOps.rope's mirror (OperationTests.swift:63-70), the fused
append of KernelEncoder.ropeQKVStore (decode_fused.metal:126-154) for prefill chunks and ragged decode batches, both
pair conventions, f16 and f32 caches, f16 queries, head_dim 6 / 12 / 32 / 64 / 128 (the vector and the scalar
kernel), unaligned views, untouched cache rows, and the hand-off into the decode attention kernel. The rotation is computed exactly as the oracle computes it (double angle, cos /
sin rounded once to f32, unfused f32 products), so results are compared for equality; the only allowance is one
f32 ulp where the device's double cos / sin and the host's differ by an ulp next to an f32 rounding boundary.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _ulps(a: np.ndarray, b: np.ndarray) -> int:
    """Largest distance in f32 units in the last place."""
    ai = a.astype(np.float32).view(np.int32).astype(np.int64)
    bi = b.astype(np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, np.int64(-2 ** 31) - ai, ai)
    bi = np.where(bi < 0, np.int64(-2 ** 31) - bi, bi)
    return int(np.abs(ai - bi).max()) if a.size else 0


def _f16_ulps(a: np.ndarray, b: np.ndarray) -> int:
    ai = a.astype(np.float16).view(np.int16).astype(np.int64)
    bi = b.astype(np.float16).view(np.int16).astype(np.int64)
    ai = np.where(ai < 0, -32768 - ai, ai)
    bi = np.where(bi < 0, -32768 - bi, bi)
    return int(np.abs(ai - bi).max()) if a.size else 0


def test_metalops_rope_mirror_on_reference_fixture(cuda_lib):
    from alpaca_b200 import rope
    c = json.loads((GOLDEN / "rope_kat.json").read_text())
    x = np.array(c["x"], np.float32).reshape(c["shape"])
    for inter, key in ((True, "expected_interleaved"), (False, "expected_split")):
        got = rope(x, c["start"], c["theta"], inter)
        err = float(np.abs(got - np.array(c[key]).reshape(c["shape"])).max())
        ulp = _ulps(got, oracle.rope(x, c["start"], c["theta"], inter))
        print(f"[metrics] GPU rope {key}: max-abs vs fixture {err:.2e}, {ulp} ulp vs oracle")
        assert err <= c["tolerance"]["atol"] and ulp <= 1


@pytest.mark.parametrize("d,inter,cache_f16,q_f16", [
    (64, True, True, False),    # the model path: GGUF pairs, f16 cache, f32 q
    (64, False, True, False),   # split halves
    (64, True, False, False),   # f32 cache (KVPrecision.float32)
    (64, True, True, True),     # f16 queries rotated in place
    (128, True, True, False),
    (32, False, False, False),
    (6, True, True, False),     # head_dim % 8 != 0: the scalar kernel
    (12, False, False, True),
])
def test_prefill_chunk_append(cuda_lib, d, inter, cache_f16, q_f16):
    """One sequence, a 37-token chunk at position 100 of a 200-row cache pre-filled with a sentinel."""
    from alpaca_b200 import rope_kv_append
    T, H, Hkv, start, cap, theta = 37, 9, 3, 100, 200, 1e5
    q = oracle.splitmix_normal(21, (T, H, d))
    k = oracle.splitmix_normal(22, (T, Hkv, d))
    v = oracle.splitmix_normal(23, (T, Hkv, d))
    dev = torch.device("cuda")
    cdt = torch.float16 if cache_f16 else torch.float32
    qd = torch.from_numpy(q).to(dev).to(torch.float16 if q_f16 else torch.float32)
    kd, vd = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
    kc = torch.full((cap, Hkv, d), 3.0, dtype=cdt, device=dev)
    vc = torch.full((cap, Hkv, d), -3.0, dtype=cdt, device=dev)
    rope_kv_append(qd, kd, vd, kc, vc, theta=theta, start_position=start, interleaved=inter)
    torch.cuda.synchronize()
    q_in = q.astype(np.float16).astype(np.float32) if q_f16 else q
    qr, kcr, vcr = oracle.rope_kv_append(q_in, k, v, np.full((cap, Hkv, d), 3.0, np.float32),
                                         np.full((cap, Hkv, d), -3.0, np.float32), start, theta, inter, cache_f16)
    qg = qd.float().cpu().numpy()
    if q_f16:
        assert _f16_ulps(qg, qr) <= 1
    else:
        assert _ulps(qg, qr) <= 1
    kg, vg = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    ulp = _f16_ulps(kg, kcr) if cache_f16 else _ulps(kg, kcr)
    print(f"[metrics] rope append d={d} inter={inter} f16cache={cache_f16} f16q={q_f16}: k cache {ulp} ulp")
    assert ulp <= 1
    assert np.array_equal(vg, vcr)  # V is copied (rounded once), bit-exact
    rest = np.r_[0:start, start + T:cap]
    assert np.all(kg[rest] == 3.0) and np.all(vg[rest] == -3.0)


def test_unaligned_views_take_the_scalar_kernel(cuda_lib):
    """Tensors offset by 2 elements (8-byte but not 16-byte aligned) are still handled exactly."""
    from alpaca_b200 import rope_kv_append
    T, H, Hkv, d, start, cap, theta = 9, 4, 2, 64, 3, 16, 1e4
    q = oracle.splitmix_normal(51, (T, H, d))
    k = oracle.splitmix_normal(52, (T, Hkv, d))
    v = oracle.splitmix_normal(53, (T, Hkv, d))
    dev = torch.device("cuda")
    qb = torch.zeros(T * H * d + 2, device=dev)
    qb[2:] = torch.from_numpy(q).to(dev).flatten()
    qd = qb[2:].view(T, H, d)
    kb = torch.zeros(T * Hkv * d + 2, device=dev)
    kb[2:] = torch.from_numpy(k).to(dev).flatten()
    vd = torch.from_numpy(v).to(dev)
    kc = torch.zeros((cap, Hkv, d), dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    rope_kv_append(qd, kb[2:].view(T, Hkv, d), vd, kc, vc, theta=theta, start_position=start)
    torch.cuda.synchronize()
    qr, kcr, vcr = oracle.rope_kv_append(q, k, v, np.zeros((cap, Hkv, d), np.float32),
                                         np.zeros((cap, Hkv, d), np.float32), start, theta, True, True)
    assert _ulps(qd.cpu().numpy(), qr) <= 1
    assert _f16_ulps(kc.float().cpu().numpy(), kcr) <= 1
    assert np.array_equal(vc.float().cpu().numpy(), vcr)


@pytest.mark.parametrize("inter", [True, False])
def test_ragged_decode_batch_positions(cuda_lib, inter):
    """64 sequences, one new token each at its own position (device positions array), caches [64][4096][3][64]."""
    from alpaca_b200 import rope_kv_append
    S, H, Hkv, d, cap, theta = 64, 9, 3, 64, 4096, 1e5
    rng = np.random.default_rng(20260104)
    pos = rng.integers(0, cap, size=S).astype(np.int32)
    q = oracle.splitmix_normal(31, (S, 1, H, d))
    k = oracle.splitmix_normal(32, (S, 1, Hkv, d))
    v = oracle.splitmix_normal(33, (S, 1, Hkv, d))
    dev = torch.device("cuda")
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    kc = torch.zeros((S, cap, Hkv, d), dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    rope_kv_append(qd, kd, vd, kc, vc, theta=theta, positions=torch.from_numpy(pos).to(dev), interleaved=inter)
    torch.cuda.synchronize()
    qg = qd.cpu().numpy()
    worst = 0
    for s in range(S):
        p = int(pos[s])
        qr, kcr, vcr = oracle.rope_kv_append(q[s], k[s], v[s], np.zeros((p + 1, Hkv, d), np.float32),
                                             np.zeros((p + 1, Hkv, d), np.float32), p, theta, inter, True)
        assert _ulps(qg[s], qr) <= 1
        kg = kc[s, p].float().cpu().numpy()
        worst = max(worst, _f16_ulps(kg, kcr[p]))
        assert np.array_equal(vc[s, p].float().cpu().numpy(), vcr[p])
    print(f"[metrics] ragged decode append inter={inter}: k cache {worst} f16 ulp over {S} sequences")
    assert worst <= 1
    # exactly one row per sequence was written
    written = (kc.float().abs().sum(dim=(2, 3)) != 0).sum(dim=1).cpu().numpy()
    assert np.all(written <= 1)


def test_hand_off_into_decode_attention(cuda_lib):
    """RoPE + append of the newest token, then split-KV decode over the cache: equals the oracle's rope followed by
    its attention (the order of MetalLlamaSession.encodeChunk, MetalLlamaModel.swift:347-351)."""
    from alpaca_b200 import Kernel, attention_device, rope_kv_append
    S, H, Hkv, d, L, theta = 8, 9, 3, 64, 700, 1e5
    dev = torch.device("cuda")
    k_prev = oracle.f16_round(oracle.splitmix_normal(41, (S, L, Hkv, d)))  # rows 0..L-2 already in the cache
    q = oracle.splitmix_normal(42, (S, 1, H, d))
    k = oracle.splitmix_normal(43, (S, 1, Hkv, d))
    v = oracle.splitmix_normal(44, (S, 1, Hkv, d))
    v_prev = oracle.f16_round(oracle.splitmix_normal(45, (S, L, Hkv, d)))
    kc = torch.from_numpy(k_prev).to(dev).half()
    vc = torch.from_numpy(v_prev).to(dev).half()
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    rope_kv_append(qd, kd, vd, kc, vc, theta=theta, start_position=L - 1)
    out = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
    attention_device(qd, kc, vc, out, start_position=L - 1, kind=Kernel.DECODE_SPLIT)
    torch.cuda.synchronize()
    gpu = out.cpu().numpy()
    worst = 0.0
    for s in range(S):
        qr, kcr, vcr = oracle.rope_kv_append(q[s], k[s], v[s], k_prev[s], v_prev[s], L - 1, theta, True, True)
        ref = oracle.attention(qr, kcr, vcr, L - 1, length=L)
        worst = max(worst, float(np.abs(gpu[s] - ref).max()))
    print(f"[metrics] rope + append -> decode attention: max-abs {worst:.2e}")
    assert worst <= 1e-5
