"""The CPU oracle pinned against the reference's own known answers (CPU only).

Mirrors Tests/AlpacaCoreTests/OperationTests.swift: testCausalGQAAttention (:72-86), testSoftmax (:55-61) and
testRoPEBothConventions (:63-70), on the fixture values committed in tests/golden/ (extracted from the reference's ops.json by
tests/golden/make_golden.py). Then cross-checks the oracle against float64 SDPA on BASELINE shapes and checks its
helpers (f16 rounding, generators, error metrics, fused == three-step).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from tests._util import compare

GOLDEN = Path(__file__).resolve().parent / "golden"


def _kat():
    c = json.loads((GOLDEN / "attention_kat.json").read_text())
    t, h, kv, hd, cap = c["tokens"], c["heads"], c["kvHeads"], c["headDim"], c["capacity"]
    q = np.array(c["q"], np.float32).reshape(t, h, hd)
    k = np.array(c["k"], np.float32).reshape(cap, kv, hd)
    v = np.array(c["v"], np.float32).reshape(cap, kv, hd)
    return c, q, k, v


def test_attention_known_answer():
    """OperationTests.testCausalGQAAttention: mask pattern and values within 3e-6 abs / 1e-5 rel."""
    c, q, k, v = _kat()
    L, start = c["length"], c["start"]
    s = oracle.attention_scores(q, k, L, start)
    H, T = c["heads"], c["tokens"]
    for hh in range(H):
        for tt in range(T):
            for p in range(L):
                assert (s[hh, tt, p] == -np.inf) == (p > start + tt)
    out = oracle.attention_apply(oracle.softmax(s), v)
    compare(out, np.array(c["expected"]), 3e-6, 1e-5, "oracle attention KAT")


def test_fused_rows_bit_identical_to_three_steps():
    c, q, k, v = _kat()
    three = oracle.attention_apply(oracle.softmax(oracle.attention_scores(q, k, c["length"], c["start"])), v)
    fused = oracle.attention(q, k, v, c["start"], length=c["length"])
    assert np.array_equal(three, fused)
    # larger GQA case with a cache longer than `length`
    rng = np.random.default_rng(5)
    T, H, kvh, d, start = 13, 9, 3, 64, 20
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((start + T + 5, kvh, d)).astype(np.float32)
    v = rng.standard_normal((start + T + 5, kvh, d)).astype(np.float32)
    three = oracle.attention_apply(oracle.softmax(oracle.attention_scores(q, k, start + T, start)), v)
    for threads in (1, 3):
        fused = oracle.attention(q, k, v, start, threads=threads)
        assert np.array_equal(three, fused)


def test_row_subset():
    rng = np.random.default_rng(6)
    T, H, kvh, d = 9, 4, 2, 32
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((T, kvh, d)).astype(np.float32)
    v = rng.standard_normal((T, kvh, d)).astype(np.float32)
    full = oracle.attention(q, k, v, 0)
    part = oracle.attention(q, k, v, 0, rows=(5, 20))
    rows = np.zeros(H * T, bool)
    rows[5:20] = True
    mask = rows.reshape(H, T).T  # [T, H]
    assert np.array_equal(part[mask], full[mask])
    assert np.all(part[~mask] == 0)


def test_softmax_known_answer():
    """OperationTests.testSoftmax: ±30-sigma inputs, 1e-6 abs / 1e-5 rel, rows sum to 1."""
    c = json.loads((GOLDEN / "softmax_kat.json").read_text())
    x = np.array(c["x"], np.float32).reshape(c["shape"])
    r = oracle.softmax(x)
    compare(r, np.array(c["expected"]), 1e-6, 1e-5, "oracle softmax KAT")
    assert np.allclose(r.sum(-1), 1.0, atol=1e-6)


def _sdpa64(q, k, v, start):
    torch = pytest.importorskip("torch")
    T, H, d = q.shape
    g = H // k.shape[1]
    L = start + T
    qt = torch.tensor(q, dtype=torch.float64).permute(1, 0, 2)
    kt = torch.tensor(k[:L], dtype=torch.float64).repeat_interleave(g, 1).permute(1, 0, 2)
    vt = torch.tensor(v[:L], dtype=torch.float64).repeat_interleave(g, 1).permute(1, 0, 2)
    mask = torch.tril(torch.ones(L, L, dtype=torch.bool))[start:start + T]
    return torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask).permute(1, 0, 2).numpy()


@pytest.mark.parametrize("T,H,kvh,d,start,f16", [
    (128, 9, 3, 64, 0, False),    # SmolLM2-135M shape, f32 N(0,1)
    (33, 9, 3, 64, 7, True),
    (1, 15, 5, 64, 300, True),    # decode row, SmolLM2-360M heads
    (40, 32, 32, 64, 0, True),    # SmolLM2-1.7B heads
    (17, 8, 2, 128, 3, True),
])
def test_oracle_vs_float64_sdpa(T, H, kvh, d, start, f16):
    q = oracle.splitmix_normal(20260101 + T, (T, H, d))
    k = oracle.splitmix_normal(20260201 + T, (start + T, kvh, d))
    v = oracle.splitmix_normal(20260301 + T, (start + T, kvh, d))
    if f16:
        q, k, v = oracle.f16_round(q), oracle.f16_round(k), oracle.f16_round(v)
    out = oracle.attention(q, k, v, start)
    exp = _sdpa64(q, k, v, start)
    m = oracle.error_metrics(out, exp)
    print(f"[metrics] oracle vs float64 SDPA T={T} H={H}/{kvh} d={d}: {oracle.format_metrics(m)}")
    assert m["maxAbs"] < 2e-6


def test_f16_rounding_matches_ieee():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 1000,
        (rng.standard_normal(20000) * 1e-5).astype(np.float32),   # subnormal halves
        np.array([65504, 65519.99, 65520, 1e9, 6.1e-5, 6.0e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-9, 0.0, -0.0,
                  np.inf, -np.inf], np.float32),
    ])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).astype(np.float32)
    got = oracle.f16_round(x)
    assert np.array_equal(got, ref)
    assert np.isnan(oracle.f16_round(np.array([np.nan], np.float32))[0])


def _splitmix_py(seed, n):
    M = (1 << 64) - 1
    st, out = seed, []
    for _ in range(n):
        st = (st + 0x9E3779B97F4A7C15) & M
        z = st
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        out.append(z ^ (z >> 31))
    return out


def test_splitmix_uniform_matches_reference_definition():
    """SplitMix.nextFloat (KernelTests.swift:105-113) restated independently in Python."""
    ref = np.array([np.float32(np.float32((x >> 11) / float(1 << 53)) * np.float32(2) - np.float32(1))
                    for x in _splitmix_py(12, 257)], np.float32)
    assert np.array_equal(oracle.splitmix_uniform(12, (257,)), ref)


def test_normal_generator_moments():
    x = oracle.splitmix_normal(20260101, (200001,))
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
    assert np.array_equal(x[:1000], oracle.splitmix_normal(20260101, (1000,)))


def test_error_metrics_definition():
    """ErrorMetrics.swift:15-27."""
    a = np.array([1.0, -2.0, 3.5], np.float32)
    e = np.array([1.5, -2.0, 3.0])
    m = oracle.error_metrics(a, e)
    d = np.abs(a - e)
    assert m["maxAbs"] == pytest.approx(d.max())
    assert m["meanAbs"] == pytest.approx(d.mean())
    assert m["rms"] == pytest.approx(np.sqrt((d * d).mean()))
    assert m["maxRelPeak"] == pytest.approx(d.max() / 3.0)


def test_oracle_rejects_bad_shapes():
    q = np.zeros((4, 3, 32), np.float32)
    k = np.zeros((8, 2, 32), np.float32)
    with pytest.raises(ValueError):
        oracle.attention_scores(q, k, 8, 0)          # 3 heads not divisible by 2 KV heads
    k = np.zeros((8, 1, 32), np.float32)
    with pytest.raises(ValueError):
        oracle.attention_scores(q, k, 8, 5)          # start + tokens > length


# ---------------------------------------------------------------------------------------------- RoPE

def _rope_kat():
    c = json.loads((GOLDEN / "rope_kat.json").read_text())
    return c, np.array(c["x"], np.float32).reshape(c["shape"])


def test_rope_known_answer_both_conventions():
    """CPUOps.rope restated (CPUOps.swift:184-210) against the reference's own fixture ops.json["rope"] at the
    tolerance of OperationTests.swift:68-69 (atol 2e-6), adjacent pairs and split halves."""
    c, x = _rope_kat()
    for inter, key in ((True, "expected_interleaved"), (False, "expected_split")):
        got = oracle.rope(x, c["start"], c["theta"], inter)
        err = float(np.abs(got - np.array(c[key]).reshape(c["shape"])).max())
        print(f"[metrics] oracle rope {key}: max-abs {err:.2e} (bound {c['tolerance']['atol']})")
        assert err <= c["tolerance"]["atol"]


def test_rope_position_zero_is_identity_and_norms_are_kept():
    x = oracle.splitmix_normal(5, (3, 4, 32))
    y = oracle.rope(x, 0, 1e4, True)
    assert np.array_equal(y[0], x[0])  # angle 0: cos 1, sin 0 exactly
    n0 = np.linalg.norm(x.reshape(3, 4, 16, 2), axis=-1)
    n1 = np.linalg.norm(y.reshape(3, 4, 16, 2), axis=-1)
    assert np.abs(n0 - n1).max() < 1e-5  # a rotation per pair


def test_rope_kv_append_composition():
    """The fused step on the CPU path (decode_fused.metal:126-154): q rotated, cache rows start..start+T-1 get
    f16(rope(k)) and f16(v), every other cache row unchanged."""
    T, H, Hkv, d, start, cap = 5, 6, 2, 16, 9, 20
    q = oracle.splitmix_normal(11, (T, H, d))
    k = oracle.splitmix_normal(12, (T, Hkv, d))
    v = oracle.splitmix_normal(13, (T, Hkv, d))
    kc0 = np.full((cap, Hkv, d), 7.0, np.float32)
    vc0 = np.full((cap, Hkv, d), -7.0, np.float32)
    qr, kc, vc = oracle.rope_kv_append(q, k, v, kc0, vc0, start, 1e5, True, True)
    assert np.array_equal(qr, oracle.rope(q, start, 1e5, True))
    assert np.array_equal(kc[start:start + T], oracle.f16_round(oracle.rope(k, start, 1e5, True)))
    assert np.array_equal(vc[start:start + T], oracle.f16_round(v))
    rest = np.r_[0:start, start + T:cap]
    assert np.all(kc[rest] == 7.0) and np.all(vc[rest] == -7.0)
    _, kc32, _ = oracle.rope_kv_append(q, k, v, kc0, vc0, start, 1e5, False, False)
    assert np.array_equal(kc32[start:start + T], oracle.rope(k, start, 1e5, False))


# ---------------------------------------------------------------------------------------------- decode projections

def _proj_kat():
    return json.loads((GOLDEN / "proj_kat.json").read_text())


def _close(got, expected, atol, rtol, label):
    e = np.asarray(expected, np.float64).reshape(-1)
    g = np.asarray(got, np.float64).reshape(-1)
    bad = np.abs(g - e) > atol + rtol * np.abs(e)
    print(f"[metrics] oracle {label}: max-abs {float(np.abs(g - e).max()):.2e} (atol {atol}, rtol {rtol})")
    assert not bad.any(), f"{label}: element {int(np.argmax(bad))}"


def test_linear_rmsnorm_silu_known_answers():
    """CPUOps.linear (f32 and f16 weights, and the single-row mat-vec of decode), rmsNorm and silu restated, against
    the reference's fixtures ops.json["linear"], ["rmsnorm"], ["silu"] at OperationTests.swift:24-53's tolerances."""
    c = _proj_kat()
    tol = c["tolerance"]
    lin = c["linear"]
    m, k, n = lin["m"], lin["k"], lin["n"]
    x = np.array(lin["x"], np.float32).reshape(m, k)
    w = np.array(lin["w"], np.float32).reshape(n, k)
    y = oracle.linear(x, np.frombuffer(w.tobytes(), np.uint8), "f32", n)
    _close(y, lin["expected"], *tol["linear"], "linear f32")
    y16 = oracle.linear(x, oracle.quantize(w, "f16"), "f16", n)
    _close(y16, lin["expected_f16"], *tol["linear"], "linear f16")
    _close(oracle.linear(x[:1], oracle.quantize(w, "f16"), "f16", n), lin["expected_f16"][:n], *tol["linear"],
           "mat-vec f16")
    rn = c["rmsnorm"]
    xr = np.array(rn["x"], np.float32).reshape(rn["shape"])
    _close(oracle.rmsnorm(xr, np.array(rn["w"], np.float32), rn["eps"]), rn["expected"], *tol["rmsnorm"], "rmsnorm")
    si = c["silu"]
    _close(oracle.silu(np.array(si["x"], np.float32)), si["expected"], *tol["silu"], "silu")


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_quantized_formats_known_answers(fmt):
    """GGUF q8_0 / q4_0 (testQuantizedFormatsAgainstGGUFReference, OperationTests.swift:88-107): the fixture's blocks
    (written by the gguf package) dequantise to its values, the quantised mat-vec matches its float mat-vec on the
    dequantised weights, and the reference quantiser restated here reproduces the blocks byte for byte."""
    import base64
    c = _proj_kat()
    q = c[fmt]
    k, n, m = q["k"], q["n"], q["m"]
    raw = np.frombuffer(base64.b64decode(q["blocks"]), np.uint8)
    assert raw.size == n * oracle.row_bytes(fmt, k)
    _close(oracle.dequantize(raw, fmt, n, k), q["dequantized"], *c["tolerance"]["dequantize"], f"{fmt} dequantize")
    x = np.array(q["x"], np.float32).reshape(m, k)
    _close(oracle.linear(x, raw, fmt, n), q["expected"], *c["tolerance"]["quantized_linear"], f"{fmt} linear")
    mine = oracle.quantize(np.array(q["original"], np.float32).reshape(n, k), fmt)
    assert np.array_equal(mine.reshape(-1), raw), f"{fmt} quantiser differs from the gguf blocks"


@pytest.mark.parametrize("fmt", ["f16", "q8_0", "q4_0"])
def test_decode_project_composition(fmt):
    """The fused projection (decode_fused.metal:32-122) on the CPU path is the composition of the restated ops:
    norm + three matrices (QKV), silu(W0 xn) * (W1 xn) (gate + up), and the residual add of the out-projection."""
    T, k = 2, 96
    x = oracle.splitmix_normal(41, (T, k))
    g = oracle.splitmix_normal(42, (k,))
    ws = [oracle.quantize(oracle.splitmix_normal(43 + i, (n, k)) * 0.05, fmt) for i, n in enumerate((8, 4, 4))]
    xn = oracle.rmsnorm(x, g, 1e-5)
    outs = oracle.decode_project(fmt, ws, x, norm_weight=g, eps=1e-5)
    for w, o in zip(ws, outs):
        assert np.array_equal(o, oracle.linear(xn, w, fmt, w.shape[0]))
    (gu,) = oracle.decode_project(fmt, ws[1:], x, norm_weight=g, eps=1e-5, silu_gate=True)
    a, b = oracle.linear(xn, ws[1], fmt, 4), oracle.linear(xn, ws[2], fmt, 4)
    assert np.array_equal(gu, (oracle.silu(a) * b).astype(np.float32))
    res = oracle.splitmix_normal(44, (T, 8))
    (yo,) = oracle.decode_project(fmt, ws[:1], x, add_to=[res])
    assert np.array_equal(yo, (res + oracle.linear(x, ws[0], fmt, 8)).astype(np.float32))
