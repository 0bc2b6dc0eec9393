"""GPU kernels vs the CPU oracle, through the C ABI (ctypes) — the parity tests proper.

The first three tests restate alpaca.swift's own kernel tests with their shape matrices, seeds and bounds
(Tests/AlpacaMetalTests/KernelTests.swift:76-88, :124-144, :146-170); the rest cover the BASELINE.json
configurations (f16 inputs: max-abs <= 2e-3 vs the oracle fed the same f16-rounded Q/K/V; f32 inputs: <= 1e-5)
and the layouts the ABI accepts (batched sequences, strides, chunked prefill, f16 output, f32 queries).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests._util import compare, max_abs_check

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F16_BOUND = 2e-3   # f16 inputs, fp32 accumulate
F32_BOUND = 1e-5   # f32 inputs


def _uniform_stream(seed, *shapes, scale=1.0):
    """Sequential SplitMix.nextFloat draws split into `shapes` (one generator, as the reference tests draw)."""
    n = [int(np.prod(s)) for s in shapes]
    flat = oracle.splitmix_uniform(seed, (sum(n),), scale)
    out, o = [], 0
    for s, c in zip(shapes, n):
        out.append(flat[o:o + c].reshape(s))
        o += c
    return out


def test_attention_causal_gqa(cuda_lib):
    """KernelTests.testAttentionCausalGQA (:76-88): f16 KV within 2e-5/1e-4, f32 KV within 2e-6/1e-5."""
    from alpaca_b200 import attention
    for tokens, start, heads, kv, hd in [(1, 0, 4, 2, 64), (1, 100, 9, 3, 64), (5, 0, 9, 3, 64), (7, 20, 8, 2, 128),
                                         (3, 1, 6, 6, 32)]:
        cap = start + tokens + 3
        q = oracle.splitmix_uniform(11, (tokens, heads, hd))
        k = oracle.splitmix_uniform(12, (cap, kv, hd))
        v = oracle.splitmix_uniform(13, (cap, kv, hd))
        cpu = oracle.attention(q, oracle.f16_round(k), oracle.f16_round(v), start)
        compare(attention(q, k, v, start), cpu, 2e-5, 1e-4, f"attention f16-KV T={tokens} start={start} H={heads}/{kv} hd={hd}")
        cpu32 = oracle.attention(q, k, v, start)
        compare(attention(q, k, v, start, kv="f32"), cpu32, 2e-6, 1e-5,
                f"attention f32-KV T={tokens} start={start} H={heads}/{kv} hd={hd}")


DECODE_CASES = [(0, 9, 3, 64), (1, 9, 3, 64), (7, 9, 3, 64), (255, 9, 3, 64), (256, 9, 3, 64), (257, 9, 3, 64),
                (511, 9, 3, 64), (1000, 9, 3, 64), (2047, 9, 3, 64), (300, 8, 2, 128), (700, 8, 8, 64),
                (90, 32, 4, 128), (500, 4, 1, 64)]


@pytest.mark.parametrize("force_split", [False, True])
def test_split_decode_matches_cpu_reference(cuda_lib, force_split):
    """testSplitDecodeAttentionMatchesCPUReference (:124-144): split boundaries, GQA 1..8, d 64/128; < 2e-6.
    With force_split every case (contexts 1..2048) runs the split kernel."""
    from alpaca_b200 import Kernel, attention
    for start, heads, kv, hd in DECODE_CASES:
        cap = start + 1
        q, k, v = _uniform_stream(start * 7 + heads, (1, heads, hd), (cap, kv, hd), (cap, kv, hd))
        cpu = oracle.attention(q, oracle.f16_round(k), oracle.f16_round(v), start)
        gpu = attention(q, k, v, start, kind=Kernel.DECODE_SPLIT if force_split else Kernel.AUTO)
        max_abs_check(gpu, cpu, 2e-6, f"split decode ctx={cap} H={heads}/{kv} hd={hd}")


TILED_CASES = [(8, 0, 9, 3, 64), (31, 0, 9, 3, 64), (32, 0, 9, 3, 64), (33, 0, 9, 3, 64), (100, 0, 9, 3, 64),
               (64, 200, 9, 3, 64), (45, 7, 8, 2, 128), (128, 128, 4, 4, 128), (17, 3, 6, 3, 64), (200, 0, 8, 2, 64)]


def test_tiled_attention_matches_cpu_reference(cuda_lib):
    """testTiledAttentionMatchesCPUReference (:146-170): partial tiles, chunked starts, GQA 1..4, d 64/128;
    maxAbs < 1.5e-3 and all finite."""
    from alpaca_b200 import attention
    for t, start, heads, kv, hd in TILED_CASES:
        cap = start + t
        q, k, v = _uniform_stream(t * 131 + start, (t, heads, hd), (cap, kv, hd), (cap, kv, hd))
        cpu = oracle.attention(q, oracle.f16_round(k), oracle.f16_round(v), start)
        for precision in ("exact", "fast"):
            gpu = attention(q, k, v, start, precision=precision)
            max_abs_check(gpu, cpu, 1.5e-3, f"tiled attention T={t} start={start} H={heads}/{kv} hd={hd} {precision}")


def test_tensor_core_prefill_on_tiled_cases(cuda_lib):
    """The tcgen05 kernel forced on every tiled case (head_dim 64 and 128) and on short prefills (T < 8 go to the
    general kernel under the dispatch policy)."""
    from alpaca_b200 import Kernel, attention
    cases = list(TILED_CASES) + [(2, 0, 9, 3, 64), (5, 9, 4, 1, 64), (1, 300, 9, 3, 64), (3, 70, 8, 2, 128),
                                 (1, 65, 4, 4, 128)]
    for t, start, heads, kv, hd in cases:
        cap = start + t
        q, k, v = _uniform_stream(t * 131 + start, (t, heads, hd), (cap, kv, hd), (cap, kv, hd))
        cpu = oracle.attention(q, oracle.f16_round(k), oracle.f16_round(v), start)
        gpu = attention(q, k, v, start, kind=Kernel.PREFILL_TC)
        max_abs_check(gpu, cpu, 1.5e-3, f"tcgen05 prefill T={t} start={start} H={heads}/{kv} hd={hd}")


# ---------------------------------------------------------------------------------------------- BASELINE configs

def _normal(seed, shape, f16=True):
    x = oracle.splitmix_normal(seed, shape)
    return oracle.f16_round(x) if f16 else x


def test_config1_exact_f32(cuda_lib):
    """Config 1: T=128, 9/3 heads, d=64, f32 N(0,1), scale 1/8, causal -> max-abs <= 1e-5 (general fp32 kernel)."""
    from alpaca_b200 import Kernel, attention
    T, H, kvh, d = 128, 9, 3, 64
    q, k, v = _normal(20260101, (T, H, d), False), _normal(20260102, (T, kvh, d), False), _normal(20260103, (T, kvh, d), False)
    cpu = oracle.attention(q, k, v, 0)
    gpu = attention(q, k, v, 0, kv="f32")
    max_abs_check(gpu, cpu, F32_BOUND, "config 1 f32 exact")
    gpu = attention(q, k, v, 0, kv="f32", kind=Kernel.GENERAL)
    max_abs_check(gpu, cpu, F32_BOUND, "config 1 f32 exact (forced general)")


def _device_prefill(qs, ks, vs, start, out_dtype=torch.float32, kind=None, q_dtype=torch.float16):
    """Batched device call: qs [S,T,H,d], ks/vs [S,L,Hkv,d] numpy f32 (already f16-representable)."""
    from alpaca_b200 import Kernel, attention_device, device_status
    dev = torch.device("cuda")
    q = torch.from_numpy(qs).to(dev).to(q_dtype)
    k = torch.from_numpy(ks).to(dev).half()
    v = torch.from_numpy(vs).to(dev).half()
    out = torch.empty(qs.shape, dtype=out_dtype, device=dev)
    attention_device(q, k, v, out, start_position=start, kind=kind if kind is not None else Kernel.AUTO)
    device_status()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("T", [2048, 4096])
def test_config2_prefill_135m(cuda_lib, T):
    """Config 2: 135M shape causal prefill, 2 of the 30 independent layers batched as sequences, f16 N(0,1).
    T=2048 checked on every row; T=4096 on every 7th (head, token) row (rows are independent, so sampling is
    exact)."""
    H, kvh, d, S = 9, 3, 64, 2
    qs = np.stack([_normal(30 + s, (T, H, d)) for s in range(S)])
    ks = np.stack([_normal(40 + s, (T, kvh, d)) for s in range(S)])
    vs = np.stack([_normal(50 + s, (T, kvh, d)) for s in range(S)])
    gpu = _device_prefill(qs, ks, vs, 0)
    for s in range(S):
        rows = np.arange(0, H * T, 1 if T <= 2048 else 7)  # row index = h*T + t
        cpu = oracle.attention_rows(qs[s], ks[s], vs[s], 0, rows)
        sel = oracle.rows_mask(rows, T, H)
        max_abs_check(gpu[s][sel], cpu[sel], F16_BOUND, f"config 2 prefill T={T} layer {s}")


def test_prefill_head_dim_128(cuda_lib):
    """head_dim 128 (the reference's attn_tensor_hd128 / attn_prefill_hd128_kv16): 2 sequences x 2048 tokens, 8/2
    heads, f16 N(0,1), every 5th (head, token) row against the oracle at the f16 bound."""
    T, H, kvh, d, S = 2048, 8, 2, 128, 2
    qs = np.stack([_normal(60 + s, (T, H, d)) for s in range(S)])
    ks = np.stack([_normal(62 + s, (T, kvh, d)) for s in range(S)])
    vs = np.stack([_normal(64 + s, (T, kvh, d)) for s in range(S)])
    gpu = _device_prefill(qs, ks, vs, 0)
    for s in range(S):
        rows = np.arange(0, H * T, 5)
        cpu = oracle.attention_rows(qs[s], ks[s], vs[s], 0, rows)
        sel = oracle.rows_mask(rows, T, H)
        max_abs_check(gpu[s][sel], cpu[sel], F16_BOUND, f"prefill d=128 T={T} seq {s}")


def test_config3_decode_ragged_batch(cuda_lib):
    """Config 3: batch 64 single-token decode, 9/3 heads, f16 KV with per-sequence lengths uniform in [1,4096]
    (device ctx_lens), N(0,1)."""
    from alpaca_b200 import Kernel, attention_device, device_status
    S, H, kvh, d, CAP = 64, 9, 3, 64, 4096
    rng = np.random.default_rng(20260103)
    lens = rng.integers(1, CAP + 1, size=S).astype(np.int32)
    q = _normal(61, (S, 1, H, d), False)
    k = _normal(62, (S, CAP, kvh, d))
    v = _normal(63, (S, CAP, kvh, d))
    dev = torch.device("cuda")
    qd = torch.from_numpy(q).to(dev)
    kd, vd = torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half()
    out = torch.empty((S, 1, H, d), dtype=torch.float32, device=dev)
    attention_device(qd, kd, vd, out, ctx_lens=torch.from_numpy(lens).to(dev), max_ctx_len=CAP,
                     kind=Kernel.DECODE_SPLIT)
    device_status()
    gpu = out.cpu().numpy()
    for s in range(S):
        L = int(lens[s])
        cpu = oracle.attention(q[s], k[s], v[s], L - 1, length=L)
        max_abs_check(gpu[s], cpu, 1e-5, f"config 3 decode seq {s} ctx={L}")


def test_config4_prefill_360m_batch(cuda_lib):
    """Config 4 shape: 15/5 heads, d=64, 8 sequences x 4096 tokens in one batched call; every 31st row of every
    sequence checked."""
    S, T, H, kvh, d = 8, 4096, 15, 5, 64
    qs = np.stack([_normal(70 + s, (T, H, d)) for s in range(S)])
    ks = np.stack([_normal(80 + s, (T, kvh, d)) for s in range(S)])
    vs = np.stack([_normal(90 + s, (T, kvh, d)) for s in range(S)])
    gpu = _device_prefill(qs, ks, vs, 0)
    for s in range(S):
        rows = np.arange(s, H * T, 31)
        cpu = oracle.attention_rows(qs[s], ks[s], vs[s], 0, rows)
        sel = oracle.rows_mask(rows, T, H)
        max_abs_check(gpu[s][sel], cpu[sel], F16_BOUND, f"config 4 prefill seq {s}")


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_layouts(cuda_lib, d):
    """Chunked prefill over a longer cache, f32 queries (converted in the workspace), f16 output, strided rows."""
    from alpaca_b200 import Kernel
    T, start, H, kvh = 300, 517, 12, 4
    q = _normal(101, (1, T, H, d))
    k = _normal(102, (1, start + T + 40, kvh, d))
    v = _normal(103, (1, start + T + 40, kvh, d))
    cpu = oracle.attention(q[0], k[0], v[0], start)
    for qdt in (torch.float16, torch.float32):
        for odt in (torch.float32, torch.float16):
            gpu = _device_prefill(q, k, v, start, out_dtype=odt, kind=Kernel.PREFILL_TC, q_dtype=qdt)
            bound = F16_BOUND + (1e-3 if odt == torch.float16 else 0.0)
            max_abs_check(gpu[0], cpu, bound, f"prefill chunk d={d} start={start} q={qdt} out={odt}")


def test_strided_cache_views(cuda_lib):
    """K/V as views into one interleaved [rows, 2, Hkv, d] buffer (row stride 2*Hkv*d), all three kernels."""
    from alpaca_b200 import Kernel, attention_device, device_status
    T, start, H, kvh, d = 40, 90, 8, 2, 64
    L = start + T
    q = _normal(111, (T, H, d))
    kv = _normal(112, (L, 2, kvh, d))
    dev = torch.device("cuda")
    kvd = torch.from_numpy(kv).to(dev).half()
    kd, vd = kvd[:, 0], kvd[:, 1]
    for kind, tq in ((Kernel.PREFILL_TC, T), (Kernel.GENERAL, T), (Kernel.DECODE_SPLIT, 1)):
        qq = q[-tq:]
        st = L - tq
        cpu = oracle.attention(qq, np.ascontiguousarray(kv[:, 0]), np.ascontiguousarray(kv[:, 1]), st)
        out = torch.empty(qq.shape, dtype=torch.float32, device=dev)
        attention_device(torch.from_numpy(qq).to(dev).half(), kd, vd, out, start_position=st, kind=kind)
        device_status()
        max_abs_check(out.cpu().numpy(), cpu, F16_BOUND, f"strided cache {kind.name}")


@pytest.mark.parametrize("d", [64, 128])
def test_pad_rows_never_read(cuda_lib, d):
    """Rows past start+tokens may hold anything (here NaN): outputs stay finite and equal the clean run."""
    from alpaca_b200 import Kernel, attention_device, device_status
    T, start, H, kvh = 100, 30, 9, 3
    L = start + T
    q = _normal(121, (T, H, d))
    k = _normal(122, (L, kvh, d))
    v = _normal(123, (L, kvh, d))
    cpu = oracle.attention(q, k, v, start)
    dev = torch.device("cuda")
    kd = torch.full((L + 200, kvh, d), float("nan"), dtype=torch.float16, device=dev)
    vd = torch.full((L + 200, kvh, d), float("nan"), dtype=torch.float16, device=dev)
    kd[:L] = torch.from_numpy(k).to(dev).half()
    vd[:L] = torch.from_numpy(v).to(dev).half()
    for kind in (Kernel.PREFILL_TC, Kernel.GENERAL):
        out = torch.empty((T, H, d), dtype=torch.float32, device=dev)
        attention_device(torch.from_numpy(q).to(dev).half(), kd, vd, out, start_position=start, kind=kind)
        device_status()
        max_abs_check(out.cpu().numpy(), cpu, F16_BOUND, f"NaN tail {kind.name} d={d}")


@pytest.mark.parametrize("d", [64, 128])
def test_large_scores_rescale_path(cuda_lib, d):
    """Scores with a large spread (q scaled by 6, rows whose max jumps between blocks) exercise the O rescale.
    The data is outside the N(0,1) regime the 2e-3 bound is stated for (attention is nearly one-hot), so the bound
    is the reference's own tolerance basis for f16 P/K/V (KernelTests.swift:116-121): 3 * 2^-11 * max|V|."""
    from alpaca_b200 import Kernel, attention_device, device_status
    T, H, kvh = 512, 4, 2
    q = oracle.f16_round(oracle.splitmix_normal(131, (T, H, d)) * 6.0)
    k = _normal(132, (T, kvh, d))
    k[300:310] *= 4.0   # late keys with much larger scores than the first blocks
    k = oracle.f16_round(k)
    v = _normal(133, (T, kvh, d))
    cpu = oracle.attention(q, k, v, 0)
    dev = torch.device("cuda")
    out = torch.empty((T, H, d), dtype=torch.float32, device=dev)
    attention_device(torch.from_numpy(q).to(dev).half(), torch.from_numpy(k).to(dev).half(),
                     torch.from_numpy(v).to(dev).half(), out, kind=Kernel.PREFILL_TC)
    device_status()
    max_abs_check(out.cpu().numpy(), cpu, 3 * 2.0 ** -11 * float(np.abs(v).max()), f"rescale path d={d}")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("odt", [torch.float32, torch.float16])
def test_prefill_output_views(cuda_lib, d, odt):
    """The prefill output written through its tensor map (TMA stores): into views of wider buffers (padded token and
    sequence strides, two sequences, a last tile that ends mid-tile) it equals the contiguous output bit for bit, and
    the padding around the view is left untouched."""
    from alpaca_b200 import Kernel, attention_device, device_status
    S, T, start, H, kvh = 2, 200, 60, 6, 2
    L = start + T
    dev = torch.device("cuda")
    q = torch.from_numpy(_normal(121, (S, T, H, d))).to(dev).half()
    k = torch.from_numpy(_normal(122, (S, L, kvh, d))).to(dev).half()
    v = torch.from_numpy(_normal(123, (S, L, kvh, d))).to(dev).half()
    ref = torch.empty((S, T, H, d), dtype=odt, device=dev)
    attention_device(q, k, v, ref, start_position=start, kind=Kernel.PREFILL_TC)
    big = torch.full((S, T + 8, H + 2, d), 7.0, dtype=odt, device=dev)  # token stride (H+2)*d, seq stride (T+8)*...
    view = big[:, 3:3 + T, 1:1 + H]
    attention_device(q, k, v, view, start_position=start, kind=Kernel.PREFILL_TC)
    device_status()
    assert torch.equal(view, ref)
    pad = torch.ones_like(big, dtype=torch.bool)
    pad[:, 3:3 + T, 1:1 + H] = False
    assert torch.all(big[pad] == 7.0)


@pytest.mark.parametrize("d", [64, 128])
def test_decode_output_ordered_for_next_launch(cuda_lib, d):
    """Every context fits one split unit (128 rows at head_dim 64, 64 at 128) while max_ctx_len allows several, so
    the split kernel finishes every sequence itself and the combine kernel has nothing to merge. A plain torch
    kernel launched right after on the same stream, with no synchronisation in between, must still read the split
    kernel's output: stream order holds across the dependent launches."""
    from alpaca_b200 import Kernel, attention_device, device_status
    S, H, kvh, cap = 64, 9, 3, 4096
    unit = 128 if d == 64 else 64
    rng = np.random.default_rng(41 + d)
    lens = rng.integers(1, unit + 1, size=S).astype(np.int32)
    q = _normal(141, (S, 1, H, d), False)
    k = _normal(142, (S, unit, kvh, d))
    v = _normal(143, (S, unit, kvh, d))
    dev = torch.device("cuda")
    qd = torch.from_numpy(q).to(dev)
    kd, vd = torch.from_numpy(k).to(dev).half(), torch.from_numpy(v).to(dev).half()
    ld = torch.from_numpy(lens).to(dev)
    out = torch.full((S, 1, H, d), float("nan"), dtype=torch.float32, device=dev)
    ws = torch.empty(1 << 24, dtype=torch.uint8, device=dev)
    for _ in range(3):
        out.fill_(float("nan"))
        attention_device(qd, kd, vd, out, ctx_lens=ld, max_ctx_len=cap, kind=Kernel.DECODE_SPLIT, workspace=ws)
        twice = out * 2.0  # next launch on the same stream, no sync
        device_status()
        got = (twice / 2.0).cpu().numpy()
        for s in range(S):
            L = int(lens[s])
            ref = oracle.attention(q[s], k[s], v[s], L - 1, length=L)
            max_abs_check(got[s], ref, 1e-5, f"ordered decode output d={d} seq {s} ctx={L}")
