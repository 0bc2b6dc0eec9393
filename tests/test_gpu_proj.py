"""Fused decode projections on the GPU (alpaca_decode_project) against the CPU oracle, through the C ABI.

The oracle composes alpaca.swift's CPUOps.rmsNorm / linear / silu / add (pinned to the reference's ops.json fixtures
in tests/test_oracle.py) the way the dec_* kernels compose them (decode_fused.metal:32-122); bounds are the
reference's own for those operations (OperationTests.swift:36-53, :88-107): f16 weights |gpu - cpu| <= 5e-6 +
1e-5 |cpu|, q8_0 / q4_0 <= 2e-5 + 1e-5 |cpu|. Weights are drawn N(0, 1/k) so outputs are O(1), as in a model.

Shapes: SmolLM2-135M (hidden 576, 9/3 heads of 64, FFN 1536) and SmolLM2-1.7B (hidden 2048, FFN 8192) layer
projections — Q/K/V with the attention norm, the out-projection with its residual, gate + up with the FFN norm and
SiLU, down with its residual, a norm + logits projection with an odd row count — plus the reference fixture's k = 96,
whose 102-byte q8_0 / 54-byte q4_0 rows put blocks at both 4-byte phases and a block at the very end of the matrix.
Token counts 1 (alpaca.swift's decode), 3 and 6 (a batched decode step: one and two passes of staged rows).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = {"f16": (5e-6, 1e-5), "q8_0": (2e-5, 1e-5), "q4_0": (2e-5, 1e-5)}


def _weights(seed: int, n: int, k: int, fmt: str):
    w = oracle.splitmix_normal(seed, (n, k)) / np.sqrt(k)
    blocks = oracle.quantize(w.astype(np.float32), fmt)
    return blocks, torch.from_numpy(blocks).cuda()


def _check(got, ref, fmt, label):
    atol, rtol = TOL[fmt]
    g = got.cpu().numpy().astype(np.float64)
    e = np.asarray(ref, np.float64)
    err = np.abs(g - e)
    print(f"[metrics] project {label}: max-abs {float(err.max()):.3e}, max |cpu| {float(np.abs(e).max()):.2f}")
    assert np.isfinite(g).all(), label
    bad = err > atol + rtol * np.abs(e)
    assert not bad.any(), f"{label}: {int(bad.sum())} elements out of bound, worst {float(err.max()):.3e}"


LAYERS = {
    # name: (k, (q rows, k rows, v rows), ffn)
    "135M": (576, (576, 192, 192), 1536),
    "1.7B": (2048, (2048, 2048, 2048), 8192),
}


@pytest.mark.parametrize("fmt", ["f16", "q8_0", "q4_0"])
@pytest.mark.parametrize("shape", list(LAYERS))
@pytest.mark.parametrize("tokens", [1, 3, 6])
def test_decode_layer_projections(cuda_lib, fmt, shape, tokens):
    """One decode layer's projections as alpaca.swift's fused path issues them (MetalLlamaModel.swift:344-354):
    QKV with the attention norm, the out-projection added to the residual, gate + up with the FFN norm and SiLU, down
    added to the residual."""
    from alpaca_b200 import decode_project, device_status
    k, (nq, nk, nv), ffn = LAYERS[shape]
    seed = 9000 + 100 * tokens + len(shape)
    x = oracle.splitmix_normal(seed, (tokens, k))
    g_att = 1.0 + 0.1 * oracle.splitmix_normal(seed + 1, (k,))
    g_ffn = 1.0 + 0.1 * oracle.splitmix_normal(seed + 2, (k,))
    wq, wq_d = _weights(seed + 3, nq, k, fmt)
    wk, wk_d = _weights(seed + 4, nk, k, fmt)
    wv, wv_d = _weights(seed + 5, nv, k, fmt)
    wo, wo_d = _weights(seed + 6, k, nq, fmt)
    wg, wg_d = _weights(seed + 7, ffn, k, fmt)
    wu, wu_d = _weights(seed + 8, ffn, k, fmt)
    wdn, wdn_d = _weights(seed + 9, k, ffn, fmt)
    dev = torch.device("cuda")
    xd = torch.from_numpy(x).to(dev)
    ga, gf = torch.from_numpy(g_att).to(dev), torch.from_numpy(g_ffn).to(dev)

    # Q / K / V with the fused norm (decodeQKV)
    outs = [torch.full((tokens, n), float("nan"), device=dev) for n in (nq, nk, nv)]
    decode_project([wq_d, wk_d, wv_d], fmt, k, xd, outs, norm_weight=ga, eps=1e-5)
    refs = oracle.decode_project(fmt, [wq, wk, wv], x, norm_weight=g_att, eps=1e-5)
    device_status()
    for name, o, r in zip("QKV", outs, refs):
        _check(o, r, fmt, f"{shape} {fmt} T={tokens} {name} (norm)")

    # the out-projection added to the residual (decodeProjection add: true): context = the Q output here
    ctx = refs[0]
    resid = torch.from_numpy(x.copy()).to(dev)
    decode_project([wo_d], fmt, nq, torch.from_numpy(ctx).to(dev), [resid], add=True)
    (ref_o,) = oracle.decode_project(fmt, [wo], ctx, add_to=[x])
    device_status()
    _check(resid, ref_o, fmt, f"{shape} {fmt} T={tokens} out-proj + residual")

    # gate + up with the FFN norm and SiLU (decodeGateUp), then down added to the residual
    gate = torch.full((tokens, ffn), float("nan"), device=dev)
    decode_project([wg_d, wu_d], fmt, k, xd, [gate], norm_weight=gf, eps=1e-5, silu_gate=True)
    (ref_g,) = oracle.decode_project(fmt, [wg, wu], x, norm_weight=g_ffn, eps=1e-5, silu_gate=True)
    device_status()
    _check(gate, ref_g, fmt, f"{shape} {fmt} T={tokens} gate*up (norm, silu)")
    resid2 = torch.from_numpy(x.copy()).to(dev)
    decode_project([wdn_d], fmt, ffn, torch.from_numpy(ref_g).to(dev), [resid2], add=True)
    (ref_d,) = oracle.decode_project(fmt, [wdn], ref_g, add_to=[x])
    device_status()
    _check(resid2, ref_d, fmt, f"{shape} {fmt} T={tokens} down + residual")


@pytest.mark.parametrize("fmt", ["f16", "q8_0", "q4_0"])
def test_logits_projection_and_block_phases(cuda_lib, fmt):
    """Norm + logits projection with an odd row count (the final decodeProjection of MetalLlamaModel.swift:377), and
    k = 96: rows of 102 (q8_0) / 54 (q4_0) bytes start at both 4-byte phases and the last block ends the matrix."""
    from alpaca_b200 import decode_project, device_status
    dev = torch.device("cuda")
    for k, n, tokens in ((576, 4099, 1), (96, 37, 2)):
        x = oracle.splitmix_normal(77 + k, (tokens, k))
        g = 1.0 + 0.1 * oracle.splitmix_normal(78 + k, (k,))
        w, wd = _weights(79 + k, n, k, fmt)
        out = torch.full((tokens, n), float("nan"), device=dev)
        decode_project([wd], fmt, k, torch.from_numpy(x).to(dev), [out], norm_weight=torch.from_numpy(g).to(dev),
                       eps=1e-5)
        device_status()
        (ref,) = oracle.decode_project(fmt, [w], x, norm_weight=g, eps=1e-5)
        _check(out, ref, fmt, f"logits {fmt} k={k} rows={n} T={tokens}")


def test_strided_rows_and_untouched_padding(cuda_lib):
    """Input and output rows with strides wider than their rows: every output element of the call is written once,
    the padding between rows is left as it was."""
    from alpaca_b200 import decode_project, device_status
    dev = torch.device("cuda")
    k, n, tokens = 576, 200, 3
    x = oracle.splitmix_normal(90, (tokens, k))
    w, wd = _weights(91, n, k, "q8_0")
    xbuf = torch.zeros((tokens, k + 64), device=dev)
    xbuf[:, :k] = torch.from_numpy(x).to(dev)
    ybuf = torch.full((tokens, n + 40), 7.0, device=dev)
    decode_project([wd], "q8_0", k, xbuf[:, :k], [ybuf[:, :n]])
    device_status()
    (ref,) = oracle.decode_project("q8_0", [w], x)
    _check(ybuf[:, :n], ref, "q8_0", "strided rows")
    assert torch.all(ybuf[:, n:] == 7.0)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_single_token_quantised_shapes(cuda_lib, fmt):
    """Single-token quantised calls (the int8 tensor-core form) beyond the model layers above: Q/K/V with the norm
    whose row counts end in partial 8-row tiles, one of them a middle matrix (8-row tiles straddling two matrices);
    80001 rows at k = 256 (one 8-block job per tile, hundreds of tiles per CTA); SwiGLU at k = 8192; the
    out-projection's residual add on a row count that ends in a partial tile."""
    from alpaca_b200 import decode_project, device_status
    dev = torch.device("cuda")
    # Q / K / V, k = 512, norm: rows 1000 + 264 + 261 and 1000 + 259 + 261
    k = 512
    x = oracle.splitmix_normal(301, (1, k))
    g = 1.0 + 0.1 * oracle.splitmix_normal(302, (k,))
    for rows in ((1000, 264, 261), (1000, 259, 261)):
        ws = [_weights(303 + i, n, k, fmt) for i, n in enumerate(rows)]
        outs = [torch.full((1, n), float("nan"), device=dev) for n in rows]
        decode_project([w[1] for w in ws], fmt, k, torch.from_numpy(x).to(dev), outs,
                       norm_weight=torch.from_numpy(g).to(dev), eps=1e-5)
        device_status()
        refs = oracle.decode_project(fmt, [w[0] for w in ws], x, norm_weight=g, eps=1e-5)
        for name, o, r in zip("QKV", outs, refs):
            _check(o, r, fmt, f"{fmt} k={k} {name} rows={rows}")
    # 80001 rows of k = 256
    k, n = 256, 80001
    x = oracle.splitmix_normal(311, (1, k))
    w, wd = _weights(312, n, k, fmt)
    out = torch.full((1, n), float("nan"), device=dev)
    decode_project([wd], fmt, k, torch.from_numpy(x).to(dev), [out])
    device_status()
    (ref,) = oracle.decode_project(fmt, [w], x)
    _check(out, ref, fmt, f"{fmt} k={k} rows={n}")
    # SwiGLU, k = 8192, 1003 rows
    k, n = 8192, 1003
    x = oracle.splitmix_normal(321, (1, k))
    g = 1.0 + 0.1 * oracle.splitmix_normal(322, (k,))
    (wg, wg_d), (wu, wu_d) = _weights(323, n, k, fmt), _weights(324, n, k, fmt)
    gate = torch.full((1, n), float("nan"), device=dev)
    decode_project([wg_d, wu_d], fmt, k, torch.from_numpy(x).to(dev), [gate],
                   norm_weight=torch.from_numpy(g).to(dev), eps=1e-5, silu_gate=True)
    device_status()
    (ref_g,) = oracle.decode_project(fmt, [wg, wu], x, norm_weight=g, eps=1e-5, silu_gate=True)
    _check(gate, ref_g, fmt, f"{fmt} k={k} gate*up rows={n}")
    # out-projection + residual, 2050 rows
    k, n = 2048, 2050
    x = oracle.splitmix_normal(331, (1, k))
    resid0 = oracle.splitmix_normal(332, (1, n))
    w, wd = _weights(333, n, k, fmt)
    resid = torch.from_numpy(resid0.copy()).to(dev)
    decode_project([wd], fmt, k, torch.from_numpy(x).to(dev), [resid], add=True)
    device_status()
    (ref,) = oracle.decode_project(fmt, [w], x, add_to=[resid0])
    _check(resid, ref, fmt, f"{fmt} k={k} rows={n} + residual")
