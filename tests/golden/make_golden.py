#!/usr/bin/env python3
"""Regenerates the golden vectors in tests/golden/ from the alpaca.swift checkout.

Run where an alpaca.swift checkout is available (path as the argument or in $ALPACA_REFERENCE):

    python tests/golden/make_golden.py /path/to/alpaca.swift

Outputs (committed; nothing reads the reference at test time):
  attention_kat.json  the reference's own attention known-answer case, Tests/AlpacaCoreTests/Fixtures/ops.json
                      ["attention"] (generated upstream by Scripts/generate_op_fixtures.py:64-74 as a float64
                      torch SDPA), copied verbatim, plus the reference tolerances of OperationTests.swift:72-86.
  softmax_kat.json    ops.json["softmax"] (±30-sigma inputs, float64 expected), OperationTests softmax case.
  rope_kat.json       ops.json["rope"] (generated upstream by Scripts/generate_op_fixtures.py:50-62 in float64, both
                      pair conventions), plus the 2e-6 tolerance of OperationTests.swift:63-70.
  proj_kat.json       ops.json["linear"] (f32 and f16 weights), ["rmsnorm"], ["silu"], ["q8_0"] and ["q4_0"] (GGUF
                      blocks, base64, from the gguf package upstream, with their dequantisation, a mat-vec and the
                      float originals the quantiser must reproduce byte for byte), with the tolerances of
                      OperationTests.swift:24-53 and :88-107: the operations the fused decode projections compose.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ALPACA_REFERENCE")
    if not src:
        sys.exit("usage: make_golden.py /path/to/alpaca.swift  (or set ALPACA_REFERENCE)")
    ref = Path(src)
    ops = json.loads((ref / "Tests/AlpacaCoreTests/Fixtures/ops.json").read_text())
    att = dict(ops["attention"])
    att["source"] = "alpaca.swift Tests/AlpacaCoreTests/Fixtures/ops.json[\"attention\"]"
    att["tolerance"] = {"atol": 3e-6, "rtol": 1e-5, "from": "Tests/AlpacaCoreTests/OperationTests.swift:85"}
    (HERE / "attention_kat.json").write_text(json.dumps(att))
    sm = dict(ops["softmax"])
    sm["source"] = "alpaca.swift Tests/AlpacaCoreTests/Fixtures/ops.json[\"softmax\"]"
    (HERE / "softmax_kat.json").write_text(json.dumps(sm))
    rp = dict(ops["rope"])
    rp["source"] = "alpaca.swift Tests/AlpacaCoreTests/Fixtures/ops.json[\"rope\"]"
    rp["tolerance"] = {"atol": 2e-6, "from": "Tests/AlpacaCoreTests/OperationTests.swift:68-69"}
    (HERE / "rope_kat.json").write_text(json.dumps(rp))
    proj = {name: dict(ops[name]) for name in ("linear", "rmsnorm", "silu", "q8_0", "q4_0")}
    proj["source"] = "alpaca.swift Tests/AlpacaCoreTests/Fixtures/ops.json [linear, rmsnorm, silu, q8_0, q4_0]"
    proj["tolerance"] = {"linear": [5e-6, 1e-5], "rmsnorm": [2e-6, 2e-6], "silu": [1e-6, 1e-6],
                         "quantized_linear": [2e-5, 1e-5], "dequantize": [1e-6, 1e-6],
                         "from": "Tests/AlpacaCoreTests/OperationTests.swift:24-53, 88-107"}
    (HERE / "proj_kat.json").write_text(json.dumps(proj))

    print("wrote", sorted(p.name for p in HERE.iterdir()))


if __name__ == "__main__":
    main()
