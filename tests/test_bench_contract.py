"""bench.py without a GPU: its options parse, every leg has its switch, and the reference arm (the CPU restatement of
alpaca.swift's attention on the host cores) prints the one JSON line of the bench contract. The reference arm runs
a 512-token prompt here to stay quick; on a GPU box it runs the config-2 length."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _bench(*args, timeout=600):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=timeout)


def test_options_parse_and_every_leg_can_be_left_out():
    r = _bench("--help", timeout=120)
    assert r.returncode == 0, r.stderr
    for leg in ("decode", "rope", "proj", "cpu", "e2e", "cfg4", "cfg5", "chunked", "sessions"):
        assert f"--no-{leg}" in r.stdout, leg
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--tokens", "--layers"):
        assert opt in r.stdout, opt


def test_reference_arm_prints_the_contract_line():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "3", "--tokens", "512")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 3 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"] and cpu["sample"]
    assert cpu["single_thread"]["cores"] == 1 and cpu["single_thread"]["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["config"]["tokens"] == 512 and line["config"]["layers"] == 30


def test_both_arms_draw_the_same_inputs_and_count_the_same_flops():
    """The GPU arm's torch generator (synth_normal) and the reference arm's C generator (oracle.splitmix_normal) give
    the same N(0,1) draws bit for bit, an odd count and a seed past 2^63 included, so both arms time the same
    config-2 inputs. Config 2's step is 30 layers of 2 * 9 * 64 * T * (T + 1) FLOPs."""
    import numpy as np

    import oracle
    sys.path.insert(0, str(ROOT))
    import bench
    for seed in (0, bench.SEED_CFG2, 2 ** 63 + 5):
        a = bench.synth_normal(seed, (4097, 3)).numpy()
        assert np.array_equal(a, oracle.splitmix_normal(seed, (4097, 3))), seed
    assert bench.LAYERS * bench.flops_prefill(bench.T_PREFILL) == 579_962_142_720
