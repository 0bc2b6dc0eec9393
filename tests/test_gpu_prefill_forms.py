"""The prefill forms the library selects by environment switch (read once per process), each checked by re-running
the prefill parity tests (and the forced bounded-wait timeout) in a child process with the switch set: the
three-tile head_dim-64 form (ALPACA_PREFILL_TILES=3: 64-row KV blocks, one softmax thread per row, three query
tiles per work item) and the one-thread-per-row two-tile form (ALPACA_PREFILL_ROWS=1). The default forms are
covered by the parent run."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
PREFILL_TESTS = ("prefill or config2 or config4 or tiled or layouts or views or rescale or pad_rows or strided "
                 "or block_index or causal or forced_wait")


@pytest.mark.parametrize("env", [{"ALPACA_PREFILL_TILES": "3"}, {"ALPACA_PREFILL_ROWS": "1"}],
                         ids=["three_tiles", "one_thread_rows"])
def test_prefill_form_parity(cuda_lib, env):
    cmd = [sys.executable, "-m", "pytest", "tests/test_gpu_parity.py", "tests/test_gpu_paged.py",
           "tests/test_gpu_failure.py", "-m", "gpu", "-q", "-x", "-p", "no:cacheprovider", "-k", PREFILL_TESTS]
    r = subprocess.run(cmd, cwd=ROOT, env={**os.environ, **env}, capture_output=True, text=True, timeout=900)
    tail = "\n".join(r.stdout.splitlines()[-25:])
    print(f"[metrics] prefill form {env}: {r.stdout.strip().splitlines()[-1] if r.stdout.strip() else ''}")
    assert r.returncode == 0, tail
    assert " passed" in r.stdout, tail
