"""The C ABI from a plain C program (tests/c_client/abi_client.c): built with gcc against include/alpaca_cuda.h and
linked to libalpaca_cuda.so and the CUDA runtime only, as a Swift / Go / C host binds it. The oracle library is
linked as the checker of the GPU leg."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CUDA = Path("/usr/local/cuda")


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    from alpaca_b200 import build
    build.build()
    import oracle
    oracle.build()
    exe = tmp_path_factory.mktemp("c_client") / "abi_client"
    lib_dirs = [ROOT / "alpaca_b200", ROOT / "oracle", CUDA / "lib64"]
    cmd = ["gcc", "-O1", "-std=c11", "-I", str(ROOT / "include"), "-I", str(ROOT / "oracle"), "-I",
           str(CUDA / "include"), str(ROOT / "tests" / "c_client" / "abi_client.c"), "-o", str(exe)]
    for d in lib_dirs:
        cmd += ["-L", str(d), f"-Wl,-rpath,{d}"]
    cmd += ["-l:libalpaca_cuda.so", "-l:liboracle.so", "-lcudart", "-lm"]
    subprocess.run(cmd, check=True)
    return exe


def test_c_client_host_entry_points(client):
    r = subprocess.run([str(client)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "host entry points ok" in r.stdout


@pytest.mark.gpu
def test_c_client_prefill_and_decode_on_gpu(client):
    r = subprocess.run([str(client), "gpu"], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "prefill through the C ABI" in r.stdout and "ragged decode through the C ABI" in r.stdout
