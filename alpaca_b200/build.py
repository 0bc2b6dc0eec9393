"""Builds alpaca_b200/libalpaca_cuda.so in-tree for sm_100a with nvcc (no JIT cache, no torch extension).

    python -m alpaca_b200.build [--force] [--verbose]

The library exports exactly the C ABI of include/alpaca_cuda.h.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libalpaca_cuda.so"
SOURCES = ["api.cu", "attn_decode.cu", "attn_general.cu", "attn_prefill_sm100.cu", "rope_kv.cu", "decode_proj.cu"]
HEADERS = ["common.cuh", "internal.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-Wall"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libalpaca_cuda.so")
    return cand


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "alpaca_cuda.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *CFLAGS, "-I", str(ROOT / "include"), "-c", str(CSRC / src), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs, "-Xlinker", "--version-script=" + str(CSRC / "exports.map")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))


if __name__ == "__main__":
    main()
