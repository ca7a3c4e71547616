"""Builds libnesle_b200.so in-tree for sm_100a (nvcc; no JIT cache).

    python -m nesle_b200.build          # incremental
    python -m nesle_b200.build --force  # rebuild
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
LIB = PKG / "libnesle_b200.so"
SOURCES = ["kernels.cu", "capi.cu", "formats.cpp"]
DEPS = SOURCES + ["kernels.h", "nes_core.cuh", "nes_render.cuh", "nes_v2.cuh", "nesle_state.h", "formats.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnesle_b200.so")
    return exe


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / d for d in DEPS] + [ROOT / "include" / "nesle_b200.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-std=c++20", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
           "-I", str(ROOT / "include"), "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=str(CSRC))
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
