"""Builds the in-tree C-ABI library ``rus_b200/liblmce.so`` with nvcc for sm_100a.

The library is compiled ahead of time (no JIT cache), so the built ``.so``
travels with the source tree. ``python -m rus_b200.build`` rebuilds it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_PATH = PKG_DIR / "liblmce.so"
SOURCES = [CSRC / "lmce_capi.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "lmce.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")
    return cand


def compile_command(out: Path = LIB_PATH, extra: list[str] | None = None) -> list[str]:
    return [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-cudart",
        "static",
        "-I",
        str(INCLUDE),
        *(extra or []),
        "-o",
        str(out),
        *[str(s) for s in SOURCES],
    ]


def needs_build(out: Path = LIB_PATH) -> bool:
    if not out.exists():
        return True
    mtime = out.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in DEPS)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile liblmce.so if it is missing or older than its sources."""
    if not force and not needs_build():
        return LIB_PATH
    cmd = compile_command()
    if verbose:
        print(" ".join(cmd), flush=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd[cmd.index("-o") + 1] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
