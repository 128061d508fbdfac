"""Builds libb200tx.so, the sm_100a kernel library behind the C-ABI in include/b200tx.h.

The library is one translation unit (csrc/b200tx.cu includes every kernel header) compiled by
nvcc for sm_100a only, with the CUDA runtime linked statically so the .so carries no dependency
on a particular libcudart next to torch's. The output goes in-tree, to
tiktoktechjam2026track3_b200/_lib/libb200tx.so, so it travels with the source tree.

Usage: python -m tiktoktechjam2026track3_b200.build [--verbose-ptxas]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC_DIR = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libb200tx.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found (set NVCC or put it on PATH)")


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu")) + sorted(CSRC_DIR.glob("*.cuh"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(verbose_ptxas: bool = False, force: bool = False) -> Path:
    if not force and not verbose_ptxas and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "--cudart",
        "static",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-shared",
        "-o",
        str(tmp),
        str(CSRC_DIR / "b200tx.cu"),
    ]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose-ptxas", action="store_true", help="print registers/spills per kernel")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(verbose_ptxas=args.verbose_ptxas, force=args.force))


if __name__ == "__main__":
    main()
