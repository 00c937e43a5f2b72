"""Build the native library in-tree: paged_decode/libpaged_decode_b200.so.

    python paged-decode-lab_b200/build.py [--force] [--verbose]

nvcc cross-compiles for sm_100a only (no GPU needed).  cudart is linked
statically, so the library depends on nothing but the NVIDIA driver at run time.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
OUT = ROOT / "paged_decode" / "libpaged_decode_b200.so"
SOURCES = [CSRC / "pd_api.cu", CSRC / "pd_plan.cpp"]
DEPENDS = SOURCES + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + [INCLUDE / "paged_decode.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    return OUT.exists() and all(OUT.stat().st_mtime >= p.stat().st_mtime for p in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH,
           "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3", "-shared",
           "-I", str(INCLUDE), "-o", str(OUT), *map(str, SOURCES)]
    if verbose:
        cmd.insert(4, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.verbose))
    sys.exit(0)
