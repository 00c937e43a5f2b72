"""Build the native library in-tree: paged_decode/libpaged_decode_b200.so.

    python paged-decode-lab_b200/build.py [--force] [--verbose] [--jobs N]

nvcc cross-compiles for sm_100a only (no GPU needed).  The kernel
instantiations live in eight translation units (dtype x head_dim x page_size)
that compile in parallel into _build/, then link into one shared library.
cudart is linked statically, so the library needs nothing but the NVIDIA
driver at run time.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
BUILD = ROOT / "_build"
OUT = ROOT / "paged_decode" / "libpaged_decode_b200.so"
SOURCES = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + [INCLUDE / "paged_decode.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
         "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, deps) -> bool:
    return not target.exists() or any(target.stat().st_mtime < d.stat().st_mtime for d in deps)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    objects = []
    todo = []
    for src in SOURCES:
        obj = BUILD / (src.name + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *HEADERS]):
            cmd = [nvcc(), *FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            todo.append(cmd)
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 1)
    if todo:
        with ThreadPoolExecutor(max_workers=jobs) as pool:
            results = list(pool.map(lambda c: subprocess.run(c, capture_output=True, text=True), todo))
        failed = [r for r in results if r.returncode]
        for r in results:
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
        if failed:
            raise RuntimeError(f"{len(failed)} translation unit(s) failed to compile")
    if force or todo or _stale(OUT, objects):
        subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(OUT), *map(str, objects)], check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(args.force, args.verbose, args.jobs))
