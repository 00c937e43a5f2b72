"""The reference's own CUDA operator, built for sm_100a.  TEST INFRASTRUCTURE ONLY.

``build(reference_root)`` compiles ensigncode/paged-decode-lab's two native
files where they lie (src/paged_decode/csrc/decode.cu and bindings.cpp) into
``oracle/_ref/ref_paged_decode.so`` with torch's extension builder and our own
flags (sm_100a only).  Nothing is copied into this repository.  The .so travels
to the GPU box with the snapshot; ``load()`` imports it there without needing
the sources.

``RefPlan`` drives the built kernel the way the reference's DecodePlan does
(workspace shapes of runtime.py:64-68, launch arguments of decode.cu:197-200):
used by GPU tests as a second, independent implementation and by the bench's
reference arm as "the reference kernel on one B200".
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import math
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
MODULE = "ref_paged_decode"
SO_PATH = REF_DIR / f"{MODULE}.so"


def build(reference_root, force=False):
    """Compile the reference kernel from the checkout at ``reference_root``; returns
    the .so path, or None if its sources are absent (a prebuilt .so is kept)."""
    csrc = Path(reference_root) / "src" / "paged_decode" / "csrc"
    sources = [csrc / "bindings.cpp", csrc / "decode.cu"]
    if not all(s.exists() for s in sources):
        return SO_PATH if SO_PATH.exists() else None
    if SO_PATH.exists() and not force:
        return SO_PATH
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load
    build_dir = REF_DIR / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    load(name=MODULE, sources=[str(s) for s in sources], build_directory=str(build_dir),
         extra_cflags=["-O3"], extra_cuda_cflags=["-O3", "-lineinfo"], verbose=False)
    built = build_dir / f"{MODULE}.so"
    built.replace(SO_PATH)
    return SO_PATH


def load():
    """Import the prebuilt reference extension (requires torch already importable)."""
    import torch  # noqa: F401 - the extension links against torch's libraries
    if not SO_PATH.exists():
        raise FileNotFoundError(f"{SO_PATH} not built")
    loader = importlib.machinery.ExtensionFileLoader(MODULE, str(SO_PATH))
    spec = importlib.util.spec_from_file_location(MODULE, str(SO_PATH), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


class RefPlan:
    """Workspace + launch arguments for the reference kernel (one decode shape)."""

    def __init__(self, layout, table, lengths, *, device, split_tokens=256, merge="serial"):
        import torch
        self.ext = load()
        self.split_tokens = split_tokens
        max_len = int(max(lengths)) if len(lengths) else 0
        splits = max(1, math.ceil(max_len / split_tokens))
        parts = splits * 4
        self.merge_mode = 1 if (merge == "shared" and parts <= 4096) else 0
        rows = (layout.batch, layout.query_heads, parts)
        self.table = torch.as_tensor(table, dtype=torch.int32, device=device)
        self.lengths = torch.as_tensor(lengths, dtype=torch.int32, device=device)
        self.numerator = torch.empty((*rows, layout.head_dim), dtype=torch.float32, device=device)
        self.stats = torch.empty((*rows, 2), dtype=torch.float32, device=device)
        self.out = torch.empty((layout.batch, layout.query_heads, layout.head_dim),
                               dtype=torch.float32, device=device)

    def run(self, q, k, v):
        self.ext.decode(q, k, v, self.table, self.lengths, self.numerator, self.stats, self.out,
                        self.split_tokens, self.merge_mode)
        return self.out
