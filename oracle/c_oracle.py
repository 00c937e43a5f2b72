"""ctypes front end for ``paged_oracle.c``.  TEST INFRASTRUCTURE ONLY.

``build()`` compiles ``liboracle.so`` next to this file with gcc; ``dense_attention``
calls it with NumPy arrays.  Same contract as ``paged_oracle.dense_attention``
(FP64 output [B, Hq, D], zero rows for empty sequences), threaded over
(sequence, KV head) units.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None


def build(force: bool = False) -> Path:
    src = _HERE / "paged_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["gcc", "-O3", "-march=x86-64-v2", "-fPIC", "-shared", "-pthread",
                        "-o", str(_LIB_PATH), str(src), "-lm"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        fn = lib.pdo_dense_attention
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] + [ctypes.c_void_p] * 2 + \
                      [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_int]
        _lib = lib
    return _lib


def dense_attention(q, k, v, table, lengths, threads: int | None = None):
    q = np.ascontiguousarray(q)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    if q.dtype not in (np.float16, np.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q/k/v must share float16 or float32 dtype")
    table = np.ascontiguousarray(table, dtype=np.int32)
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    batch, q_heads, head_dim = q.shape
    _, page_size, kv_heads, _ = k.shape
    out = np.empty((batch, q_heads, head_dim), dtype=np.float64)
    threads = threads or os.cpu_count() or 1
    rc = _load().pdo_dense_attention(
        q.ctypes.data, k.ctypes.data, v.ctypes.data, q.dtype.itemsize,
        table.ctypes.data, lengths.ctypes.data, batch, q_heads, kv_heads, head_dim,
        page_size, table.shape[1], out.ctypes.data, int(threads))
    if rc != 0:
        raise RuntimeError("C oracle failed (bad arguments or out of memory)")
    return out
