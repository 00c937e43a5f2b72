"""Plan contract: the cache geometry and the host-side metadata checks.

Mirrors ``Layout`` and ``validate_metadata`` of ensigncode/paged-decode-lab
(src/paged_decode/oracle.py:11-47), which the reference's ``DecodePlan`` uses
to reject bad metadata before anything reaches the GPU.  Same fields, same
accepted inputs, same exception types; tests pin the verdicts against
fixtures produced by the reference itself.
"""
from __future__ import annotations

from dataclasses import dataclass
from numbers import Integral

import numpy as np


@dataclass(frozen=True)
class Layout:
    """Cache geometry: q [batch, query_heads, head_dim];
    k, v [physical_pages, page_size, kv_heads, head_dim]."""
    batch: int
    query_heads: int
    kv_heads: int
    head_dim: int
    page_size: int
    physical_pages: int

    def __post_init__(self):
        values = tuple(vars(self).values())
        if any(isinstance(x, (bool, np.bool_)) or not isinstance(x, Integral) for x in values):
            raise TypeError("layout dimensions must be integers, not booleans")
        if min(values) <= 0:
            raise ValueError("layout dimensions must be positive")
        if self.query_heads % self.kv_heads:
            raise ValueError("query_heads must be divisible by kv_heads")

    @property
    def group(self) -> int:
        """Query heads per KV head (G)."""
        return self.query_heads // self.kv_heads


def validate_metadata(layout: Layout, table, lengths):
    """Check a page table [batch, logical_pages] and lengths [batch].

    Every live logical page (the first ceil(len/page_size) of a row) must name a
    physical page in [0, physical_pages); entries past them are padding and may
    be -1.  Returns int32 copies, so later edits of the caller's arrays cannot
    reach a plan.
    """
    table, lengths = np.asarray(table), np.asarray(lengths)
    if table.ndim != 2 or table.shape[0] != layout.batch:
        raise ValueError("page table must have shape [batch, logical_pages]")
    if lengths.shape != (layout.batch,):
        raise ValueError("lengths must have shape [batch]")
    if table.dtype.kind not in "iu" or lengths.dtype.kind not in "iu":
        raise TypeError("metadata must contain integers")
    if (lengths < 0).any() or (lengths > table.shape[1] * layout.page_size).any():
        raise ValueError("sequence length exceeds page table capacity")
    if max(table.shape[1], layout.physical_pages) > np.iinfo(np.int32).max:
        raise ValueError("metadata exceeds int32 addressing limits")
    live_pages = -(-lengths.astype(np.int64) // layout.page_size)
    live = np.arange(table.shape[1])[None, :] < live_pages[:, None]
    used = table[live]
    if used.size and ((used < 0).any() or (used >= layout.physical_pages).any()):
        raise ValueError("live logical page maps outside physical cache")
    return table.astype(np.int32, copy=True), lengths.astype(np.int32, copy=True)
