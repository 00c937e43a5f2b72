"""FP64 NumPy restatement of the reference oracle.  TEST INFRASTRUCTURE ONLY.

Each function restates one function of ensigncode/paged-decode-lab's
``src/paged_decode/oracle.py`` (cited per function).  The arithmetic is the
published algorithm: gather the live tokens of a sequence through its page
table, score them against the query in float64, softmax with max subtraction,
and average the values.  The split-K helpers restate the reference's running
(maximum, denominator, numerator) update and its max-corrected merge.

Inputs follow the reference's layout:
  q      [batch, query_heads, head_dim]
  k, v   [physical_pages, page_size, kv_heads, head_dim]
  table  [batch, logical_pages] int, -1 padding allowed past the live pages
  lengths[batch] int
Query head ``h`` reads KV head ``h // (query_heads // kv_heads)``.
"""
from __future__ import annotations

import math
import numpy as np


def check_layout(batch, query_heads, kv_heads, head_dim, page_size, physical_pages):
    """Restates Layout.__post_init__ (oracle.py:20-27): integer, positive, Hq % Hkv == 0."""
    dims = (batch, query_heads, kv_heads, head_dim, page_size, physical_pages)
    for value in dims:
        if isinstance(value, (bool, np.bool_)) or not isinstance(value, (int, np.integer)):
            raise TypeError("layout dimensions must be integers, not booleans")
    if min(dims) <= 0:
        raise ValueError("layout dimensions must be positive")
    if query_heads % kv_heads:
        raise ValueError("query_heads must be divisible by kv_heads")


def validate_metadata(batch, page_size, physical_pages, table, lengths):
    """Restates validate_metadata (oracle.py:30-47); returns int32 copies."""
    table = np.asarray(table)
    lengths = np.asarray(lengths)
    if table.ndim != 2 or table.shape[0] != batch:
        raise ValueError("page table must have shape [batch, logical_pages]")
    if lengths.shape != (batch,):
        raise ValueError("lengths must have shape [batch]")
    if table.dtype.kind not in "iu" or lengths.dtype.kind not in "iu":
        raise TypeError("metadata must contain integers")
    capacity = table.shape[1] * page_size
    if (lengths < 0).any() or (lengths > capacity).any():
        raise ValueError("sequence length exceeds page table capacity")
    if max(table.shape[1], physical_pages) > np.iinfo(np.int32).max:
        raise ValueError("metadata exceeds int32 addressing limits")
    for row, length in enumerate(lengths.tolist()):
        live = table[row, : -(-int(length) // page_size)]
        if live.size and ((live < 0).any() or (live >= physical_pages).any()):
            raise ValueError("live logical page maps outside physical cache")
    return table.astype(np.int32, copy=True), lengths.astype(np.int32, copy=True)


def gather_cache(cache, pages, length, kv_head):
    """Restates gather_cache (oracle.py:50-56).

    Token ``t`` of a sequence lives in physical page ``pages[t // T]`` at slot
    ``t % T``; only the ``length`` live tokens are read, so -1 padding past them
    is never dereferenced.  Returns float64 [length, head_dim].
    """
    page_size = cache.shape[1]
    if length == 0:
        return np.zeros((0, cache.shape[-1]), dtype=np.float64)
    token = np.arange(int(length))
    physical = np.asarray(pages)[token // page_size]
    return np.asarray(cache[physical, token % page_size, kv_head], dtype=np.float64)


def dense_attention(q, k, v, table, lengths):
    """Restates dense_attention (oracle.py:59-71): FP64 softmax attention per (b, h).

    A sequence of length 0 yields a zero row.  Returns float64 [B, Hq, D].
    """
    batch, query_heads, head_dim = q.shape
    group = query_heads // k.shape[2]
    out = np.zeros((batch, query_heads, head_dim), dtype=np.float64)
    inv_sqrt_d = 1.0 / math.sqrt(head_dim)
    for b in range(batch):
        length = int(lengths[b])
        if length == 0:
            continue
        for h in range(query_heads):
            keys = gather_cache(k, table[b], length, h // group)
            values = gather_cache(v, table[b], length, h // group)
            scores = (keys @ np.asarray(q[b, h], dtype=np.float64)) * inv_sqrt_d
            weights = np.exp(scores - scores.max())
            out[b, h] = (weights @ values) / weights.sum()
    return out


def partial_softmax(scores, values):
    """Restates partial_softmax (oracle.py:74-85).

    Streams (score, value) pairs through the running triple (m, l, n):
    m' = max(m, s); n' = n*exp(m-m') + exp(s-m')*value; l' likewise.
    An empty input returns the identity (-inf, 0, zeros).
    """
    running_max = -np.inf
    denominator = 0.0
    numerator = np.zeros(np.shape(values)[-1], dtype=np.float64)
    for score, value in zip(scores, values):
        new_max = max(running_max, score)
        keep = np.exp(running_max - new_max)
        take = np.exp(score - new_max)
        numerator = numerator * keep + take * np.asarray(value, dtype=np.float64)
        denominator = denominator * keep + take
        running_max = new_max
    return running_max, denominator, numerator


def merge_partials(partials):
    """Restates merge_partials (oracle.py:88-96).

    Partials with l == 0 are empty and skipped before any exponential, so an
    all-empty list gives zeros instead of NaN.
    """
    live = [p for p in partials if p[1] > 0]
    if not live:
        return np.zeros_like(partials[0][2])
    top = max(p[0] for p in live)
    denominator = sum(np.exp(m - top) * l for m, l, _ in live)
    numerator = sum(np.exp(m - top) * n for m, _, n in live)
    return numerator / denominator


def split_bounds(length, split_tokens):
    """The reference's context partitions: range(0, max(len, 1), split) (oracle.py:110-111)."""
    if split_tokens <= 0:
        raise ValueError("split_tokens must be positive")
    return [(start, min(start + split_tokens, int(length)))
            for start in range(0, max(int(length), 1), split_tokens)]


def streaming_attention(q, k, v, table, lengths, split_tokens=256, warps=4):
    """Restates streaming_attention (oracle.py:99-117).

    Each context partition is streamed by ``warps`` interleaved token subsets
    (token start+w, start+w+warps, ...), exactly as the reference kernel's
    four warps do, and all partials are combined with merge_partials.
    """
    batch, query_heads, head_dim = q.shape
    group = query_heads // k.shape[2]
    out = np.zeros((batch, query_heads, head_dim), dtype=np.float64)
    inv_sqrt_d = 1.0 / math.sqrt(head_dim)
    for b in range(batch):
        length = int(lengths[b])
        for h in range(query_heads):
            keys = gather_cache(k, table[b], length, h // group)
            values = gather_cache(v, table[b], length, h // group)
            scores = (keys @ np.asarray(q[b, h], dtype=np.float64)) * inv_sqrt_d
            parts = []
            for start, stop in split_bounds(length, split_tokens):
                for w in range(warps):
                    parts.append(partial_softmax(scores[start + w:stop:warps],
                                                 values[start + w:stop:warps]))
            out[b, h] = merge_partials(parts)
    return out


def algorithmic_bytes(q_shape, kv_heads, elem_bytes, table, lengths, page_size):
    """Bytes one decode step must move at minimum.

    Unique live (physical page, token slot) K and V rows for every KV head,
    plus q, the FP32 output and the live page-table entries.  A physical page
    shared by several sequences counts once per token slot it holds live data
    for (shared prefixes are read once by an ideal kernel).
    """
    batch, query_heads, head_dim = q_shape
    table = np.asarray(table)
    slots = []
    table_entries = 0
    for b in range(batch):
        length = int(lengths[b])
        table_entries += -(-length // page_size)
        token = np.arange(length, dtype=np.int64)
        slots.append(table[b][token // page_size].astype(np.int64) * page_size + token % page_size)
    unique = np.unique(np.concatenate(slots)).size if slots else 0
    kv = 2 * unique * kv_heads * head_dim * elem_bytes
    return kv + batch * query_heads * head_dim * (elem_bytes + 4) + table_entries * 4
