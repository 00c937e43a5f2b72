"""Seeded synthetic decode workloads.

``make_metadata`` and ``make_tensors`` reproduce ensigncode/paged-decode-lab's
generators (src/paged_decode/workload.py:7-35) draw for draw, so equal seeds give
bit-identical page tables, lengths and tensors (pinned by golden fixtures made
with the reference).  The ``config*`` builders produce the five BASELINE
workloads, two of which (ragged + shared prefix, and the large-batch pool) need
their own generators because ``make_metadata`` cannot express them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from .layout import Layout


def make_metadata(batch, heads, kv_heads, dim, context, page_size, *, seed=123, ragged=True):
    """Fragmented page table + lengths, identical to the reference's for equal seeds.

    Draw order (workload.py:13-18): one permutation of batch*width page ids,
    then ``batch`` lengths uniform in [max(1, context//4), context]; non-ragged
    workloads overwrite every length with ``context``; row 0 is always full.
    Entries past each row's live pages become -1.
    """
    if min(batch, heads, kv_heads, dim, context, page_size) <= 0:
        raise ValueError("workload dimensions must be positive")
    rng = np.random.default_rng(seed)
    width = math.ceil(context / page_size)
    table = rng.permutation(batch * width).reshape(batch, width).astype(np.int32)
    lengths = rng.integers(max(1, context // 4), context + 1, size=batch, dtype=np.int32)
    if not ragged:
        lengths[:] = context
    lengths[0] = context
    layout = Layout(batch, heads, kv_heads, dim, page_size, batch * width)
    live = -(-lengths.astype(np.int64) // page_size)
    table[np.arange(width)[None, :] >= live[:, None]] = -1
    return layout, table, lengths


def make_tensors(layout, *, device="cuda", dtype=None, seed=123):
    """q [B,Hq,D] then k, v [P,T,Hkv,D], all N(0,1) from one generator on ``device``.

    Same generator, seed and draw order as the reference (workload.py:25-35).
    """
    import torch
    dtype = torch.float16 if dtype is None else dtype
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn((layout.batch, layout.query_heads, layout.head_dim),
                    device=device, dtype=dtype, generator=gen)
    cache_shape = (layout.physical_pages, layout.page_size, layout.kv_heads, layout.head_dim)
    k = torch.randn(cache_shape, device=device, dtype=dtype, generator=gen)
    v = torch.randn(cache_shape, device=device, dtype=dtype, generator=gen)
    return q, k, v


@dataclass
class Workload:
    """One BASELINE configuration: metadata plus how to draw its tensors."""
    name: str
    layout: Layout
    table: np.ndarray
    lengths: np.ndarray
    split_tokens: int
    dtype: str = "float16"
    std: float = 1.0
    seed: int = 123
    notes: dict = field(default_factory=dict)

    def tensors(self, device="cuda"):
        import torch
        q, k, v = make_tensors(self.layout, device=device, dtype=getattr(torch, self.dtype),
                               seed=self.seed)
        if self.std != 1.0:
            for t in (q, k, v):
                t.mul_(self.std)
        return q, k, v


def config1(seed=123):
    """GQA, Llama-3-8B heads: B4, 32:8, D128, every sequence 4096, page 16, split 256."""
    layout, table, lengths = make_metadata(4, 32, 8, 128, 4096, 16, seed=seed, ragged=False)
    return Workload("config1_b4_gqa32x8_l4096", layout, table, lengths, 256, seed=seed)


def config2(seed=123, batch=32, context=8192, page_size=16, prefix_pages=64):
    """Ragged + shared-prefix GQA: B32, 32:8, D128, page 16, split 256.

    Lengths are uniform integers in [0, context]; two sequences are forced empty
    and two get a tail that does not end on a page boundary.  A quarter of the
    sequences (only ones at least ``prefix_pages`` pages long) map their first
    ``prefix_pages`` logical pages to one shared run of physical pages.  All
    other pages are a random permutation of a pool sized to the total demand.
    """
    rng = np.random.default_rng(seed)
    lengths = rng.integers(0, context + 1, size=batch).astype(np.int64)
    order = rng.permutation(batch)
    empty, tails = order[:2], order[2:4]
    lengths[empty] = 0
    for i in tails:
        if lengths[i] % page_size == 0:
            lengths[i] = max(1, lengths[i] - int(rng.integers(1, page_size)))
    prefix_tokens = prefix_pages * page_size
    eligible = [int(i) for i in order[4:] if lengths[i] >= prefix_tokens]
    sharers = sorted(eligible[: batch // 4])
    for i in order[4:]:
        if len(sharers) >= batch // 4:
            break
        if int(i) not in sharers:
            lengths[i] = int(rng.integers(prefix_tokens, context + 1))
            sharers.append(int(i))
    sharers = sorted(sharers)
    pages = -(-lengths // page_size)
    own = pages.copy()
    own[sharers] -= prefix_pages
    pool = prefix_pages + int(own.sum())
    perm = rng.permutation(pool).astype(np.int32)
    prefix, rest = perm[:prefix_pages], perm[prefix_pages:]
    width = -(-context // page_size)
    table = np.full((batch, width), -1, dtype=np.int32)
    cursor = 0
    for b in range(batch):
        start = 0
        if b in sharers:
            table[b, :prefix_pages] = prefix
            start = prefix_pages
        n = int(pages[b]) - start
        table[b, start:start + n] = rest[cursor:cursor + n]
        cursor += n
    layout = Layout(batch, 32, 8, 128, page_size, pool)
    return Workload("config2_b32_ragged_shared_prefix", layout, table,
                    lengths.astype(np.int32), 256, seed=seed,
                    notes={"empty": sorted(int(i) for i in empty),
                           "ragged_tail": sorted(int(i) for i in tails),
                           "shared_prefix": sharers, "prefix_pages": prefix_pages})


def config3(variant, seed=123):
    """Head-ratio sweep at context 2048, B64, page 32, split 128.

    (a) MHA 32:32 D64 FP32, (b) MQA 32:1 D128 FP16, (c) GQA 64:8 D128 FP16.
    """
    heads, kv_heads, dim, dtype = {"a": (32, 32, 64, "float32"),
                                   "b": (32, 1, 128, "float16"),
                                   "c": (64, 8, 128, "float16")}[variant]
    layout, table, lengths = make_metadata(64, heads, kv_heads, dim, 2048, 32,
                                           seed=seed, ragged=False)
    return Workload(f"config3{variant}_b64_{heads}x{kv_heads}_d{dim}", layout, table, lengths,
                    128, dtype=dtype, seed=seed)


def config4(seed=123, batch=256, low=1024, high=8192, page_size=16):
    """Large batch, Llama-3-70B heads: B256, 64:8, D128, page 16, N(0, 0.5) (std 0.5).

    Lengths uniform integers in [low, high]; pages are a random permutation of
    a pool sized to the total demand.
    """
    rng = np.random.default_rng(seed)
    lengths = rng.integers(low, high + 1, size=batch).astype(np.int64)
    pages = -(-lengths // page_size)
    pool = int(pages.sum())
    perm = rng.permutation(pool).astype(np.int32)
    width = -(-high // page_size)
    table = np.full((batch, width), -1, dtype=np.int32)
    cursor = 0
    for b in range(batch):
        n = int(pages[b])
        table[b, :n] = perm[cursor:cursor + n]
        cursor += n
    layout = Layout(batch, 64, 8, 128, page_size, pool)
    return Workload(f"config4_b{batch}_gqa64x8_l1k_8k", layout, table, lengths.astype(np.int32),
                    256, std=0.5, seed=seed)


def config5(seed=123):
    """Long context: B2, 32:8, D128, 131072 tokens each, page 32, 8192 pages, split 256."""
    layout, table, lengths = make_metadata(2, 32, 8, 128, 131072, 32, seed=seed, ragged=False)
    return Workload("config5_b2_gqa32x8_l131072", layout, table, lengths, 256, seed=seed)


CONFIGS = {
    "c1": config1, "c2": config2, "c3a": lambda seed=123: config3("a", seed),
    "c3b": lambda seed=123: config3("b", seed), "c3c": lambda seed=123: config3("c", seed),
    "c4": config4, "c5": config5,
    # config 4's generator with 32 sequences: a config-4-shaped case small
    # enough for a full profiler capture (its traffic scales to config 4)
    "c4s": lambda seed=123: config4(seed, batch=32),
}
