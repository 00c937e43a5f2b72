"""Host planner logic (no GPU): the balanced work list covers every live page once.

The plan's unit is a page tile of one group = (sequence, KV head, query-head
tile).  Invariants checked here, for many shapes and CTA counts:
  * every group's segments tile [0, ceil(len/T)) exactly, in order, no overlap;
  * every CTA streams floor or ceil of total_pages / num_ctas pages;
  * pieces: a group with one segment has piece -1, otherwise consecutive
    slots piece0 .. piece0+n-1, each used exactly once;
  * empty sequences appear as zero-page segments (they write zero rows);
  * the reference's split partitions (range(0, max(len,1), split)) are reported unchanged.
"""
import math

import numpy as np
import pytest

from oracle import paged_oracle
from paged_decode.layout import Layout
from paged_decode.runtime import inspect_plan
from paged_decode import workload


def check_worklist(layout, table, lengths, plan):
    info, segs, groups, offs = plan["info"], plan["segments"], plan["groups"], plan["cta_offsets"]
    T = layout.page_size
    G = layout.query_heads // layout.kv_heads
    gt = info["group_tile"]
    assert gt == (8 if G <= 8 else 16 if G <= 16 else 32)
    hg = info["heads_per_tile"]
    assert hg in (1, 2, 4, 8) and layout.kv_heads % hg == 0 and hg * gt // 8 <= 8
    # FP16 page tile (K + V of hg heads) within the 64 KiB target unless hg == 1
    assert hg == 1 or hg * 2 * layout.head_dim * 2 * T <= 64 * 1024
    splits = math.ceil(G / gt)
    kv_groups = layout.kv_heads // hg
    assert info["num_groups"] == layout.batch * kv_groups * splits
    # groups enumerate (b, KV-head group, query-head tile) in order
    for gi, g in enumerate(groups):
        b, rest = divmod(gi, kv_groups * splits)
        kg, s = divmod(rest, splits)
        assert tuple(g[:5]) == (b, kg * hg, s * gt, min(gt, G - s * gt), lengths[b])
    C = info["num_ctas"]
    assert offs[0] == 0 and offs[-1] == len(segs) and (np.diff(offs) >= 0).all()
    total = sum(-(-int(lengths[g[0]]) // T) for g in groups)
    assert info["total_pages"] == total
    # balance: equal page counts, or for the tcgen05 kernel equal counts of
    # 128-token steps with cuts on step boundaries of the group
    unit = 128 // T if info["engine"] == 1 else 1
    if unit > 1 and sum(-(-(-(-int(lengths[g[0]]) // T)) // unit) for g in groups) < 4 * C:
        unit = 1   # too few steps per CTA: balanced by pages
    per_cta = [sum(-(-int(s[2] - s[1]) // unit) for s in segs[offs[c]:offs[c + 1]]) for c in range(C)]
    if unit > 1:
        assert all(int(s[1]) % unit == 0 for s in segs)
    units = sum(-(-(-(-int(lengths[g[0]]) // T)) // unit) for g in groups)
    if units:
        assert min(per_cta) >= units // C and max(per_cta) <= -(-units // C)
    stride = info["slot_stride"]
    # FP16 plans: consumer warps per tile = hg * gt/8 <= 8; sub-pipelines by tile size
    cpt = hg * gt // 8
    assert cpt <= 8
    # one partial slot per segment when the kernel shape folds its sub-pipelines'
    # states inside the CTA (FP32, or four FP16 sub-pipelines), else one per sub-pipeline
    tile = 2 * layout.head_dim * 2 * T * hg
    nsub = 1 if tile >= 32768 else min(4, 8 // cpt)
    if info["engine"] == 1:
        # FP16 group tiles of 32 query heads: the tcgen05 kernel, one KV head per tile
        assert gt == 32 and hg == 1 and stride == 1
    else:
        assert stride == (1 if nsub >= 4 else max(1, nsub))
    covered = {gi: [] for gi in range(len(groups))}
    for c in range(C):
        for s in segs[offs[c]:offs[c + 1]]:
            covered[int(s[0])].append((int(s[1]), int(s[2]), int(s[3])))
    slot_ranges = []
    for gi, ranges in covered.items():
        pages = -(-int(groups[gi][4]) // T)
        ranges.sort()
        assert ranges, f"group {gi} has no segment"
        assert groups[gi][6] == len(ranges)
        if pages == 0:
            assert len(ranges) == 1 and ranges[0][:2] == (0, 0)
        else:
            assert ranges[0][0] == 0 and ranges[-1][1] == pages
            for (a0, a1, _), (b0, b1, _) in zip(ranges, ranges[1:]):
                assert a1 == b0 and a0 < a1
        slots = [r[2] for r in ranges]
        if groups[gi][5] < 0:
            # whole group on one CTA: direct output
            assert len(ranges) == 1 and stride == 1 and slots == [-1]
        else:
            base = int(groups[gi][5])
            assert sorted(slots) == [base + k * stride for k in range(len(ranges))]
            slot_ranges.append((base, base + len(ranges) * stride))
    slot_ranges.sort()
    assert all(a[1] == b[0] for a, b in zip(slot_ranges, slot_ranges[1:]))
    assert (slot_ranges[0][0] if slot_ranges else 0) == 0
    assert (slot_ranges[-1][1] if slot_ranges else 0) == info["num_pieces"]


@pytest.mark.parametrize("ctas", [1, 2, 3, 7, 64, 148, 1000])
@pytest.mark.parametrize("kv_heads,heads", [(2, 8), (1, 32), (4, 4), (1, 64), (2, 24), (8, 32), (6, 12)])
def test_worklist_invariants_small(ctas, kv_heads, heads):
    rng = np.random.default_rng(ctas * 31 + heads)
    layout = Layout(5, heads, kv_heads, 64 if heads % 3 else 128, 16, 60)
    lengths = np.array([0, 1, 17, 160, 191], dtype=np.int32)
    table = rng.integers(0, 60, size=(5, 12)).astype(np.int32)
    plan = inspect_plan(layout, table, lengths, split_tokens=33, num_ctas=ctas)
    check_worklist(layout, table, lengths, plan)
    assert plan["info"]["splits"] == math.ceil(191 / 33)


@pytest.mark.parametrize("name", ["c1", "c2", "c3b", "c5"])
def test_worklist_invariants_baseline_configs(name):
    w = workload.CONFIGS[name]()
    plan = inspect_plan(w.layout, w.table, w.lengths, split_tokens=w.split_tokens, num_ctas=148)
    check_worklist(w.layout, w.table, w.lengths, plan)
    info = plan["info"]
    assert info["num_ctas"] == 148
    assert info["splits"] == max(1, math.ceil(int(w.lengths.max()) / w.split_tokens))


def test_all_empty_batch_writes_zero_rows_only():
    layout = Layout(2, 4, 4, 64, 16, 1026)
    table = np.arange(1026, dtype=np.int32).reshape(2, 513)
    plan = inspect_plan(layout, table, np.array([0, 0], dtype=np.int32), split_tokens=257, num_ctas=148)
    assert plan["info"]["total_pages"] == 0 and plan["info"]["num_ctas"] == 1
    check_worklist(layout, table, np.array([0, 0]), plan)


def test_split_bounds_match_reference_partitions():
    for length in (0, 1, 255, 256, 257, 8193):
        for split in (1, 13, 256, 257):
            if length // split > 2000:
                continue
            expected = [(s, min(s + split, length)) for s in range(0, max(length, 1), split)]
            assert paged_oracle.split_bounds(length, split) == expected


def test_plan_errors_mirror_reference_messages():
    layout = Layout(1, 4, 2, 64, 16, 4)
    with pytest.raises(ValueError, match="split_tokens"):
        inspect_plan(layout, [[0, 1]], [17], split_tokens=0)
    with pytest.raises(ValueError, match="split_tokens"):
        inspect_plan(layout, [[0, 1]], [17], split_tokens=True)
    with pytest.raises(ValueError, match="outside physical cache"):
        inspect_plan(layout, [[0, 9]], [17])
    with pytest.raises(TypeError):
        inspect_plan(layout, [[0.0, 1.0]], [17])


@pytest.mark.parametrize("dim,page,kv_heads,dtype,expected", [
    (128, 16, 8, "float16", 8), (128, 32, 8, "float16", 4), (64, 16, 8, "float16", 8),
    (64, 32, 32, "float16", 8), (128, 32, 1, "float16", 1), (128, 16, 6, "float16", 2),
    (128, 16, 8, "float32", 2), (64, 32, 32, "float32", 2), (128, 32, 8, "float32", 1)])
def test_heads_per_tile_targets_64kib_fp16_32kib_fp32_tiles(dim, page, kv_heads, dtype, expected):
    layout = Layout(2, kv_heads * 4, kv_heads, dim, page, 8)
    plan = inspect_plan(layout, np.arange(8, dtype=np.int32).reshape(2, 4), [page * 4, 1], num_ctas=3,
                        dtype=dtype)
    assert plan["info"]["heads_per_tile"] == expected


def test_dynamic_plan_covers_each_sequence_up_to_its_capacity():
    """A dynamic plan's groups and segments cover max_lengths, not lengths."""
    layout = Layout(3, 8, 2, 128, 16, 30)
    table = np.arange(30, dtype=np.int32).reshape(3, 10)
    table[0, 2:] = -1                      # pages past the live length may be unallocated
    lengths = np.array([20, 0, 100], dtype=np.int32)
    max_lengths = np.array([60, 5, 160], dtype=np.int32)
    plan = inspect_plan(layout, table, lengths, num_ctas=7, max_lengths=max_lengths)
    assert plan["info"]["dynamic"] == 1 and plan["info"]["max_span"] == 160
    check_worklist(layout, table, max_lengths, plan)
    static = inspect_plan(layout, np.arange(30, dtype=np.int32).reshape(3, 10), lengths, num_ctas=7)
    assert static["info"]["dynamic"] == 0 and static["info"]["max_span"] == 100
    with pytest.raises(ValueError, match="max_lengths"):
        inspect_plan(layout, table, lengths, num_ctas=7, max_lengths=np.array([60, 5, 161]))
    with pytest.raises(ValueError, match="max_lengths"):
        inspect_plan(layout, table, lengths, num_ctas=7, max_lengths=np.array([19, 5, 160]))


@pytest.mark.parametrize("ctas", [1, 3, 7, 148, 1000])
@pytest.mark.parametrize("kv_heads,heads,dim,page", [(1, 32, 128, 32), (1, 64, 64, 16), (2, 48, 128, 16)])
def test_tcgen05_plans_cut_on_step_boundaries(ctas, kv_heads, heads, dim, page, monkeypatch):
    """PD_MQA_ENGINE=tcgen05 plans balance 128-token steps, not pages: every cut
    falls on a step boundary of its group and CTAs get equal step counts."""
    monkeypatch.setenv("PD_MQA_ENGINE", "tcgen05")
    rng = np.random.default_rng(ctas + heads)
    lengths = np.array([0, 1, 129, 1000, 4096, 77], dtype=np.int32)
    width = -(-int(lengths.max()) // page)
    layout = Layout(len(lengths), heads, kv_heads, dim, page, len(lengths) * width)
    table = rng.integers(0, layout.physical_pages, size=(len(lengths), width)).astype(np.int32)
    plan = inspect_plan(layout, table, lengths, num_ctas=ctas)
    assert plan["info"]["engine"] == 1
    check_worklist(layout, table, lengths, plan)


def test_tcgen05_plan_of_config_3b(monkeypatch):
    monkeypatch.setenv("PD_MQA_ENGINE", "tcgen05")
    w = workload.CONFIGS["c3b"]()
    plan = inspect_plan(w.layout, w.table, w.lengths, split_tokens=w.split_tokens, num_ctas=148)
    assert plan["info"]["engine"] == 1
    check_worklist(w.layout, w.table, w.lengths, plan)
