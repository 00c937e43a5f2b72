"""Pair plans: clusters of two CTAs that split each group and merge it in shared memory.

When the tcgen05 kernel serves a plan with an automatic CTA count, groups of
about equal length, and enough groups that two CTAs each fill at least 3/4 of
the SMs (BASELINE config 3b: 64 sequences of 2048 tokens, one KV head), the
planner gives CTAs 2g and 2g + 1 the two halves of group g, cut on a 128-token
step. The launch groups them in clusters of two. Each CTA sends the partial
(m, l, o) rows of the other CTA's 16 query heads into that CTA's shared memory
(distributed shared memory), and after a cluster barrier each merges and
writes its own 16 heads. No partial touches global memory, and there is no
grid barrier and no merge kernel.

The CPU tests pin the planner's choice and its work list. The GPU tests check
pair plans against the FP64 oracle on the shapes the kernel serves, forced with
PD_PAIR=1 where the default would not choose them: empty and one-page groups,
17 and 64 query heads per KV head, and head_dim 64 and pages of 16 tokens.
They also check (m, l) statistics against the one-CTA-per-SM plan, bit-equal
repeats and CUDA-graph replays, dynamic plans, and that the exchange launch
rejects pair plans.
"""
import ctypes
import os

import numpy as np
import pytest

from paged_decode import workload
from paged_decode.layout import Layout
from paged_decode.runtime import inspect_plan


def _uniform(batch, heads, kv_heads, dim, page, length, seed=5):
    rng = np.random.default_rng(seed)
    width = max(1, -(-length // page))
    layout = Layout(batch, heads, kv_heads, dim, page, batch * width)
    table = rng.permutation(batch * width).reshape(batch, width).astype(np.int32)
    return layout, table, np.full(batch, length, dtype=np.int32)


def _with_env(fn, **env):
    old = {k: os.environ.get(k) for k in env}
    try:
        for k, v in env.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
        return fn()
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _inspect(layout, table, lengths, pair=None, engine=None, **kw):
    return _with_env(lambda: inspect_plan(layout, table, lengths, **kw), PD_PAIR=pair, PD_MQA_ENGINE=engine)


def _check_pairs(layout, lengths, plan):
    """CTA 2g and 2g + 1 hold one segment each: the two halves of group g, cut
    on a step of 128 tokens (the first half rounded up), no partial slots."""
    info, segs, groups, offs = plan["info"], plan["segments"], plan["groups"], plan["cta_offsets"]
    T = layout.page_size
    unit = 128 // T
    assert info["cluster_ctas"] == 2
    assert info["num_ctas"] == 2 * len(groups) == len(segs)
    assert info["num_pieces"] == 0 and info["merge_rows"] == 0 and info["merge_in_kernel"] == 0
    np.testing.assert_array_equal(offs, np.arange(len(segs) + 1))
    for gi, g in enumerate(groups):
        pages = -(-int(lengths[g[0]]) // T)
        cut = min(pages, (-(-pages // unit) + 1) // 2 * unit)
        assert tuple(segs[2 * gi]) == (gi, 0, cut, -1)
        assert tuple(segs[2 * gi + 1]) == (gi, cut, pages, -1)
        assert g[5] == -1 and g[6] == 2


# ---------------------------------------------------------------- planner (no GPU)
def test_config_3b_is_a_pair_plan():
    w = workload.CONFIGS["c3b"]()
    plan = _inspect(w.layout, w.table, w.lengths, split_tokens=w.split_tokens, num_ctas=None)
    assert plan["info"]["engine"] == 1
    _check_pairs(w.layout, w.lengths, plan)
    assert plan["info"]["num_ctas"] == 128
    # two CTAs of 32 pages each per sequence of 64 pages
    assert {(int(s[1]), int(s[2])) for s in plan["segments"]} == {(0, 32), (32, 64)}


def test_pair_plans_only_where_chosen():
    w = workload.CONFIGS["c3b"]()
    args = (w.layout, w.table, w.lengths)
    # an explicit CTA count, PD_PAIR=0, the warp-level kernel, FP32: one CTA per SM
    assert _inspect(*args, num_ctas=148)["info"]["cluster_ctas"] == 1
    assert _inspect(*args, num_ctas=None, pair="0")["info"]["cluster_ctas"] == 1
    assert _inspect(*args, num_ctas=None, engine="warp")["info"]["cluster_ctas"] == 1
    assert _inspect(*args, num_ctas=None, dtype="float32")["info"]["cluster_ctas"] == 1
    # too few groups to fill 3/4 of the SMs two CTAs each: not by default, forced with PD_PAIR=1
    few = _uniform(40, 32, 1, 128, 32, 2048)
    assert _inspect(*few, num_ctas=None)["info"]["cluster_ctas"] == 1
    _check_pairs(few[0], few[2], _inspect(*few, num_ctas=None, pair="1"))
    # more groups than half the SMs: never
    many = _uniform(75, 32, 1, 128, 32, 256)
    assert _inspect(*many, num_ctas=None, pair="1")["info"]["cluster_ctas"] == 1
    # groups of unequal length: not by default
    layout, table, lengths = _uniform(64, 32, 1, 128, 32, 2048)
    lengths[::2] = 1024
    assert _inspect(layout, table, lengths, num_ctas=None)["info"]["cluster_ctas"] == 1
    _check_pairs(layout, lengths, _inspect(layout, table, lengths, num_ctas=None, pair="1"))


@pytest.mark.parametrize("dim,page", [(128, 32), (64, 16)])
def test_pair_work_list_covers_every_page_once(dim, page):
    rng = np.random.default_rng(dim + page)
    lengths = np.array([0, 1, page, 127, 128, 129, 4 * 128 + 5, 2048, 3000, 17], dtype=np.int32)
    width = -(-int(lengths.max()) // page)
    layout = Layout(len(lengths), 64, 2, dim, page, len(lengths) * width)
    table = rng.permutation(len(lengths) * width).reshape(len(lengths), width).astype(np.int32)
    plan = _inspect(layout, table, lengths, num_ctas=None, pair="1", engine="tcgen05")
    _check_pairs(layout, lengths, plan)
    seen = {}
    for s in plan["segments"]:
        b = int(plan["groups"][s[0]][0])
        for p in range(int(s[1]), int(s[2])):
            seen[(int(s[0]), p)] = seen.get((int(s[0]), p), 0) + 1
    expected = {(gi, p) for gi, g in enumerate(plan["groups"]) for p in range(-(-int(lengths[g[0]]) // page))}
    assert set(seen) == expected and set(seen.values()) <= {1}


# ---------------------------------------------------------------- GPU parity
def _torch():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("NVIDIA GPU required")
    return torch


def _oracle(q, k, v, table, lengths):
    from oracle.paged_oracle import dense_attention
    return dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)


TOL = dict(atol=2e-3, rtol=1e-3)   # the FP16 tolerance of the reference's benchmark checks


def _plan(layout, table, lengths, pair="1", engine="tcgen05", **kw):
    from paged_decode.runtime import DecodePlan
    return _with_env(lambda: DecodePlan(layout, table, lengths, **kw), PD_PAIR=pair, PD_MQA_ENGINE=engine)


def _stats_run(plan, q, k, v):
    torch = _torch()
    L = plan.layout
    out = torch.full((L.batch, L.query_heads, L.head_dim), float("nan"), device=q.device)
    stats = torch.full((L.batch, L.query_heads, 2), float("nan"), device=q.device)
    plan.run_with_stats(q, k, v, out, stats)
    return out, stats


@pytest.mark.gpu
@pytest.mark.parametrize("dim,page", [(128, 32), (64, 16), (128, 16), (64, 32)])
@pytest.mark.parametrize("heads,kv_heads", [(32, 1), (17, 1), (64, 2)])
def test_pair_plan_matches_oracle(dim, page, heads, kv_heads):
    torch = _torch()
    from paged_decode.workload import make_tensors
    lengths = [0, 1, page - 1, page + 1, 127, 128, 129, 4 * page + 3, 9 * page, 700, 2100, 2048]
    rng = np.random.default_rng(dim + heads + page)
    width = -(-max(lengths) // page)
    layout = Layout(len(lengths), heads, kv_heads, dim, page, len(lengths) * width)
    table = rng.permutation(len(lengths) * width).reshape(len(lengths), width).astype(np.int32)
    lengths = np.asarray(lengths, dtype=np.int32)
    for b, n in enumerate(lengths):
        table[b, -(-int(n) // page):] = -1
    q, k, v = make_tensors(layout, seed=heads + page)
    expected = _oracle(q, k, v, table, lengths)
    plan = _plan(layout, table, lengths)
    assert plan.info.engine == 1 and plan.info.cluster_ctas == 2
    out, stats = _stats_run(plan, q, k, v)
    assert plan.read_errors() == 0
    np.testing.assert_allclose(out.cpu().numpy(), expected, **TOL)
    # the same (m, l) as the one-CTA-per-SM plan, and the same rows within tolerance
    single = _plan(layout, table, lengths, pair="0")
    assert single.info.cluster_ctas == 1
    out1, stats1 = _stats_run(single, q, k, v)
    torch.testing.assert_close(out, out1, atol=2e-3, rtol=1e-3)
    live = torch.as_tensor(lengths > 0, device=q.device)
    torch.testing.assert_close(stats[live, :, 0], stats1[live, :, 0], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(stats[live, :, 1], stats1[live, :, 1], atol=1e-3, rtol=1e-3)
    assert torch.equal(stats[~live], stats1[~live])
    # run to run: the same bits
    again, _ = _stats_run(plan, q, k, v)
    assert torch.equal(out, again)


@pytest.mark.gpu
def test_pair_plan_ignores_nan_past_the_sequence_end():
    torch = _torch()
    from paged_decode.workload import make_tensors
    page = 32
    lengths = np.array([40, 2047, 1000, 129] * 16, dtype=np.int32)
    layout, table, _ = _uniform(len(lengths), 32, 1, 128, page, 2048, seed=9)
    q, k, v = make_tensors(layout, seed=11)
    # every token slot past a sequence's end in its last page holds NaN
    for b, n in enumerate(lengths):
        if n % page:
            pid = int(table[b, n // page])
            k[pid, n % page:] = float("nan")
            v[pid, n % page:] = float("nan")
    expected = _oracle(q, k, v, table, lengths)
    plan = _plan(layout, table, lengths)
    assert plan.info.cluster_ctas == 2
    out = plan.run(q, k, v).cpu().numpy()
    assert np.isfinite(out).all() and plan.read_errors() == 0
    np.testing.assert_allclose(out, expected, **TOL)


@pytest.mark.gpu
def test_config_3b_pair_plan_by_default_and_in_a_cuda_graph():
    torch = _torch()
    w = workload.CONFIGS["c3b"]()
    q, k, v = w.tensors("cuda")
    plan = _plan(w.layout, w.table, w.lengths, pair=None, engine=None, split_tokens=w.split_tokens)
    assert plan.info.cluster_ctas == 2 and plan.num_ctas == 128
    ref = plan.run(q, k, v).clone()
    assert plan.read_errors() == 0
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(3):
            out = plan.run(q, k, v)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    del g
    # against the oracle on a slice of the batch (the whole of it is the config test's)
    rows = slice(0, 8)
    expected = _oracle(q[rows], k, v, w.table[rows], w.lengths[rows])
    np.testing.assert_allclose(ref[rows].cpu().numpy(), expected, **TOL)


@pytest.mark.gpu
def test_dynamic_pair_plan_follows_live_lengths():
    torch = _torch()
    from paged_decode.runtime import DecodePlan
    from paged_decode.workload import make_tensors
    layout, table, cap = _uniform(64, 32, 1, 128, 32, 1024, seed=13)
    q, k, v = make_tensors(layout, seed=14)
    start = np.full(64, 1, dtype=np.int32)
    plan = _with_env(lambda: DecodePlan(layout, table, start, max_lengths=cap), PD_PAIR="1",
                     PD_MQA_ENGINE=None)
    assert plan.info.cluster_ctas == 2 and plan.info.dynamic == 1
    dev_table = torch.as_tensor(table, device=q.device)
    for live in (1, 200, 513, 1024):
        lengths = np.full(64, live, dtype=np.int32)
        lengths[::3] = max(1, live // 2)
        out = plan.run_dynamic(q, k, v, dev_table, torch.as_tensor(lengths, device=q.device))
        np.testing.assert_allclose(out.cpu().numpy(), _oracle(q, k, v, table, lengths), **TOL)
    assert plan.read_errors() == 0


@pytest.mark.gpu
def test_exchange_rejects_pair_plans():
    torch = _torch()
    from paged_decode import _native
    from paged_decode.workload import make_tensors
    layout, table, lengths = _uniform(64, 32, 1, 128, 32, 256, seed=15)
    q, k, v = make_tensors(layout, seed=16)
    plan = _plan(layout, table, lengths)
    assert plan.info.cluster_ctas == 2
    lib = _native.load()
    buf = torch.empty(1 << 20, dtype=torch.uint8, device=q.device)
    ptrs = (ctypes.c_void_p * 1)(buf.data_ptr())
    out = torch.empty((64, 32, 128), device=q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    status = lib.pd_decode_exchange(plan._native[_native.PD_FLOAT16].handle, q.data_ptr(), k.data_ptr(),
                                    v.data_ptr(), _native.PD_FLOAT16, ptrs, 0, 1, out.data_ptr(), None, stream)
    assert status == _native.PD_ERR_VALUE
    assert b"CTA pairs" in lib.pd_last_error()


@pytest.mark.gpu
def test_gather_on_a_pair_plan_is_bit_exact_and_decode_repeats():
    # the gather debug mode walks a pair plan's two segments per group on the
    # warp-level kernel (no cluster); decodes before and after it (the K tensor
    # map switches between the page view and the token-group view) agree bit for bit
    torch = _torch()
    from oracle.paged_oracle import gather_cache
    from paged_decode.workload import make_tensors
    layout, table, lengths = _uniform(64, 32, 1, 128, 32, 200, seed=17)
    q, k, v = make_tensors(layout, seed=18)
    plan = _plan(layout, table, lengths, pair=None, engine=None)
    assert plan.info.cluster_ctas == 2
    before = plan.run(q, k, v).clone()
    dense_k, dense_v = plan.gather(k, v)
    after = plan.run(q, k, v)
    assert torch.equal(before, after)
    dk, dv = dense_k.cpu().numpy(), dense_v.cpu().numpy()
    kc, vc = k.cpu().numpy(), v.cpu().numpy()
    for b in range(layout.batch):
        n = int(lengths[b])
        np.testing.assert_array_equal(dk[b, 0, :n].astype(np.float64), gather_cache(kc, table[b], n, 0))
        np.testing.assert_array_equal(dv[b, 0, :n].astype(np.float64), gather_cache(vc, table[b], n, 0))
    assert plan.read_errors() == 0


@pytest.mark.gpu
def test_pair_plans_only_where_all_clusters_fit_at_once():
    # as many groups as half the SMs: a pair plan only if the device holds that
    # many clusters of two CTAs at once (otherwise a cluster would wait for a
    # second wave), else one CTA per SM; the output is right either way
    torch = _torch()
    from paged_decode.workload import make_tensors
    groups = torch.cuda.get_device_properties(0).multi_processor_count // 2
    layout, table, lengths = _uniform(groups, 32, 1, 128, 32, 512, seed=19)
    q, k, v = make_tensors(layout, seed=20)
    plan = _plan(layout, table, lengths, pair="1", engine=None)
    print(f"{groups} groups: cluster_ctas {plan.info.cluster_ctas}, num_ctas {plan.num_ctas}")
    if plan.info.cluster_ctas == 2:
        assert plan.num_ctas == 2 * groups
    out = plan.run(q, k, v).cpu().numpy()
    np.testing.assert_allclose(out, _oracle(q, k, v, table, lengths), **TOL)
    assert plan.read_errors() == 0
    # config 3b's 64 groups stay a pair plan
    layout, table, lengths = _uniform(64, 32, 1, 128, 32, 512, seed=21)
    assert _plan(layout, table, lengths, pair=None, engine=None).info.cluster_ctas == 2
