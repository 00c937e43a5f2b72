"""The tcgen05 decode kernel for wide query groups (FP16, 17..32 query heads per KV head).

FP16 plans whose group tile holds 32 query heads run on the kernel that issues
its QK^T and PV products from single threads into tensor memory
(csrc/pd_decode_mqa.cuh) by default (PD_MQA_ENGINE=warp keeps them on the
warp-level kernel).  The CPU tests pin the planner's choice (engine,
one KV head per page tile, one partial slot per segment).  The GPU tests check
that kernel against the FP64 oracle on the shapes it serves (head_dim 64 and
128, pages of 16 and 32 tokens, groups of 17, 24, 32 and 64 query heads per
KV head), across split and unsplit groups, the in-kernel merge and the merge kernel,
dynamic plans, rows past the sequence end holding NaN, logits whose running
maximum keeps growing (the path that rescales the output block in tensor
memory), (m, l) statistics, run-to-run repeatability, and agreement with the
warp-level kernel on the same inputs.
"""
import os

import numpy as np
import pytest

from paged_decode.layout import Layout
from paged_decode.runtime import inspect_plan

TCGEN05 = 1
LOG2E = 1.4426950408889634


def _fragmented(batch, heads, kv_heads, dim, page, lengths, seed=3):
    rng = np.random.default_rng(seed)
    width = max(1, -(-max(lengths) // page))
    pages = batch * width
    layout = Layout(batch, heads, kv_heads, dim, page, pages)
    table = rng.permutation(pages)[: batch * width].reshape(batch, width).astype(np.int32)
    lengths = np.asarray(lengths, dtype=np.int32)
    for b, n in enumerate(lengths):
        table[b, -(-int(n) // page):] = -1
    return layout, table, lengths


# ---------------------------------------------------------------- planner (no GPU)
@pytest.mark.parametrize("heads,kv_heads,expected", [(32, 1, 1), (24, 1, 1), (40, 2, 1), (64, 1, 1),
                                                     (64, 4, 0), (16, 1, 0), (8, 1, 0), (64, 8, 0)])
@pytest.mark.parametrize("dim,page", [(64, 16), (128, 32)])
def test_fp16_group_tiles_of_32_heads_choose_the_tcgen05_kernel(heads, kv_heads, expected, dim, page, monkeypatch):
    monkeypatch.setenv("PD_MQA_ENGINE", "tcgen05")
    layout, table, lengths = _fragmented(3, heads, kv_heads, dim, page, [0, 70, 900])
    fp16 = inspect_plan(layout, table, lengths, num_ctas=7)["info"]
    fp32 = inspect_plan(layout, table, lengths, num_ctas=7, dtype="float32")["info"]
    assert fp16["engine"] == expected and fp32["engine"] == 0
    if expected:
        # one KV head per page tile, one partial slot per segment
        assert fp16["group_tile"] == 32 and fp16["heads_per_tile"] == 1 and fp16["slot_stride"] == 1


def test_default_engine_and_overrides(monkeypatch):
    """By default the tcgen05 kernel takes every FP16 group tile of 32 query
    heads (head_dim 64 or 128, pages of 16 or 32 tokens: measured faster);
    PD_MQA_ENGINE=warp keeps such plans on the warp-level kernel."""
    monkeypatch.delenv("PD_MQA_ENGINE", raising=False)
    layout, table, lengths = _fragmented(2, 32, 1, 128, 32, [500, 70])
    assert inspect_plan(layout, table, lengths)["info"]["engine"] == TCGEN05
    for dim, page in ((128, 16), (64, 32), (64, 16)):
        small = _fragmented(2, 32, 1, dim, page, [500, 70])
        assert inspect_plan(*small)["info"]["engine"] == TCGEN05
        monkeypatch.setenv("PD_MQA_ENGINE", "warp")
        assert inspect_plan(*small)["info"]["engine"] == 0
        monkeypatch.delenv("PD_MQA_ENGINE")
    monkeypatch.setenv("PD_MQA_ENGINE", "warp")
    info = inspect_plan(layout, table, lengths)["info"]
    # two sub-pipelines of four warps on 16 KiB tiles, one partial slot each
    assert info["engine"] == 0 and info["heads_per_tile"] == 1 and info["slot_stride"] == 2
    layout, table, lengths = _fragmented(2, 64, 2, 128, 32, [500, 70])
    info = inspect_plan(layout, table, lengths)["info"]
    assert info["engine"] == 0 and info["heads_per_tile"] == 2


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


def _plan(layout, table, lengths, engine="tcgen05", **kw):
    from paged_decode.runtime import DecodePlan
    old = os.environ.pop("PD_MQA_ENGINE", None)
    try:
        if engine:
            os.environ["PD_MQA_ENGINE"] = engine
        return DecodePlan(layout, table, lengths, **kw)
    finally:
        os.environ.pop("PD_MQA_ENGINE", None)
        if old is not None:
            os.environ["PD_MQA_ENGINE"] = old


@pytest.mark.gpu
@pytest.mark.parametrize("dim,page", [(64, 16), (64, 32), (128, 16), (128, 32)])
@pytest.mark.parametrize("heads,kv_heads", [(32, 1), (17, 1), (48, 2), (64, 1)])
def test_tcgen05_kernel_matches_oracle(dim, page, heads, kv_heads):
    torch = _torch()
    from paged_decode.workload import make_tensors
    lengths = [0, 1, page - 1, page + 1, 4 * page + 3, 9 * page, 700, 2100]
    layout, table, lengths = _fragmented(len(lengths), heads, kv_heads, dim, page, lengths, seed=dim + heads)
    q, k, v = make_tensors(layout, seed=heads + page)
    expected = _oracle(q, k, v, table, lengths)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for ctas in (1, 5, None, sms + 3):
        plan = _plan(layout, table, lengths, num_ctas=ctas)
        assert plan.info.engine == TCGEN05
        out = plan.run(q, k, v).cpu().numpy()
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, expected, **TOL)
        assert plan.read_errors() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dim,page", [(64, 16), (128, 32)])
def test_tcgen05_kernel_is_repeatable_and_agrees_with_the_warp_kernel(dim, page):
    torch = _torch()
    from paged_decode.workload import make_tensors
    layout, table, lengths = _fragmented(6, 32, 1, dim, page, [0, 5, 333, 1024, 2047, 4100], seed=7)
    q, k, v = make_tensors(layout, seed=8)
    expected = _oracle(q, k, v, table, lengths)
    tc = _plan(layout, table, lengths)
    warp = _plan(layout, table, lengths, engine="warp")
    assert tc.info.engine == TCGEN05 and warp.info.engine == 0
    first = tc.run(q, k, v).clone()
    for _ in range(3):
        assert torch.equal(tc.run(q, k, v), first)   # identical bits every launch
    other = warp.run(q, k, v).clone()
    np.testing.assert_allclose(first.cpu().numpy(), expected, **TOL)
    np.testing.assert_allclose(other.cpu().numpy(), expected, **TOL)
    np.testing.assert_allclose(first.cpu().numpy(), other.cpu().numpy(), atol=1e-3, rtol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("dim,page", [(64, 16), (128, 32)])
def test_rows_past_the_end_hold_nan_and_inf(dim, page):
    torch = _torch()
    from paged_decode.workload import make_tensors
    lengths = [page * 3 + 5, page - 1, 7 * page + 1, 1, 0]
    layout, table, lengths = _fragmented(len(lengths), 32, 1, dim, page, lengths, seed=dim)
    q, k, v = make_tensors(layout, seed=13)
    expected = _oracle(q, k, v, table, lengths)
    live = torch.zeros((layout.physical_pages, page), dtype=torch.bool)
    for b, n in enumerate(lengths):
        for t in range(int(n)):
            live[int(table[b, t // page]), t % page] = True
    dead = ~live.to(k.device)
    k[dead] = float("nan")
    v[dead] = float("nan")
    for ctas in (1, 3, None):
        plan = _plan(layout, table, lengths, num_ctas=ctas)
        assert plan.info.engine == TCGEN05
        out = plan.run(q, k, v).cpu().numpy()
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, expected, **TOL)


@pytest.mark.gpu
def test_growing_logits_rescale_the_output_block():
    """Scores that rise along each sequence (slopes of 1/3, 1/10 and 1/40 in
    log2 units per token) push the running maximum past the weights'
    reference by more than 2^8 every step, or every few steps, so the output
    block in tensor memory is rescaled between steps."""
    torch = _torch()
    from paged_decode.workload import make_tensors
    page = 32
    lengths = [4000, 1500, 2600]
    slopes = [1 / 3, 1 / 10, 1 / 40]
    layout, table, lengths = _fragmented(3, 32, 1, 128, page, lengths, seed=2)
    q, k, v = make_tensors(layout, seed=3)
    # q ~ e0 (+ a little noise), K[t] . e0 = t * slope * sqrt(D) / log2(e): s(t) ~ t * slope
    q.mul_(0.02)
    q[:, :, 0] = 1.0
    unit = float(np.sqrt(128) / LOG2E)
    for b, n in enumerate(lengths):
        pages = torch.as_tensor(table[b, : -(-int(n) // page)].astype(np.int64), device=k.device)
        tok = torch.arange(pages.numel() * page, device=k.device, dtype=torch.float32)
        k[pages, :, 0, 0] = (tok * slopes[b] * unit).view(-1, page).to(k.dtype)
    expected = _oracle(q, k, v, table, lengths)
    for ctas in (1, None):
        plan = _plan(layout, table, lengths, num_ctas=ctas)
        assert plan.info.engine == TCGEN05
        out = plan.run(q, k, v).cpu().numpy()
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, expected, **TOL)


@pytest.mark.gpu
def test_statistics_are_true_maximum_and_denominator():
    torch = _torch()
    from oracle.paged_oracle import gather_cache
    from paged_decode.workload import make_tensors
    layout, table, lengths = _fragmented(3, 32, 1, 128, 16, [0, 50, 1333], seed=4)
    q, k, v = make_tensors(layout, seed=4)
    plan = _plan(layout, table, lengths, num_ctas=3)
    assert plan.info.engine == TCGEN05
    out = torch.empty((3, 32, 128), device=q.device)
    stats = torch.empty((3, 32, 2), device=q.device)
    plan.run_with_stats(q, k, v, out, stats)
    st = stats.cpu().numpy()
    qn, kn = q.cpu().numpy().astype(np.float64), k.cpu().numpy()
    for b in range(3):
        n = int(lengths[b])
        for h in range(32):
            if n == 0:
                assert st[b, h, 0] == -np.inf and st[b, h, 1] == 0
                continue
            s = gather_cache(kn, table[b], n, 0) @ qn[b, h] / np.sqrt(128) * LOG2E
            np.testing.assert_allclose(st[b, h, 0], s.max(), rtol=1e-4, atol=1e-4)
            np.testing.assert_allclose(st[b, h, 1], np.exp2(s - st[b, h, 0]).sum(), rtol=2e-3)


@pytest.mark.gpu
def test_dynamic_plan_on_the_tcgen05_kernel():
    torch = _torch()
    from paged_decode.workload import make_tensors
    layout, table, lengths = _fragmented(4, 32, 1, 128, 32, [900, 40, 3000, 0], seed=9)
    full = table.copy()
    cap = np.array([900, 40, 3000, 0], dtype=np.int32)
    live = np.array([640, 33, 2999, 0], dtype=np.int32)
    q, k, v = make_tensors(layout, seed=10)
    plan = _plan(layout, full, live, max_lengths=cap)
    assert plan.info.engine == TCGEN05 and plan.info.dynamic == 1
    dev_table = torch.as_tensor(full, device=q.device)
    for step in range(3):
        now = np.minimum(live + 97 * step, cap).astype(np.int32)
        out = plan.run_dynamic(q, k, v, dev_table, torch.as_tensor(now, device=q.device)).cpu().numpy()
        np.testing.assert_allclose(out, _oracle(q, k, v, full, now), **TOL)
    assert plan.read_errors() == 0
