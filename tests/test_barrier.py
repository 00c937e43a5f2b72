"""The grid barrier before the in-kernel merge, in its three launch modes.

"plain" (the default) launches the decode without the cooperative attribute,
so that it starts on SMs as the previous kernel leaves them; a CTA that waits
at the barrier while another CTA of the launch has not started leaves, and the
CTA that completes the barrier merges the rows of those that left.
"cooperative" is the launch that guarantees residency.  "leave_at_once" makes
every CTA that has to wait leave, so the fallback merge runs on every launch.
All three must give the same bits as each other, and match the FP64 oracle.
"""
import ctypes
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("NVIDIA GPU required", allow_module_level=True)

from oracle.paged_oracle import dense_attention
from paged_decode import _native, workload
from paged_decode.layout import Layout
from paged_decode.runtime import DecodePlan
from paged_decode.workload import make_tensors

pytestmark = pytest.mark.gpu


def _case(batch, heads, kv_heads, dim, page, lengths, seed):
    rng = np.random.default_rng(seed)
    width = max(1, -(-max(lengths) // page))
    pages = batch * width
    layout = Layout(batch, heads, kv_heads, dim, page, pages)
    table = rng.permutation(pages).reshape(batch, width).astype(np.int32)
    lengths = np.asarray(lengths, dtype=np.int32)
    for b, n in enumerate(lengths):
        table[b, -(-int(n) // page):] = -1
    return layout, table, lengths


CASES = {
    # many merge rows: whole rows per warp
    "f16_d128_rows": (torch.float16, (3, 32, 8, 128, 16, [5, 3000, 6000], 1)),
    "f32_d64_rows": (torch.float32, (4, 8, 8, 64, 16, [2000, 1, 4100, 900], 2)),
    # 32 merge rows over every SM: teams of warps share a row
    "f16_d128_teams": (torch.float16, (1, 32, 8, 128, 16, [8000], 3)),
    "f32_d128_teams": (torch.float32, (1, 16, 4, 128, 32, [5000], 4)),
}


def _modes(plan, q, k, v, dtype):
    """Output and stats of 3 launches per mode, and the fallback count of each mode."""
    out = torch.empty((plan.layout.batch, plan.layout.query_heads, plan.layout.head_dim), device=q.device)
    stats = torch.empty((plan.layout.batch, plan.layout.query_heads, 2), device=q.device)
    results = {}
    for mode in ("cooperative", "plain", "leave_at_once", "plain"):
        plan.set_barrier(mode)
        runs = []
        for _ in range(3):
            plan.run_with_stats(q, k, v, out, stats)
            runs.append((out.clone(), stats.clone()))
        results.setdefault(mode, []).extend(runs)
        results[mode + "_fallbacks"] = results.get(mode + "_fallbacks", 0) + plan.read_barrier_fallbacks()
        assert plan.read_errors() == 0
    return results


@pytest.mark.parametrize("name", sorted(CASES))
def test_barrier_modes_give_identical_bits(name):
    dtype, args = CASES[name]
    layout, table, lengths = _case(*args)
    q, k, v = make_tensors(layout, dtype=dtype, seed=args[-1])
    plan = DecodePlan(layout, table, lengths)
    info = plan.native_info(dtype)
    assert info.merge_in_kernel == 1 and info.merge_rows > 0
    res = _modes(plan, q, k, v, dtype)
    ref_out, ref_stats = res["cooperative"][0]
    for mode in ("cooperative", "plain", "leave_at_once"):
        for out, stats in res[mode]:
            assert torch.equal(out, ref_out), mode
            assert torch.equal(stats, ref_stats), mode
    assert res["cooperative_fallbacks"] == 0
    assert res["plain_fallbacks"] == 0           # every CTA resident on an idle GPU: nobody leaves
    assert res["leave_at_once_fallbacks"] >= 1   # CTAs left and the last one merged for them
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    expected = dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)
    np.testing.assert_allclose(ref_out.cpu().numpy(), expected, **tol)


def test_barrier_fallback_on_config2_and_in_a_cuda_graph():
    """BASELINE config 2 (ragged, shared prefix): the fallback merge of every
    launch, replayed in a CUDA graph, repeats the cooperative launch's bits, and
    a plain launch after it finds the barrier's counters consistent."""
    w = workload.CONFIGS["c2"]()
    q, k, v = w.tensors("cuda")
    plan = DecodePlan(w.layout, w.table, w.lengths, split_tokens=w.split_tokens)
    assert plan.native_info(q.dtype).merge_in_kernel == 1
    plan.set_barrier("cooperative")
    ref = plan.run(q, k, v).clone()
    plan.set_barrier("leave_at_once")
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        plan.run(q, k, v)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out = plan.run(q, k, v)
        for _ in range(10):
            graph.replay()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert plan.read_barrier_fallbacks() >= 1
    del graph
    plan.set_barrier("plain")
    for _ in range(5):
        assert torch.equal(plan.run(q, k, v), ref)
    assert plan.read_barrier_fallbacks() == 0
    assert plan.read_errors() == 0


def test_set_barrier_rejects_unknown_modes():
    layout, table, lengths = _case(*CASES["f16_d128_rows"][1])
    plan = DecodePlan(layout, table, lengths)
    with pytest.raises(ValueError):
        plan.set_barrier("spin")
    lib = _native.load()
    handle = next(iter(plan._native.values())).handle
    assert lib.pd_plan_set_barrier(handle, 7) == _native.PD_ERR_VALUE


def test_barrier_leaves_only_when_a_cta_has_not_started():
    """One CTA at a barrier for two: with the partner never started it leaves
    (recording the leave in the count's high bits and its bit), with the partner
    started but never arriving it stays and times out -- an error, not a hang."""
    lib = _native.load()
    outcomes = (ctypes.c_uint32 * 4)()
    start = time.time()
    assert lib.pd_selftest_barrier_leave(torch.cuda.current_device(), 200, outcomes) == 0
    assert list(outcomes) == [2, 1, 1, 3]
    assert time.time() - start < 10


def test_two_plans_on_two_streams_share_the_gpu():
    """Two one-kernel plans launched on two streams at once compete for SMs, so
    neither grid can count on being resident (a CTA waiting for one of its own
    launch that has not started would leave).  However the hardware interleaves
    them, every launch of both gives the bits each gives alone."""
    la, ta, na = _case(4, 32, 8, 128, 16, [3000, 500, 8000, 1200], 11)
    lb, tb, nb = _case(3, 32, 8, 128, 16, [6000, 40, 2500], 12)
    qa, ka, va = make_tensors(la, dtype=torch.float16, seed=11)
    qb, kb, vb = make_tensors(lb, dtype=torch.float16, seed=12)
    pa, pb = DecodePlan(la, ta, na), DecodePlan(lb, tb, nb)
    assert pa.native_info(torch.float16).merge_in_kernel == 1 and pb.native_info(torch.float16).merge_in_kernel == 1
    ref_a, ref_b = pa.run(qa, ka, va).clone(), pb.run(qb, kb, vb).clone()
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    outs_a = [torch.empty_like(ref_a) for _ in range(30)]
    outs_b = [torch.empty_like(ref_b) for _ in range(30)]
    torch.cuda.synchronize()
    for i in range(30):
        with torch.cuda.stream(sa):
            pa.run(qa, ka, va, out=outs_a[i])
        with torch.cuda.stream(sb):
            pb.run(qb, kb, vb, out=outs_b[i])
    torch.cuda.synchronize()
    for i in range(30):
        assert torch.equal(outs_a[i], ref_a) and torch.equal(outs_b[i], ref_b), i
    assert pa.read_errors() == 0 and pb.read_errors() == 0
    print("barrier fallbacks under contention:", pa.read_barrier_fallbacks(), pb.read_barrier_fallbacks())
