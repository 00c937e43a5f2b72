"""GPU parity tests: the sm_100a kernel against the FP64 oracle on the same tensors.

The first block ports the reference's own acceptance tests
(ensigncode/paged-decode-lab tests/test_cuda.py:16-149) unchanged in substance:
same shapes, seeds, split sizes and tolerances (atol = rtol = 5e-4, 3e-3 for
large logits).  The second block adds what this implementation needs proven:
the TMA page gather is bit-exact, results do not depend on how pages are
balanced over CTAs and repeat bit for bit across launches, the (m, l)
statistics and cross-shard merge used by sequence sharding, wide query
groups, a randomized stress set, and agreement with the reference's own
kernel built for sm_100a.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("NVIDIA GPU required", allow_module_level=True)

from oracle.paged_oracle import dense_attention, gather_cache
from paged_decode import _native
from paged_decode.layout import Layout
from paged_decode.runtime import DecodePlan
from paged_decode.workload import make_metadata, make_tensors

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634


def oracle(q, k, v, table, lengths):
    return dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)


# ---------------------------------------------------------------- reference acceptance tests
@pytest.mark.parametrize("merge", ["serial", "shared"])
@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("page_size", [16, 32])
@pytest.mark.parametrize("split", [1, 33, 256])
def test_ragged_decode(dim, dtype, page_size, split, merge):
    layout = Layout(4, 8, 2, dim, page_size, 32)
    table = np.random.default_rng(5).permutation(32).reshape(4, 8).astype(np.int32)
    lengths = np.array([0, 1, page_size + 1, 127], dtype=np.int32)
    for b, length in enumerate(lengths):
        table[b, (int(length) + page_size - 1) // page_size:] = -1
    q, k, v = make_tensors(layout, dtype=dtype)
    plan = DecodePlan(layout, table, lengths, split_tokens=split, merge=merge)
    actual = plan.run(q, k, v).cpu().numpy()
    expected = oracle(q, k, v, table, lengths)
    np.testing.assert_allclose(actual, expected, atol=5e-4, rtol=5e-4)
    assert np.isfinite(actual).all()
    assert plan.read_errors() == 0


@pytest.mark.parametrize("merge", ["serial", "shared"])
def test_nondefault_stream_and_graph_capture(merge):
    layout = Layout(1, 8, 2, 64, 16, 8)
    table, lengths = np.arange(8, dtype=np.int32)[None], np.array([127], dtype=np.int32)
    q, k, v = make_tensors(layout)
    plan = DecodePlan(layout, table, lengths, merge=merge)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        expected = plan.run(q, k, v).clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            output = plan.run(q, k, v)
        graph.replay()
        torch.testing.assert_close(output, expected)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()


@pytest.mark.parametrize("merge", ["serial", "shared"])
def test_large_logits_and_repeated_pages(merge):
    layout = Layout(2, 8, 1, 128, 16, 4)
    table = np.array([[2, 0, 1, 3], [2, 0, 1, 3]], dtype=np.int32)
    lengths = np.array([64, 37], dtype=np.int32)
    q, k, v = make_tensors(layout, dtype=torch.float32)
    q *= 100
    plan = DecodePlan(layout, table, lengths, split_tokens=17, merge=merge)
    actual = plan.run(q, k, v).cpu().numpy()
    np.testing.assert_allclose(actual, oracle(q, k, v, table, lengths), atol=3e-3, rtol=3e-3)


def test_rejects_invalid_inputs():
    layout = Layout(1, 8, 2, 64, 16, 8)
    plan = DecodePlan(layout, np.arange(8, dtype=np.int32)[None], np.array([127]))
    q, k, v = make_tensors(layout)
    with pytest.raises(TypeError):
        plan.run(q.double(), k, v)
    with pytest.raises(ValueError):
        plan.run(q.transpose(1, 2), k, v)
    with pytest.raises(ValueError):
        plan.run(q.requires_grad_(), k, v)


@pytest.mark.parametrize("merge", ["serial", "shared"])
def test_all_empty_contexts_and_long_partition_tail(merge):
    for lengths in (np.array([0, 0], dtype=np.int32), np.array([8193, 17], dtype=np.int32)):
        layout = Layout(2, 4, 4, 64, 16, 1026)
        table = np.arange(1026, dtype=np.int32).reshape(2, 513)
        q, k, v = make_tensors(layout, dtype=torch.float32)
        plan = DecodePlan(layout, table, lengths, split_tokens=257, merge=merge)
        actual = plan.run(q, k, v).cpu().numpy()
        np.testing.assert_allclose(actual, oracle(q, k, v, table, lengths), atol=5e-4, rtol=5e-4)


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("merge", ["serial", "shared"])
def test_randomized_layout_and_content(seed, merge):
    rng = np.random.default_rng(seed)
    dim, page = int(rng.choice([64, 128])), int(rng.choice([16, 32]))
    heads = int(rng.choice([1, 4, 8]))
    kv_heads = int(rng.choice([h for h in [1, 2, 4, 8] if heads % h == 0]))
    layout = Layout(3, heads, kv_heads, dim, page, 20)
    lengths = np.array([0, int(rng.integers(1, 64)), 257], dtype=np.int32)
    table = rng.integers(0, 20, size=(3, (257 + page - 1) // page), dtype=np.int32)
    dtype = torch.float16 if seed % 2 else torch.float32
    q, k, v = make_tensors(layout, dtype=dtype, seed=seed + 200)
    if seed % 3 == 0:
        q.zero_()  # uniform attention reduces to a mean over logical tokens
    plan = DecodePlan(layout, table, lengths, split_tokens=int(rng.choice([1, 31, 128, 511])), merge=merge)
    actual = plan.run(q, k, v).cpu().numpy()
    np.testing.assert_allclose(actual, oracle(q, k, v, table, lengths), atol=5e-4, rtol=5e-4)


@pytest.mark.parametrize("merge", ["serial", "shared"])
def test_changing_decode_across_page_boundaries(merge):
    layout = Layout(1, 4, 2, 64, 16, 4)
    table = np.array([[2, 0, 3, 1]], dtype=np.int32)
    q, k, v = make_tensors(layout, dtype=torch.float32, seed=333)
    for length in [0, 1, 15, 16, 17, 31, 32, 33, 63, 64]:
        q.add_(0.01)
        if length:
            page = int(table[0, (length - 1) // 16])
            v[page, (length - 1) % 16].mul_(0.9)
        plan = DecodePlan(layout, table, np.array([length]), split_tokens=13, merge=merge)
        actual = plan.run(q, k, v).cpu().numpy()
        np.testing.assert_allclose(actual, oracle(q, k, v, table, [length]), atol=5e-4, rtol=5e-4)


def test_shared_merge_resource_bound_uses_explicit_fallback():
    layout = Layout(1, 4, 1, 64, 16, 70)
    table = np.arange(70, dtype=np.int32)[None]
    lengths = np.array([1100], dtype=np.int32)
    q, k, v = make_tensors(layout, dtype=torch.float32)
    plan = DecodePlan(layout, table, lengths, split_tokens=1, merge="shared")
    assert plan.merge_implementation == "serial_fallback"
    np.testing.assert_allclose(plan.run(q, k, v).cpu().numpy(), oracle(q, k, v, table, lengths),
                               atol=5e-4, rtol=5e-4)


def test_rejects_same_shape_noncontiguous_and_wrong_device():
    layout = Layout(1, 8, 2, 64, 16, 8)
    plan = DecodePlan(layout, np.arange(8, dtype=np.int32)[None], np.array([127]))
    q, k, v = make_tensors(layout)
    strided = torch.empty((1, 8, 128), device=q.device, dtype=q.dtype)[..., ::2]
    assert strided.shape == q.shape and not strided.is_contiguous()
    with pytest.raises(ValueError):
        plan.run(strided, k, v)
    with pytest.raises(ValueError):
        plan.run(q.cpu(), k, v)


# ---------------------------------------------------------------- B200 implementation checks
def _fragmented(batch, heads, kv_heads, dim, page, lengths, pages=None, seed=3):
    rng = np.random.default_rng(seed)
    width = max(1, -(-max(lengths) // page))
    pages = pages or batch * width
    layout = Layout(batch, heads, kv_heads, dim, page, pages)
    table = rng.integers(0, pages, size=(batch, width)).astype(np.int32)
    lengths = np.asarray(lengths, dtype=np.int32)
    for b, n in enumerate(lengths):
        table[b, -(-int(n) // page):] = -1
    return layout, table, lengths


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("dim,page", [(64, 16), (128, 16), (64, 32), (128, 32)])
def test_tma_gather_is_bit_exact(dtype, dim, page):
    layout, table, lengths = _fragmented(3, 8, 4, dim, page, [0, page * 3 + 5, 200], seed=dim + page)
    q, k, v = make_tensors(layout, dtype=dtype, seed=9)
    plan = DecodePlan(layout, table, lengths, num_ctas=5)
    dense_k, dense_v = plan.gather(k, v)
    dk, dv = dense_k.cpu().numpy(), dense_v.cpu().numpy()
    kc, vc = k.cpu().numpy(), v.cpu().numpy()
    for b in range(3):
        n = int(lengths[b])
        for h in range(layout.kv_heads):
            np.testing.assert_array_equal(dk[b, h, :n].astype(np.float64), gather_cache(kc, table[b], n, h))
            np.testing.assert_array_equal(dv[b, h, :n].astype(np.float64), gather_cache(vc, table[b], n, h))
            assert not dk[b, h, n:].any() and not dv[b, h, n:].any()
    assert plan.read_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("dim,page,heads,kv_heads", [(64, 16, 8, 4), (128, 16, 8, 4), (64, 32, 32, 32),
                                                     (128, 32, 32, 1), (128, 16, 64, 8)])
def test_rows_past_each_sequence_end_are_never_read(dtype, dim, page, heads, kv_heads):
    # The reference reads only live tokens (decode.cu loops to the length), so
    # whatever sits in the rest of a sequence's last page, or in a page no
    # sequence uses, must not reach the output: fill all of it with NaN and inf.
    lengths = [0, page * 3 + 5, page - 1, 7 * page + 1, 1]
    layout, table, lengths = _fragmented(len(lengths), heads, kv_heads, dim, page, lengths, seed=dim + heads)
    q, k, v = make_tensors(layout, dtype=dtype, seed=13)
    expected = oracle(q, k, v, table, lengths)
    live = torch.zeros((layout.physical_pages, page), dtype=torch.bool)
    for b, n in enumerate(lengths):
        for t in range(int(n)):
            live[int(table[b, t // page]), t % page] = True
    dead = ~live.to(k.device)
    k[dead] = float("nan")
    v[dead] = float("inf")
    v[dead & dead[:, :1]] = float("nan")        # pages no sequence reads: NaN
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    for ctas in (1, 3, None):
        plan = DecodePlan(layout, table, lengths, num_ctas=ctas)
        out = plan.run(q, k, v).cpu().numpy()
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, expected, **tol)
        assert plan.read_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_result_independent_of_cta_balance_and_repeatable(dtype):
    layout, table, lengths = _fragmented(4, 16, 4, 128, 16, [0, 33, 400, 1000], seed=21)
    q, k, v = make_tensors(layout, dtype=dtype, seed=5)
    expected = oracle(q, k, v, table, lengths)
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    for ctas in (1, 2, 5, 37, 148, 1000):
        plan = DecodePlan(layout, table, lengths, num_ctas=ctas)
        first = plan.run(q, k, v).clone()
        for _ in range(3):   # deterministic: identical bits every launch
            again = plan.run(q, k, v)
            assert torch.equal(first, again)
        np.testing.assert_allclose(first.cpu().numpy(), expected, **tol)
        assert plan.read_errors() == 0


def _sm_count():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("dtype,dim,heads,kv_heads,page", [
    (torch.float16, 128, 32, 8, 16), (torch.float16, 64, 16, 2, 32), (torch.float32, 64, 8, 8, 16),
    (torch.float32, 128, 16, 4, 32), (torch.float16, 128, 32, 1, 32)])
def test_in_kernel_merge_and_merge_kernel_agree(dtype, dim, heads, kv_heads, page):
    """num_ctas <= SMs merges the partials inside the decode kernel (one launch);
    more CTAs than SMs use the dependent merge kernel.  Both match the oracle,
    and their (m, l) statistics agree."""
    layout, table, lengths = _fragmented(3, heads, kv_heads, dim, page, [5, 3000, 6000], seed=dim + heads)
    q, k, v = make_tensors(layout, dtype=dtype, seed=4)
    expected = oracle(q, k, v, table, lengths)
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    stats_by_path = []
    for ctas, fused in ((None, 1), (_sm_count() + 3, 0)):
        plan = DecodePlan(layout, table, lengths, num_ctas=ctas)
        info = plan.native_info(dtype)
        assert plan.num_ctas == (ctas or _sm_count())   # more page tiles than CTAs
        assert info.merge_rows > 0 and info.merge_in_kernel == fused
        assert plan.kernels_per_run(dtype) == 2 - fused
        out = torch.empty((3, heads, dim), device=q.device)
        stats = torch.empty((3, heads, 2), device=q.device)
        plan.run_with_stats(q, k, v, out, stats)
        np.testing.assert_allclose(out.cpu().numpy(), expected, **tol)
        torch.testing.assert_close(out, plan.run(q, k, v), rtol=0, atol=0)
        assert plan.read_errors() == 0
        stats_by_path.append(stats)
    torch.testing.assert_close(stats_by_path[0], stats_by_path[1], rtol=1e-5, atol=1e-5)


def test_in_kernel_merge_graph_replay_and_interleaved_plans():
    """Each plan keeps its own grid-barrier count: interleaved launches of two
    plans and CUDA-graph replays repeat the first result bit for bit."""
    layout, table, lengths = _fragmented(4, 32, 8, 128, 16, [100, 3000, 4096, 17], seed=2)
    q, k, v = make_tensors(layout, seed=8)
    a = DecodePlan(layout, table, lengths)
    b = DecodePlan(layout, table, lengths, num_ctas=37)
    assert a.native_info(q.dtype).merge_in_kernel == 1 and b.native_info(q.dtype).merge_in_kernel == 1
    ra, rb = a.run(q, k, v).clone(), b.run(q, k, v).clone()
    np.testing.assert_allclose(ra.cpu().numpy(), oracle(q, k, v, table, lengths), atol=2e-3, rtol=1e-3)
    for _ in range(60):
        oa = a.run(q, k, v)
        ob = b.run(q, k, v)
    assert torch.equal(oa, ra) and torch.equal(ob, rb)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        a.run(q, k, v)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            og = a.run(q, k, v)
        for _ in range(20):
            graph.replay()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    assert torch.equal(og, ra)
    assert a.read_errors() == 0 and b.read_errors() == 0


def test_plan_from_csr_metadata_matches_the_table_plan():
    """FlashInfer-style CSR metadata (indptr / indices / last_page_len) builds the
    same plan as the page table it came from: identical output bits."""
    from paged_decode.competitors import paged_csr
    layout, table, lengths = _fragmented(4, 32, 8, 128, 16, [1, 700, 4096, 33], seed=6)
    q, k, v = make_tensors(layout, seed=6)
    indptr, indices, last = paged_csr(layout, table, lengths)
    from_csr = DecodePlan.from_csr(layout, indptr, indices, last).run(q, k, v).clone()
    torch.testing.assert_close(from_csr, DecodePlan(layout, table, lengths).run(q, k, v), rtol=0, atol=0)
    np.testing.assert_allclose(from_csr.cpu().numpy(), oracle(q, k, v, table, lengths), atol=2e-3, rtol=1e-3)


def test_bounded_waits_time_out_with_an_error_not_a_hang():
    """An mbarrier phase nobody completes and a grid barrier only one of two CTAs
    reaches: both waits give up after 20 ms, record PD_DEVERR_TIMEOUT, and the
    context stays usable."""
    import ctypes
    import time
    lib = _native.load()
    words = (ctypes.c_uint32 * 2)()
    start = time.time()
    assert lib.pd_selftest_wait_timeouts(torch.cuda.current_device(), 20000, words) == 0
    assert list(words) == [1, 1]
    assert time.time() - start < 10
    layout, table, lengths = _fragmented(2, 8, 2, 128, 16, [40, 300], seed=1)
    q, k, v = make_tensors(layout, seed=1)
    plan = DecodePlan(layout, table, lengths)
    np.testing.assert_allclose(plan.run(q, k, v).cpu().numpy(), oracle(q, k, v, table, lengths),
                               atol=2e-3, rtol=1e-3)
    assert plan.read_errors() == 0


@pytest.mark.parametrize("heads,kv_heads", [(12, 1), (16, 2), (24, 1), (32, 1), (40, 2), (64, 1)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_wide_query_groups(heads, kv_heads, dtype):
    layout, table, lengths = _fragmented(2, heads, kv_heads, 128, 32, [300, 77], seed=heads)
    q, k, v = make_tensors(layout, dtype=dtype, seed=heads)
    plan = DecodePlan(layout, table, lengths, num_ctas=7)
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(plan.run(q, k, v).cpu().numpy(), oracle(q, k, v, table, lengths), **tol)


def test_stats_report_running_max_and_denominator():
    layout, table, lengths = _fragmented(3, 8, 2, 128, 16, [0, 50, 333], seed=4)
    q, k, v = make_tensors(layout, dtype=torch.float32, seed=4)
    plan = DecodePlan(layout, table, lengths, num_ctas=3)
    out = torch.empty((3, 8, 128), device=q.device)
    stats = torch.empty((3, 8, 2), device=q.device)
    plan.run_with_stats(q, k, v, out, stats)
    torch.testing.assert_close(out, plan.run(q, k, v).clone(), rtol=0, atol=0)
    st = stats.cpu().numpy()
    qn, kn = q.cpu().numpy().astype(np.float64), k.cpu().numpy()
    for b in range(3):
        n = int(lengths[b])
        for h in range(8):
            if n == 0:
                assert st[b, h, 0] == -np.inf and st[b, h, 1] == 0
                continue
            s = gather_cache(kn, table[b], n, h // 4) @ qn[b, h] / np.sqrt(128) * LOG2E
            np.testing.assert_allclose(st[b, h, 0], s.max(), rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(st[b, h, 1], np.exp2(s - st[b, h, 0]).sum(), rtol=1e-4)


@pytest.mark.parametrize("shards", [2, 3, 4])
def test_sequence_shards_merge_to_full_attention(shards):
    """Sequence sharding on one GPU: each shard decodes a contiguous page range."""
    layout, table, lengths = _fragmented(2, 32, 8, 128, 32, [4000, 1500], seed=shards)
    q, k, v = make_tensors(layout, seed=shards)
    width = table.shape[1]
    bounds = [width * r // shards for r in range(shards + 1)]
    outs, stats = [], []
    for r in range(shards):
        lo, hi = bounds[r], bounds[r + 1]
        sub_len = np.clip(lengths - lo * 32, 0, (hi - lo) * 32).astype(np.int32)
        sub_tab = table[:, lo:hi].copy()
        plan = DecodePlan(layout, sub_tab, sub_len, num_ctas=11)
        o = torch.empty((2, 32, 128), device=q.device)
        s = torch.empty((2, 32, 2), device=q.device)
        plan.run_with_stats(q, k, v, o, s)
        outs.append(o)
        stats.append(s)
    merged = torch.empty((2, 32, 128), device=q.device)
    lib = _native.load()
    # one packed buffer per shard ([rows * D outputs][rows * 2 stats]), as the all-gather lays it out
    rows = 64
    packed = torch.cat([torch.cat([o.reshape(-1), s.reshape(-1)]) for o, s in zip(outs, stats)])
    _native.check(lib.pd_merge_shards(packed.data_ptr(), packed.data_ptr() + rows * 128 * 4, shards,
                                      rows * 130, rows, 128, merged.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream))
    np.testing.assert_allclose(merged.cpu().numpy(), oracle(q, k, v, table, lengths), atol=2e-3, rtol=1e-3)


def test_randomized_stress_against_oracle():
    """1000 random cases in the style of the reference's 1000-case stress run (seed 97531)."""
    rng = np.random.default_rng(97531)
    worst = 0.0
    for seed in range(1000):
        b = int(rng.choice([1, 2, 3]))
        kv = int(rng.choice([1, 2, 4]))
        h = kv * int(rng.choice([1, 2, 4, 8]))
        d = int(rng.choice([64, 128]))
        page = int(rng.choice([16, 32]))
        length = int(rng.choice([1, 15, 16, 17, 31, 32, 33, 127, 129, 257, 513]))
        layout, table, lengths = make_metadata(b, h, kv, d, length, page, seed=seed)
        if seed % 3 == 0:
            lengths[-1] = 0
            table[-1, :] = -1
        if seed % 5 == 0:
            table[table >= 0] = 0
        dtype = torch.float16 if seed % 2 else torch.float32
        q, k, v = make_tensors(layout, dtype=dtype, seed=seed + 10000)
        if seed % 7 == 0:
            q.mul_(20)
            k.mul_(20)
        ref = oracle(q, k, v, table, lengths)
        plan = DecodePlan(layout, table, lengths, split_tokens=int(rng.choice([1, 7, 31, 128, 256, 511])),
                          num_ctas=int(rng.choice([1, 3, 148])))
        out = plan.run(q, k, v).cpu().numpy()
        worst = max(worst, float(np.abs(out - ref).max()))
        np.testing.assert_allclose(out, ref, atol=3e-3, rtol=3e-3)
    print(f"stress max abs err {worst:.3e}")


def test_reference_kernel_agrees_on_the_same_inputs():
    """The reference's own kernel (built for sm_100a from its sources) as a second opinion."""
    from oracle import ref_kernel
    if not ref_kernel.SO_PATH.exists():
        pytest.skip("reference kernel not built")
    layout, table, lengths = make_metadata(4, 32, 8, 128, 1024, 16, seed=123)
    q, k, v = make_tensors(layout)
    ours = DecodePlan(layout, table, lengths).run(q, k, v).clone()
    theirs = ref_kernel.RefPlan(layout, table, lengths, device=q.device).run(q, k, v)
    torch.testing.assert_close(ours, theirs, atol=2e-3, rtol=1e-3)


# ---------------------------------------------------------------- maximum sizes
def _c_oracle(q, k, v, table, lengths):
    from oracle.c_oracle import dense_attention as c_dense
    return c_dense(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_maximum_context_of_one_million_tokens(dtype):
    """The reference's longest context (2^20 tokens, runtime.py:47) in one
    sequence: 32768 pages of 32 tokens, beside a short and an empty one."""
    page, width = 32, 32768
    lengths = np.array([1 << 20, 77, 0], dtype=np.int32)
    layout = Layout(3, 8, 1, 64, page, width + 3)
    rng = np.random.default_rng(11)
    table = np.full((3, width), -1, dtype=np.int32)
    table[0] = rng.permutation(width + 3)[:width]
    table[1, :3] = rng.choice(width + 3, 3, replace=False)
    q, k, v = make_tensors(layout, dtype=dtype, seed=11)
    plan = DecodePlan(layout, table, lengths)
    assert plan.max_context == 1 << 20
    out = plan.run(q, k, v).cpu().numpy()
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(out, _c_oracle(q, k, v, table, lengths), **tol)
    assert not out[2].any() and plan.read_errors() == 0


def test_maximum_batch_of_65535_sequences():
    """The reference's largest batch (65535, runtime.py:39), ragged lengths, one
    page each at most, pages shared at random."""
    batch = 65535
    rng = np.random.default_rng(12)
    lengths = rng.integers(0, 17, batch).astype(np.int32)
    layout = Layout(batch, 4, 2, 128, 16, 4096)
    table = rng.integers(0, 4096, (batch, 1)).astype(np.int32)
    q, k, v = make_tensors(layout, seed=12)
    plan = DecodePlan(layout, table, lengths)
    out = plan.run(q, k, v).cpu().numpy()
    np.testing.assert_allclose(out, _c_oracle(q, k, v, table, lengths), atol=2e-3, rtol=1e-3)
    assert not out[lengths == 0].any() and plan.read_errors() == 0


def test_run_into_a_caller_buffer():
    """run(..., out=buf) writes the same bits into the caller's buffer and returns it."""
    layout, table, lengths = _fragmented(3, 16, 4, 128, 16, [7, 900, 2500], seed=12)
    q, k, v = make_tensors(layout, seed=12)
    plan = DecodePlan(layout, table, lengths)
    ref = plan.run(q, k, v).clone()
    buf = torch.full_like(ref, float("nan"))
    assert plan.run(q, k, v, out=buf) is buf
    assert torch.equal(buf, ref)
    for bad in (torch.empty_like(ref, dtype=torch.float16), ref[:, :, :64], ref.cpu(),
                torch.empty((3, 16, 256), device=ref.device)[:, :, :128]):
        with pytest.raises(ValueError):
            plan.run(q, k, v, out=bad)
    assert plan.read_errors() == 0
