"""Dynamic plans: a decode loop grows its sequences on the device, without a new plan.

A plan built with ``max_lengths`` covers each sequence up to its capacity;
``run_dynamic`` reads the live page table and lengths from device tensors at
every launch.  Checked against the FP64 oracle on the live metadata, inside
and outside a CUDA graph, and for the clamp of lengths above capacity.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("NVIDIA GPU required", allow_module_level=True)

from oracle.paged_oracle import dense_attention
from paged_decode.layout import Layout
from paged_decode.runtime import DecodePlan
from paged_decode.workload import make_tensors

pytestmark = pytest.mark.gpu
PD_DEVERR_LENGTH = 8


def _oracle(q, k, v, table, lengths):
    return dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)


def _setup(dtype, lengths, reserve, seed=3, heads=32, kv_heads=8, page=16):
    lengths = np.asarray(lengths, dtype=np.int32)
    max_lengths = lengths + reserve
    width = int(-(-max_lengths.max() // page))
    pages = len(lengths) * width
    layout = Layout(len(lengths), heads, kv_heads, 128, page, pages)
    rng = np.random.default_rng(seed)
    full = rng.permutation(pages).reshape(len(lengths), width).astype(np.int32)   # pages to hand out
    table = full.copy()
    for b, n in enumerate(lengths):
        table[b, -(-int(n) // page):] = -1           # not allocated yet
    q, k, v = make_tensors(layout, dtype=dtype, seed=seed)
    return layout, full, table, lengths, max_lengths, q, k, v


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_decode_loop_appends_tokens_without_a_new_plan(dtype):
    layout, full, table, lengths, max_lengths, q, k, v = _setup(dtype, [5, 100, 0, 250], reserve=40)
    plan = DecodePlan(layout, table, lengths, max_lengths=max_lengths)
    assert plan.info.dynamic == 1 and plan.info.max_span == int(max_lengths.max())
    dev_table = torch.tensor(table, device="cuda")
    dev_len = torch.tensor(lengths, device="cuda")
    host_table, host_len = table.copy(), lengths.copy()
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    for step in range(41):
        if step:
            # one token per sequence; a sequence entering a new page gets its page id
            for b in range(layout.batch):
                n = int(host_len[b])
                if n % layout.page_size == 0:
                    host_table[b, n // layout.page_size] = full[b, n // layout.page_size]
                    dev_table[b, n // layout.page_size] = int(full[b, n // layout.page_size])
            host_len += 1
            dev_len += 1
        out = plan.run_dynamic(q, k, v, dev_table, dev_len)
        if step % 10 == 0:
            np.testing.assert_allclose(out.cpu().numpy(), _oracle(q, k, v, host_table, host_len), **tol)
    assert plan.read_errors() == 0


def test_dynamic_decode_loop_replays_in_a_cuda_graph():
    layout, full, _, lengths, max_lengths, q, k, v = _setup(torch.float16, [31, 64, 200, 1], reserve=48, seed=5)
    table = full.copy()                                # all capacity pages handed out up front
    plan = DecodePlan(layout, table, lengths, max_lengths=max_lengths)
    dev_table = torch.tensor(table, device="cuda")
    dev_len = torch.tensor(lengths, device="cuda")
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        plan.run_dynamic(q, k, v, dev_table, dev_len)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            dev_len.add_(1)
            out = plan.run_dynamic(q, k, v, dev_table, dev_len)
        dev_len.copy_(torch.tensor(lengths, device="cuda"))
        for _ in range(48):
            graph.replay()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), _oracle(q, k, v, table, lengths + 48), atol=2e-3, rtol=1e-3)
    assert plan.read_errors() == 0


def test_length_above_capacity_is_clamped_and_flagged():
    layout, full, _, lengths, max_lengths, q, k, v = _setup(torch.float16, [40, 17], reserve=16, seed=9)
    table = full.copy()
    plan = DecodePlan(layout, table, lengths, max_lengths=max_lengths)
    dev_table = torch.tensor(table, device="cuda")
    over = torch.tensor(max_lengths + 5, dtype=torch.int32, device="cuda")
    out = plan.run_dynamic(q, k, v, dev_table, over).clone()
    assert plan.read_errors() & PD_DEVERR_LENGTH
    np.testing.assert_allclose(out.cpu().numpy(), _oracle(q, k, v, table, max_lengths), atol=2e-3, rtol=1e-3)
    assert plan.read_errors() == 0                     # read_errors clears the word


def test_dynamic_plan_runs_its_own_metadata_and_rejects_misuse():
    layout, full, table, lengths, max_lengths, q, k, v = _setup(torch.float32, [9, 300, 0], reserve=20, seed=2)
    plan = DecodePlan(layout, table, lengths, max_lengths=max_lengths)
    np.testing.assert_allclose(plan.run(q, k, v).cpu().numpy(), _oracle(q, k, v, table, lengths),
                               atol=1e-5, rtol=1e-5)
    assert plan.read_errors() == 0
    with pytest.raises(ValueError):
        plan.run_dynamic(q, k, v, torch.tensor(table), torch.tensor(lengths))          # host tensors
    with pytest.raises(ValueError):
        plan.run_dynamic(q, k, v, torch.tensor(table[:, :-1], device="cuda"),
                         torch.tensor(lengths, device="cuda"))                         # wrong width
    with pytest.raises(ValueError):
        DecodePlan(layout, table, lengths).run_dynamic(
            q, k, v, torch.tensor(table, device="cuda"), torch.tensor(lengths, device="cuda"))
    with pytest.raises(ValueError):
        DecodePlan(layout, table, lengths, max_lengths=lengths - 1)
