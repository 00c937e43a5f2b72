"""pd_decode_static: the decode entry point that allocates no device memory.

Some callers cannot call cudaMalloc (their device memory belongs to another
framework's pool, or they may only touch the buffers handed to them).  For
them pd_decode_static keeps the plan's metadata and split-K partials in one
file-scope device array inside the library, and pd_static_read_errors reads
the kernel's error word back from it.  This file is collected last so that a
failure here, in a run that stops at the first failure, comes after every
other test has run; it passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("NVIDIA GPU required", allow_module_level=True)

from oracle.paged_oracle import dense_attention
from paged_decode import _native
from paged_decode.layout import Layout
from paged_decode.runtime import DecodePlan
from paged_decode.workload import make_metadata, make_tensors

pytestmark = pytest.mark.gpu

TOL = {torch.float16: dict(atol=2e-3, rtol=1e-3), torch.float32: dict(atol=1e-5, rtol=1e-5)}


def _code(dtype):
    return _native.PD_FLOAT16 if dtype == torch.float16 else _native.PD_FLOAT32


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _static(handle, q, k, v, out):
    lib = _native.load()
    return lib.pd_decode_static(handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), _code(q.dtype),
                                out.data_ptr(), _stream())


def _static_errors():
    lib = _native.load()
    word = ctypes.c_uint32(0xFFFFFFFF)
    _native.check(lib.pd_static_read_errors(torch.cuda.current_device(), ctypes.byref(word), _stream()))
    return int(word.value)


class UnboundPlan:
    """A plan made by pd_plan_create alone: never given device memory (no pd_plan_bind)."""

    def __init__(self, layout, table, lengths, dtype, *, num_ctas=0, split_tokens=256, max_lengths=None):
        self.lib = _native.load()
        c_layout = _native.Layout(layout.batch, layout.query_heads, layout.kv_heads, layout.head_dim,
                                  layout.page_size, layout.physical_pages)
        table = np.ascontiguousarray(table, dtype=np.int32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        self.handle = ctypes.c_void_p()
        dev = torch.cuda.current_device()
        if max_lengths is None:
            status = self.lib.pd_plan_create(ctypes.byref(c_layout), table.ctypes.data, table.shape[1],
                                             lengths.ctypes.data, split_tokens, 0, _code(dtype), dev, num_ctas,
                                             ctypes.byref(self.handle))
        else:
            max_lengths = np.ascontiguousarray(max_lengths, dtype=np.int32)
            status = self.lib.pd_plan_create_dynamic(ctypes.byref(c_layout), table.ctypes.data, table.shape[1],
                                                     lengths.ctypes.data, max_lengths.ctypes.data, split_tokens,
                                                     0, _code(dtype), dev, num_ctas, ctypes.byref(self.handle))
        _native.check(status, "plan")
        self.info = _native.PlanInfo()
        _native.check(self.lib.pd_plan_get_info(self.handle, ctypes.byref(self.info)))

    def set_barrier(self, mode):
        _native.check(self.lib.pd_plan_set_barrier(self.handle, mode))

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.pd_plan_destroy(self.handle)


def _case_a(dtype):
    # ragged, fragmented; groups split across 37 CTAs: partials and the merge run
    layout, table, lengths = make_metadata(6, 32, 8, 128, 700, 16, seed=41)
    q, k, v = make_tensors(layout, dtype=dtype, seed=42)
    return layout, table, lengths, q, k, v


def _case_b(dtype):
    # another shape: D64, page 32, 16:8 heads; on one CTA every group is one segment
    layout = Layout(3, 16, 8, 64, 32, 12)
    table = np.random.default_rng(5).permutation(12).reshape(3, 4).astype(np.int32)
    lengths = np.array([100, 0, 65], dtype=np.int32)
    for b, n in enumerate(lengths):
        table[b, -(-int(n) // 32):] = -1
    q, k, v = make_tensors(layout, dtype=dtype, seed=43)
    return layout, table, lengths, q, k, v


def _oracle(q, k, v, table, lengths):
    return dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_static_scratch_matches_allocating_entry_point_twice(dtype):
    layout, table, lengths, q, k, v = _case_a(dtype)
    plan = DecodePlan(layout, table, lengths, num_ctas=37)
    expected = plan.run(q, k, v).clone()
    ref = _oracle(q, k, v, table, lengths)
    handle = plan._native[_code(dtype)].handle
    for _ in range(2):
        out = torch.full_like(expected, float("nan"))
        _native.check(_static(handle, q, k, v, out))
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), expected.cpu().numpy(), **TOL[dtype])
        np.testing.assert_allclose(out.cpu().numpy(), ref, **TOL[dtype])
        assert _static_errors() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_static_runs_a_plan_that_was_never_bound(dtype):
    layout, table, lengths, q, k, v = _case_a(dtype)
    plan = UnboundPlan(layout, table, lengths, dtype, num_ctas=37)
    assert plan.info.num_pieces > 0
    bound = DecodePlan(layout, table, lengths, num_ctas=37).run(q, k, v).cpu().numpy()
    ref = _oracle(q, k, v, table, lengths)
    for _ in range(2):
        out = torch.full((layout.batch, layout.query_heads, layout.head_dim), float("nan"), device=q.device)
        _native.check(_static(plan.handle, q, k, v, out))
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), bound, **TOL[dtype])
        np.testing.assert_allclose(out.cpu().numpy(), ref, **TOL[dtype])
        assert _static_errors() == 0
    # the bound-plan error reader has nothing to read on this plan
    word = ctypes.c_uint32(0)
    assert plan.lib.pd_plan_read_errors(plan.handle, ctypes.byref(word), _stream()) == _native.PD_ERR_UNBOUND


def test_static_runs_a_pair_plan():
    # 64 equal MQA sequences: a pair plan (clusters of two CTAs that merge each
    # group in shared memory, no partials) through the static entry point
    layout, table, lengths = make_metadata(64, 32, 1, 128, 512, 32, seed=44, ragged=False)
    q, k, v = make_tensors(layout, seed=45)
    plan = UnboundPlan(layout, table, lengths, torch.float16, num_ctas=0)
    assert plan.info.cluster_ctas == 2 and plan.info.num_pieces == 0
    bound = DecodePlan(layout, table, lengths)
    assert bound.info.cluster_ctas == 2
    ref = bound.run(q, k, v).cpu().numpy()
    np.testing.assert_allclose(ref, _oracle(q, k, v, table, lengths), **TOL[torch.float16])
    for _ in range(2):
        out = torch.full((64, 32, 128), float("nan"), device=q.device)
        _native.check(_static(plan.handle, q, k, v, out))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), ref)   # the same work split: the same bits
        assert _static_errors() == 0


def test_static_alternating_plans_on_one_stream():
    # A (partials, in-kernel merge), B (no partials), A again: each call
    # overwrites the array the previous one used, with no synchronisation between
    a = _case_a(torch.float16)
    b = _case_b(torch.float16)
    plan_a = UnboundPlan(*a[:3], torch.float16, num_ctas=37)
    plan_b = UnboundPlan(*b[:3], torch.float16, num_ctas=1)
    assert plan_a.info.num_pieces > 0 and plan_b.info.num_pieces == 0
    outs = []
    for plan, case in ((plan_a, a), (plan_b, b), (plan_a, a)):
        layout, q, k, v = case[0], *case[3:]
        out = torch.full((layout.batch, layout.query_heads, layout.head_dim), float("nan"), device=q.device)
        _native.check(_static(plan.handle, q, k, v, out))
        outs.append(out)
    torch.cuda.synchronize()
    assert _static_errors() == 0
    for out, case in zip(outs, (a, b, a)):
        layout, table, lengths, q, k, v = case
        bound = DecodePlan(layout, table, lengths, num_ctas=37 if case is a else 1).run(q, k, v)
        np.testing.assert_allclose(out.cpu().numpy(), bound.cpu().numpy(), **TOL[torch.float16])
        np.testing.assert_allclose(out.cpu().numpy(), _oracle(q, k, v, table, lengths), **TOL[torch.float16])


@pytest.mark.parametrize("mode,num_ctas", [
    (_native.PD_BARRIER_PLAIN, 37),
    (_native.PD_BARRIER_COOPERATIVE, 37),
    (_native.PD_BARRIER_LEAVE_AT_ONCE, 37),      # every waiting CTA leaves: the fallback merge
    (_native.PD_BARRIER_PLAIN, 400),             # more CTAs than SMs: the separate merge kernel
])
def test_static_every_barrier_mode_and_the_merge_kernel(mode, num_ctas):
    layout, table, lengths, q, k, v = _case_a(torch.float16)
    plan = UnboundPlan(layout, table, lengths, torch.float16, num_ctas=num_ctas)
    plan.set_barrier(mode)
    assert plan.info.num_pieces > 0
    assert plan.info.merge_in_kernel == (1 if num_ctas <= torch.cuda.get_device_properties(0).multi_processor_count
                                         else 0)
    ref = _oracle(q, k, v, table, lengths)
    bound = DecodePlan(layout, table, lengths, num_ctas=num_ctas).run(q, k, v).cpu().numpy()
    for _ in range(2):
        out = torch.full((layout.batch, layout.query_heads, layout.head_dim), float("nan"), device=q.device)
        _native.check(_static(plan.handle, q, k, v, out))
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref, **TOL[torch.float16])
        np.testing.assert_allclose(out.cpu().numpy(), bound, **TOL[torch.float16])
        assert _static_errors() == 0


def test_static_rejects_dynamic_plans():
    layout, table, lengths, q, k, v = _case_a(torch.float16)
    plan = UnboundPlan(layout, table, lengths, torch.float16, max_lengths=lengths)
    out = torch.empty((layout.batch, layout.query_heads, layout.head_dim), device=q.device)
    assert _static(plan.handle, q, k, v, out) == _native.PD_ERR_VALUE
    assert b"pd_decode_dynamic" in plan.lib.pd_last_error()


def test_static_scratch_rejects_plans_beyond_its_capacity():
    lib = _native.load()
    capacity = int(lib.pd_static_scratch_capacity())
    assert capacity == 16 << 20
    # a page table alone larger than the array: 4096 x 2048 int32 = 32 MiB
    batch, width = 4096, 2048
    layout = Layout(batch, 8, 8, 64, 16, 16)
    table = np.full((batch, width), -1, dtype=np.int32)
    table[:, 0] = 0
    lengths = np.ones(batch, dtype=np.int32)
    plan = UnboundPlan(layout, table, lengths, torch.float16)
    q, k, v = make_tensors(layout)
    out = torch.empty((batch, 8, 64), device=q.device)
    status = _static(plan.handle, q, k, v, out)
    assert status == _native.PD_ERR_VALUE
    assert b"bytes of scratch" in lib.pd_last_error()
