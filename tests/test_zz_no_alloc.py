"""pd_decode_static: the decode entry point that allocates no device memory.

Some callers cannot call cudaMalloc (their device memory belongs to another
framework's pool, or they may only touch the buffers handed to them).  For
them pd_decode_static keeps the plan's metadata and split-K partials in one
file-scope device array inside the library.  This file is collected last so
that a failure here, in a run that stops at the first failure, comes after
every other test has run; it passes alone in a fresh process as well.
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


def _static(plan, q, k, v, out):
    lib = _native.load()
    code = _native.PD_FLOAT16 if q.dtype == torch.float16 else _native.PD_FLOAT32
    handle = plan._native[code].handle
    stream = torch.cuda.current_stream().cuda_stream
    return lib.pd_decode_static(handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), code,
                                out.data_ptr(), stream)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_static_scratch_matches_allocating_entry_point_twice(dtype):
    # ragged, fragmented, some groups split across CTAs: partials are exercised
    layout, table, lengths = make_metadata(6, 32, 8, 128, 700, 16, seed=41)
    q, k, v = make_tensors(layout, dtype=dtype, seed=42)
    plan = DecodePlan(layout, table, lengths, num_ctas=37)
    expected = plan.run(q, k, v).clone()
    ref = dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    for _ in range(2):
        out = torch.full_like(expected, float("nan"))
        _native.check(_static(plan, q, k, v, out))
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), expected.cpu().numpy(), **tol)
        np.testing.assert_allclose(out.cpu().numpy(), ref, **tol)


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
    plan = DecodePlan(layout, table, lengths)
    q, k, v = make_tensors(layout)
    out = torch.empty((batch, 8, 64), device=q.device)
    status = _static(plan, q, k, v, out)
    assert status == _native.PD_ERR_VALUE
    assert b"bytes of scratch" in lib.pd_last_error()
