"""The peer-exchange decode (pd_decode_exchange) with a world of one rank, on one GPU.

With one rank every output row still takes the exchange path: the decode stores
its rows (normalised o, m, l) into the rank's own exchange buffer with the
launch's tag, then merges them back out once the tags show this launch.  That
runs the in-kernel merge's exchange writes (direct rows, whole-row merges,
teams of warps, and the row streaming of kernels with four or fewer consumer
warps) without a second GPU.  The result must match the ordinary decode.
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
    # 64 sequences over every SM: ~14 split rows per CTA, 4 consumer warps (row streaming)
    "f16_p32_streamed_rows": (torch.float16, (64, 32, 8, 128, 32, [2048] * 64, 21)),
    # a few long sequences: teams of warps per row, plus short unsplit ones written directly
    "f16_p16_teams": (torch.float16, (4, 32, 8, 128, 16, [7000, 3, 0, 5000], 22)),
    "f32_d64_rows": (torch.float32, (8, 8, 8, 64, 16, [900, 2500, 1, 4000, 0, 300, 1700, 64], 23)),
    # MQA tiles of 32 query heads on the tcgen05 kernel: its own exchange writes (two warps per row)
    "f16_mqa_tcgen05": (torch.float16, (64, 32, 1, 128, 32, [2048] * 64, 24)),
    "f16_mqa_tcgen05_ragged": (torch.float16, (8, 64, 1, 128, 32, [4000, 3, 0, 2000, 64, 700, 1, 5000], 25)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_one_rank_exchange_matches_the_plain_decode(name):
    dtype, args = CASES[name]
    layout, table, lengths = _case(*args)
    q, k, v = make_tensors(layout, dtype=dtype, seed=args[-1])
    # exchange plans take one CTA per SM (num_ctas > 0: no CTA-pair plan)
    plan = DecodePlan(layout, table, lengths, num_ctas=torch.cuda.get_device_properties(0).multi_processor_count)
    if "tcgen05" in name:
        assert plan.info.engine == _native.PD_ENGINE_TCGEN05
    ref = plan.run(q, k, v).clone()
    lib = _native.load()
    code = _native.PD_FLOAT16 if dtype == torch.float16 else _native.PD_FLOAT32
    handle = plan._native[code].handle
    dev = q.device.index
    nbytes = int(lib.pd_exchange_bytes(handle, 1))
    assert nbytes > 0
    buf, ipc = ctypes.c_void_p(), ctypes.create_string_buffer(64)
    assert lib.pd_exchange_alloc(dev, nbytes, ctypes.byref(buf), ipc) == _native.PD_OK
    try:
        ptrs = (ctypes.c_void_p * 1)(buf.value)
        out = torch.empty_like(ref)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        for _ in range(5):      # both buffer parities, launch tags 1..5
            out.fill_(float("nan"))
            assert lib.pd_decode_exchange(handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), code, ptrs, 0, 1,
                                          out.data_ptr(), None, stream) == _native.PD_OK
            torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
        torch.cuda.synchronize()
        assert plan.read_errors() == 0
    finally:
        torch.cuda.synchronize()
        lib.pd_exchange_free(dev, buf)
    tol = dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    expected = dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)
    np.testing.assert_allclose(out.cpu().numpy(), expected, **tol)
