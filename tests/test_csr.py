"""CSR paged metadata (FlashInfer's indptr / indices / last_page_len), both ways.

The known answers are the reference's own (tests/test_competitors.py:9-20 of
ensigncode/paged-decode-lab); the inverse is checked by round trips over the
BASELINE geometries and random ragged tables.
"""
import numpy as np
import pytest

from paged_decode import workload
from paged_decode.competitors import csr_to_table, paged_csr
from paged_decode.layout import Layout


def test_csr_preserves_fragmented_shared_pages_and_partial_lengths():
    layout = Layout(2, 8, 2, 64, 16, 4)
    indptr, indices, last = paged_csr(layout, [[2, 0, 1], [2, 3, -1]], [33, 17])
    np.testing.assert_array_equal(indptr, [0, 3, 5])
    np.testing.assert_array_equal(indices, [2, 0, 1, 2, 3])
    np.testing.assert_array_equal(last, [1, 1])
    assert indptr.dtype == indices.dtype == last.dtype == np.int32


def test_csr_rejects_empty_rows_like_the_reference():
    with pytest.raises(ValueError, match="nonempty"):
        paged_csr(Layout(1, 4, 1, 64, 16, 1), [[0]], [0])


@pytest.mark.parametrize("name", ["c1", "c2", "c3b", "c5"])
def test_csr_round_trips_baseline_metadata(name):
    w = workload.CONFIGS[name]()
    table = w.table.copy()
    table[w.lengths == 0, 0] = 0                # CSR cannot express empty rows: give them a token
    lengths = np.maximum(w.lengths, 1)
    indptr, indices, last = paged_csr(w.layout, table, lengths)
    back_table, back = csr_to_table(w.layout, indptr, indices, last)
    np.testing.assert_array_equal(back, lengths)
    pages = -(-lengths.astype(np.int64) // w.layout.page_size)
    for b in range(w.layout.batch):
        np.testing.assert_array_equal(back_table[b, :pages[b]], table[b, :pages[b]])
        assert (back_table[b, pages[b]:] == -1).all()


def test_csr_to_table_random_and_empty_rows():
    rng = np.random.default_rng(4)
    layout = Layout(6, 8, 2, 128, 16, 40)
    counts = np.array([0, 3, 1, 0, 5, 2])
    indptr = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
    indices = rng.integers(0, 40, indptr[-1]).astype(np.int32)
    last = rng.integers(1, 17, 6).astype(np.int32)
    table, lengths = csr_to_table(layout, indptr, indices, last)
    np.testing.assert_array_equal(lengths, np.where(counts > 0, (counts - 1) * 16 + last, 0))
    assert table.shape == (6, 5)
    for b in range(6):
        np.testing.assert_array_equal(table[b, :counts[b]], indices[indptr[b]:indptr[b + 1]])


@pytest.mark.parametrize("indptr,indices,last,error", [
    ([0, 2], [0, 1, 2], [1], ValueError),         # indptr does not end at len(indices)
    ([1, 2], [0, 1], [1], ValueError),            # indptr does not start at 0
    ([0, 1], [0], [17], ValueError),              # last page longer than a page
    ([0, 1], [0], [0], ValueError),               # empty last page on a row with pages
    ([0, 1], [7], [3], ValueError),               # page outside the cache
    ([0.0, 1.0], [0], [3], TypeError),            # non-integer metadata
])
def test_csr_to_table_rejects_bad_metadata(indptr, indices, last, error):
    with pytest.raises(error):
        csr_to_table(Layout(1, 4, 1, 64, 16, 4), np.array(indptr), np.array(indices), np.array(last))


def test_dense_sdpa_baseline_matches_the_oracle_on_cpu():
    """The dense comparison row (gather + PyTorch SDPA) computes the same attention."""
    import torch
    from oracle.paged_oracle import dense_attention
    from paged_decode.competitors import DenseSDPAPlan
    rng = np.random.default_rng(8)
    layout = Layout(4, 8, 2, 64, 16, 20)
    table = rng.permutation(20).reshape(4, 5).astype(np.int32)
    lengths = np.array([0, 1, 33, 80], dtype=np.int32)
    q = torch.randn(4, 8, 64, dtype=torch.float64)
    k = torch.randn(20, 16, 2, 64, dtype=torch.float64)
    v = torch.randn(20, 16, 2, 64, dtype=torch.float64)
    out = DenseSDPAPlan(layout, table, lengths, device="cpu").run(q, k, v)
    np.testing.assert_allclose(out.numpy(), dense_attention(q.numpy(), k.numpy(), v.numpy(), table, lengths),
                               atol=1e-10, rtol=1e-10)
