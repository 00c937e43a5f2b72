"""Product-side plan contract and workload generators against the reference.

Layout / validate_metadata must accept and reject exactly what the reference
does (fixture verdicts from the reference itself, plus the reference's own
CPU test cases, tests/test_oracle.py:26-90).  make_metadata / make_tensors must
be bit-identical to the reference's for equal seeds.
"""
import json

import numpy as np
import pytest

from paged_decode.layout import Layout, validate_metadata
from paged_decode import workload
from tests.conftest import GOLDEN


def test_validation_verdicts_match_reference():
    for probe in json.loads((GOLDEN / "validation_probes.json").read_text()):
        try:
            validate_metadata(Layout(*probe["dims"]), np.array(probe["table"]), np.array(probe["lengths"]))
            verdict = "ok"
        except (ValueError, TypeError) as exc:
            verdict = type(exc).__name__
        assert verdict == probe["verdict"], probe


@pytest.mark.parametrize("bad_lengths", [[-1, 1], [33, 1]])
def test_invalid_lengths_rejected(bad_lengths):
    with pytest.raises(ValueError):
        validate_metadata(Layout(2, 4, 2, 64, 16, 4), np.array([[0, 1], [2, 3]]), np.array(bad_lengths))


def test_padding_is_not_a_live_page():
    layout = Layout(1, 4, 2, 64, 16, 2)
    table, lengths = validate_metadata(layout, np.array([[0, -1]]), np.array([1]))
    assert table.dtype == lengths.dtype == np.int32
    with pytest.raises(ValueError):
        validate_metadata(layout, np.array([[0, -1]]), np.array([17]))
    with pytest.raises(ValueError):
        validate_metadata(layout, np.array([[2, 0]]), np.array([1]))
    with pytest.raises(TypeError):
        validate_metadata(layout, np.array([[0., 1.]]), np.array([1]))


def test_metadata_validation_copies_caller_arrays():
    layout = Layout(1, 4, 2, 64, 16, 2)
    table, lengths = np.array([[0, 1]]), np.array([17])
    copied_table, copied_lengths = validate_metadata(layout, table, lengths)
    table[:] = -1
    lengths[:] = 0
    np.testing.assert_array_equal(copied_table, [[0, 1]])
    np.testing.assert_array_equal(copied_lengths, [17])


@pytest.mark.parametrize("value", [True, False, 1.5, "4", np.float64(4)])
def test_layout_requires_integer_dimensions(value):
    with pytest.raises(TypeError):
        Layout(value, 4, 2, 64, 16, 2)


@pytest.mark.parametrize("value", [0, -1])
def test_layout_requires_positive_dimensions(value):
    with pytest.raises(ValueError):
        Layout(value, 4, 2, 64, 16, 2)


def test_invalid_head_ratio_is_rejected():
    with pytest.raises(ValueError):
        Layout(1, 3, 2, 64, 16, 2)


def test_oracle_module_reexports_contract():
    from paged_decode import oracle
    assert oracle.Layout is Layout and oracle.validate_metadata is validate_metadata


def test_make_metadata_is_bit_identical_to_reference(golden):
    data = golden("workload")
    indices = sorted({key.split("/")[0] for key in data if key.startswith("meta")})
    assert len(indices) == 9
    for idx in indices:
        B, H, KV, D, ctx, T, seed, ragged = (int(x) for x in data[f"{idx}/args"])
        layout, table, lengths = workload.make_metadata(B, H, KV, D, ctx, T, seed=seed, ragged=bool(ragged))
        np.testing.assert_array_equal(table, data[f"{idx}/table"])
        np.testing.assert_array_equal(lengths, data[f"{idx}/lengths"])
        assert table.dtype == data[f"{idx}/table"].dtype and lengths.dtype == data[f"{idx}/lengths"].dtype
        assert layout.physical_pages == int(data[f"{idx}/physical_pages"])


def test_make_tensors_cpu_is_bit_identical_to_reference(golden):
    import torch
    data = golden("workload")
    layout = Layout(2, 4, 2, 64, 16, 5)
    for name, dtype in (("f16", torch.float16), ("f32", torch.float32)):
        q, k, v = workload.make_tensors(layout, device="cpu", dtype=dtype, seed=77)
        for tensor, key in ((q, "q"), (k, "k"), (v, "v")):
            np.testing.assert_array_equal(tensor.numpy(), data[f"tensors_{name}/{key}"])


def test_make_metadata_rejects_nonpositive():
    with pytest.raises(ValueError):
        workload.make_metadata(0, 4, 2, 64, 16, 16)


def test_config2_ragged_shared_prefix_properties():
    w = workload.config2()
    L, table, lengths = w.layout, w.table, w.lengths
    assert (L.batch, L.query_heads, L.kv_heads, L.head_dim, L.page_size) == (32, 32, 8, 128, 16)
    assert w.split_tokens == 256
    assert (lengths >= 0).all() and (lengths <= 8192).all()
    assert sorted(np.flatnonzero(lengths == 0).tolist()) == w.notes["empty"]
    assert all(lengths[i] % 16 != 0 for i in w.notes["ragged_tail"])
    sharers = w.notes["shared_prefix"]
    assert len(sharers) == 8
    prefix = table[sharers[0], :64]
    for b in sharers:
        np.testing.assert_array_equal(table[b, :64], prefix)
        assert lengths[b] >= 64 * 16
    validate_metadata(L, table, lengths)
    live = np.concatenate([table[b, :-(-int(lengths[b]) // 16)] for b in range(32) if lengths[b]])
    # every physical page is used; only the prefix pages are used more than once
    counts = np.bincount(live, minlength=L.physical_pages)
    assert (counts >= 1).all()
    assert set(np.flatnonzero(counts > 1)) == set(prefix.tolist())


def test_config4_and_config5_geometry():
    w4 = workload.config4()
    assert (w4.layout.batch, w4.layout.query_heads, w4.layout.kv_heads) == (256, 64, 8)
    assert (w4.lengths >= 1024).all() and (w4.lengths <= 8192).all()
    assert w4.std == 0.5
    validate_metadata(w4.layout, w4.table, w4.lengths)
    live = np.concatenate([w4.table[b, :-(-int(w4.lengths[b]) // 16)] for b in range(256)])
    assert np.array_equal(np.sort(live), np.arange(w4.layout.physical_pages))
    w5 = workload.config5()
    assert w5.layout.physical_pages == 8192 and (w5.lengths == 131072).all()
    for v in ("a", "b", "c"):
        w3 = workload.config3(v)
        assert w3.split_tokens == 128 and (w3.lengths == 2048).all()
