"""Pin the oracle restatements to vectors produced by the reference's own oracle.

tests/golden/*.npz come from tests/golden/make_golden.py, which imports the
reference package (src/paged_decode/oracle.py).  Both the NumPy restatement and
the C restatement must reproduce them to FP64 round-off; the gather is exact.
"""
import json

import numpy as np
import pytest

from oracle import c_oracle, paged_oracle
from tests.conftest import GOLDEN

CASES = ["gqa_d64_t16_f32", "gqa_d128_t16_f16", "mha_d64_t32_f32", "mqa_d128_t32_f16",
         "large_logits_f32", "empty_rows_f32", "ragged_split1_f16"]


def _case(golden, name):
    data = golden("attention")
    return {key.split("/", 1)[1]: value for key, value in data.items() if key.startswith(name + "/")}


@pytest.mark.parametrize("name", CASES)
def test_numpy_dense_matches_reference(golden, name):
    c = _case(golden, name)
    out = paged_oracle.dense_attention(c["q"], c["k"], c["v"], c["table"], c["lengths"])
    np.testing.assert_allclose(out, c["dense"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", CASES)
def test_numpy_streaming_matches_reference(golden, name):
    c = _case(golden, name)
    out = paged_oracle.streaming_attention(c["q"], c["k"], c["v"], c["table"], c["lengths"],
                                           int(c["split"]))
    np.testing.assert_allclose(out, c["stream"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", CASES)
def test_c_dense_matches_reference(golden, name):
    c = _case(golden, name)
    out = c_oracle.dense_attention(c["q"], c["k"], c["v"], c["table"], c["lengths"], threads=3)
    np.testing.assert_allclose(out, c["dense"], rtol=1e-11, atol=1e-11)


@pytest.mark.parametrize("name", CASES)
def test_gather_is_bit_exact(golden, name):
    c = _case(golden, name)
    got = paged_oracle.gather_cache(c["k"], c["table"][-1], int(c["lengths"][-1]), c["k"].shape[2] - 1)
    assert got.dtype == np.float64
    np.testing.assert_array_equal(got, c["gather_last"])


def test_partial_softmax_and_merge_match_reference(golden):
    g = golden("merge")
    parts = [paged_oracle.partial_softmax(g["scores"][:0], g["values"][:0]),
             paged_oracle.partial_softmax(g["scores"][:1], g["values"][:1]),
             paged_oracle.partial_softmax(g["scores"][1:3], g["values"][1:3]),
             paged_oracle.partial_softmax(g["scores"][3:], g["values"][3:])]
    np.testing.assert_array_equal([p[0] for p in parts], g["parts_m"])
    np.testing.assert_allclose([p[1] for p in parts], g["parts_l"], rtol=1e-15)
    np.testing.assert_allclose(np.stack([p[2] for p in parts]), g["parts_n"], rtol=1e-15)
    np.testing.assert_allclose(paged_oracle.merge_partials(parts), g["merged"], rtol=1e-15)
    np.testing.assert_array_equal(paged_oracle.merge_partials(parts[:1]), g["merged_empty"])


def test_validation_verdicts_match_reference():
    probes = json.loads((GOLDEN / "validation_probes.json").read_text())
    for probe in probes:
        B, Hq, Hkv, D, T, P = probe["dims"]
        try:
            paged_oracle.validate_metadata(B, T, P, np.array(probe["table"]), np.array(probe["lengths"]))
            verdict = "ok"
        except (ValueError, TypeError) as exc:
            verdict = type(exc).__name__
        assert verdict == probe["verdict"], probe


def test_split_bounds_follow_reference_partitions():
    assert paged_oracle.split_bounds(0, 256) == [(0, 0)]
    assert paged_oracle.split_bounds(257, 256) == [(0, 256), (256, 257)]
    assert paged_oracle.split_bounds(5, 1) == [(i, i + 1) for i in range(5)]


def test_algorithmic_bytes_config1_matches_published_figure():
    import sys
    from paged_decode.workload import config1
    w = config1()
    nbytes = paged_oracle.algorithmic_bytes((4, 32, 128), 8, 2, w.table, w.lengths, 16)
    assert nbytes == 67_211_264
