"""Generate the golden fixtures that pin the oracle and the workload generator.

Run in a container that holds the reference checkout (its Python package is
imported read-only, bytecode writing disabled):

    python tests/golden/make_golden.py --reference-src <checkout>/src

Every array in the .npz files is produced by the REFERENCE's own functions:
``paged_decode.oracle.{dense_attention, streaming_attention, partial_softmax,
merge_partials, validate_metadata}`` and ``paged_decode.workload.{make_metadata,
make_tensors}`` (CPU generator).  Inputs are seeded NumPy draws, so the files
are reproducible.  The tests compare this repository's oracle restatement and
its product-side workload generator against these files; the reference itself
is never needed at test time.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _cases():
    """(name, batch, Hq, Hkv, D, T, lengths, dtype, split, q_scale, seed)."""
    return [
        ("gqa_d64_t16_f32", 3, 8, 2, 64, 16, [0, 1, 35], np.float32, 17, 1.0, 11),
        ("gqa_d128_t16_f16", 2, 8, 2, 128, 16, [47, 16], np.float16, 256, 1.0, 12),
        ("mha_d64_t32_f32", 2, 4, 4, 64, 32, [33, 64], np.float32, 7, 1.0, 13),
        ("mqa_d128_t32_f16", 2, 8, 1, 128, 32, [65, 31], np.float16, 31, 1.0, 14),
        ("large_logits_f32", 2, 8, 1, 128, 16, [64, 37], np.float32, 17, 100.0, 15),
        ("empty_rows_f32", 2, 4, 4, 64, 16, [0, 0], np.float32, 257, 1.0, 16),
        ("ragged_split1_f16", 3, 4, 2, 64, 16, [1, 17, 30], np.float16, 1, 1.0, 17),
    ]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True, type=Path)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(args.reference_src))
    import torch
    from paged_decode import oracle as ref_oracle
    from paged_decode import workload as ref_workload

    # 1. attention cases: random fragmented tables with shared pages.
    attention = {}
    for name, B, Hq, Hkv, D, T, lengths, dtype, split, scale, seed in _cases():
        rng = np.random.default_rng(seed)
        width = max(1, -(-max(lengths) // T))
        pages = B * width
        table = rng.integers(0, pages, size=(B, width)).astype(np.int32)
        lengths = np.asarray(lengths, dtype=np.int32)
        for b, length in enumerate(lengths):
            table[b, -(-int(length) // T):] = -1
        q = (rng.normal(size=(B, Hq, D)) * scale).astype(dtype)
        k = rng.normal(size=(pages, T, Hkv, D)).astype(dtype)
        v = rng.normal(size=(pages, T, Hkv, D)).astype(dtype)
        dense = ref_oracle.dense_attention(q, k, v, table, lengths)
        stream = ref_oracle.streaming_attention(q, k, v, table, lengths, split)
        for key, value in dict(q=q, k=k, v=v, table=table, lengths=lengths, dense=dense,
                               stream=stream, split=np.int64(split),
                               gather_last=ref_oracle.gather_cache(k, table[-1], int(lengths[-1]), Hkv - 1),
                               ).items():
            attention[f"{name}/{key}"] = value
    np.savez_compressed(HERE / "attention.npz", **attention)

    # 2. split-softmax identities (oracle.py:74-96) with extreme logits.
    scores = np.array([-10000.0, 10000.0, 9999.0, 3.0, -2.5])
    values = np.arange(20, dtype=np.float64).reshape(5, 4) - 7.0
    parts = [ref_oracle.partial_softmax(scores[:0], values[:0]),
             ref_oracle.partial_softmax(scores[:1], values[:1]),
             ref_oracle.partial_softmax(scores[1:3], values[1:3]),
             ref_oracle.partial_softmax(scores[3:], values[3:])]
    merge = {
        "scores": scores, "values": values,
        "parts_m": np.array([p[0] for p in parts]), "parts_l": np.array([p[1] for p in parts]),
        "parts_n": np.stack([p[2] for p in parts]),
        "merged": ref_oracle.merge_partials(parts),
        "merged_empty": ref_oracle.merge_partials(parts[:1]),
    }
    np.savez_compressed(HERE / "merge.npz", **merge)

    # 3. workload generator: make_metadata for the BASELINE geometries + edge cases,
    #    make_tensors on the CPU generator (small shapes).
    workload = {}
    for i, args_ in enumerate([
            (4, 32, 8, 128, 4096, 16, 123, False),   # config 1
            (64, 32, 32, 64, 2048, 32, 123, False),  # config 3a
            (64, 32, 1, 128, 2048, 32, 123, False),  # config 3b
            (64, 64, 8, 128, 2048, 32, 123, False),  # config 3c
            (2, 32, 8, 128, 131072, 32, 123, False),  # config 5
            (16, 32, 8, 128, 4096, 16, 123, True),   # reference bench ragged shape
            (3, 4, 2, 64, 35, 16, 123, True),
            (5, 8, 8, 64, 129, 32, 87, True),
            (1, 4, 1, 64, 1, 16, 5, True)]):
        B, H, KV, D, ctx, T, seed, ragged = args_
        layout, table, lengths = ref_workload.make_metadata(B, H, KV, D, ctx, T, seed=seed, ragged=ragged)
        workload[f"meta{i}/args"] = np.array([B, H, KV, D, ctx, T, seed, int(ragged)], dtype=np.int64)
        workload[f"meta{i}/table"] = table
        workload[f"meta{i}/lengths"] = lengths
        workload[f"meta{i}/physical_pages"] = np.int64(layout.physical_pages)
    layout = ref_oracle.Layout(2, 4, 2, 64, 16, 5)
    for dtype_name, dtype in (("f16", torch.float16), ("f32", torch.float32)):
        q, k, v = ref_workload.make_tensors(layout, device="cpu", dtype=dtype, seed=77)
        workload[f"tensors_{dtype_name}/q"] = q.numpy()
        workload[f"tensors_{dtype_name}/k"] = k.numpy()
        workload[f"tensors_{dtype_name}/v"] = v.numpy()
    np.savez_compressed(HERE / "workload.npz", **workload)

    # 4. metadata validation: which inputs the reference rejects, and with what type.
    verdicts = []
    probes = [
        ((2, 4, 2, 64, 16, 4), [[0, 1], [2, 3]], [-1, 1]),
        ((2, 4, 2, 64, 16, 4), [[0, 1], [2, 3]], [33, 1]),
        ((2, 4, 2, 64, 16, 4), [[0, 1], [2, 3]], [32, 32]),
        ((1, 4, 2, 64, 16, 2), [[0, -1]], [1]),
        ((1, 4, 2, 64, 16, 2), [[0, -1]], [17]),
        ((1, 4, 2, 64, 16, 2), [[2, 0]], [1]),
        ((1, 4, 2, 64, 16, 2), [[2, 0]], [0]),
        ((1, 4, 2, 64, 16, 2), [[0.0, 1.0]], [1]),
        ((1, 4, 2, 64, 16, 2), [[0, 1]], [1.0]),
        ((2, 4, 2, 64, 16, 4), [[0, 1]], [1, 1]),
        ((2, 4, 2, 64, 16, 4), [[0, 1], [2, 3]], [1]),
        ((1, 4, 2, 64, 16, 4), [0, 1], [1]),
    ]
    for dims, table, lengths in probes:
        try:
            ref_oracle.validate_metadata(ref_oracle.Layout(*dims), np.array(table), np.array(lengths))
            verdicts.append("ok")
        except Exception as exc:  # noqa: BLE001 - the exception type is the fixture
            verdicts.append(type(exc).__name__)
    import json
    (HERE / "validation_probes.json").write_text(json.dumps(
        [{"dims": list(p[0]), "table": p[1], "lengths": p[2], "verdict": v}
         for p, v in zip(probes, verdicts)], indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
