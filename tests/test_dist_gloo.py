"""Multi-GPU host logic on CPU: gloo ranks, world size 2.

Sequence and KV-head sharding are checked for exact coverage; the sequence
sharded path (local split-K over each rank's pages -> packed (o, m, l) ->
all_gather_into_tensor -> max-corrected merge) is run end to end with FP64
oracle math in place of the GPU kernels and compared with dense attention on
the unsharded inputs.  Failure handling: a rank that raises before the
collective, and a rank that never joins, end the other rank with an error
within the process-group timeout instead of hanging.
"""
import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest

from oracle import paged_oracle
from paged_decode import dist as pd_dist
from paged_decode.layout import Layout
from paged_decode.workload import make_metadata

LOG2E = 1.4426950408889634


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------------- pure logic
def test_kv_head_ranges_partition_heads():
    layout = Layout(2, 64, 8, 128, 16, 4)
    for world in (1, 2, 4, 8):
        kv = [pd_dist.kv_head_range(8, r, world) for r in range(world)]
        qh = [pd_dist.query_head_range(layout, r, world) for r in range(world)]
        assert kv[0][0] == 0 and kv[-1][1] == 8 and all(a[1] == b[0] for a, b in zip(kv, kv[1:]))
        assert qh[0][0] == 0 and qh[-1][1] == 64 and all(a[1] == b[0] for a, b in zip(qh, qh[1:]))
        for (klo, khi), (qlo, qhi) in zip(kv, qh):
            # query head h reads KV head h // G
            assert qlo // layout.group == klo and (qhi - 1) // layout.group == khi - 1
    with pytest.raises(ValueError):
        pd_dist.kv_head_range(8, 0, 3)
    with pytest.raises(ValueError):
        pd_dist.kv_head_range(8, 2, 2)


def test_kv_head_shards_reassemble_the_tensors():
    import torch
    layout = Layout(2, 16, 4, 64, 16, 3)
    q = torch.randn(2, 16, 64)
    k = torch.randn(3, 16, 4, 64)
    v = torch.randn(3, 16, 4, 64)
    parts = [pd_dist.shard_kv_heads(layout, q, k, v, r, 2) for r in range(2)]
    torch.testing.assert_close(torch.cat([p[0] for p in parts], dim=1), q)
    torch.testing.assert_close(torch.cat([p[1] for p in parts], dim=2), k)
    assert all(t.is_contiguous() for p in parts for t in p)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_sequence_shards_cover_every_token_once(world):
    layout, table, lengths = make_metadata(5, 8, 2, 64, 333, 16, seed=world)
    covered = np.zeros(len(lengths), dtype=np.int64)
    for r in range(world):
        lt, ll, (lo, hi) = pd_dist.shard_sequence_metadata(table, lengths, 16, r, world)
        paged_oracle.validate_metadata(layout.batch, 16, layout.physical_pages, lt, ll)
        for b in range(layout.batch):
            n = int(ll[b])
            # local token t is global token lo*16 + t and maps to the same physical slot
            np.testing.assert_array_equal(lt[b, : -(-n // 16)], table[b, lo:lo + -(-n // 16)])
            covered[b] += n
    np.testing.assert_array_equal(covered, lengths)


def test_localize_pages_round_trips():
    layout, table, lengths = make_metadata(4, 8, 2, 64, 300, 16, seed=2)
    lt, ll, _ = pd_dist.shard_sequence_metadata(table, lengths, 16, 1, 3)
    local, ids = pd_dist.localize_pages(lt, ll, 16)
    live = np.arange(lt.shape[1])[None, :] < (-(-ll.astype(np.int64) // 16))[:, None]
    np.testing.assert_array_equal(ids[local[live]], lt[live])
    assert (local[~live] == -1).all() and len(np.unique(local[live])) == len(ids)


def test_packed_size():
    assert pd_dist.packed_size(Layout(2, 32, 8, 128, 32, 8192)) * 4 == 33_280


# ---------------------------------------------------------------------- gloo ranks
def _rank_partial(q, k, v, table, lengths):
    """This rank's (normalised o, m in log2 units, l) per (b, h), FP64, as the GPU kernel emits."""
    B, Hq, D = q.shape
    G = Hq // k.shape[2]
    o = np.zeros((B, Hq, D))
    ml = np.zeros((B, Hq, 2))
    for b in range(B):
        n = int(lengths[b])
        for h in range(Hq):
            if n == 0:
                ml[b, h] = (-np.inf, 0.0)
                continue
            keys = paged_oracle.gather_cache(k, table[b], n, h // G)
            vals = paged_oracle.gather_cache(v, table[b], n, h // G)
            x = keys @ q[b, h].astype(np.float64) / np.sqrt(D) * LOG2E
            m = x.max()
            w = np.exp2(x - m)
            o[b, h] = w @ vals / w.sum()
            ml[b, h] = (m, w.sum())
    return o, ml


def _sequence_worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=20))
        layout, table, lengths = make_metadata(3, 8, 2, 64, 200, 16, seed=7)
        rng = np.random.default_rng(3)
        q = rng.normal(size=(3, 8, 64))
        k = rng.normal(size=(layout.physical_pages, 16, 2, 64))
        v = rng.normal(size=k.shape)
        lt, ll, _ = pd_dist.shard_sequence_metadata(table, lengths, 16, rank, world)
        o, ml = _rank_partial(q, k, v, lt, ll)
        rows = 3 * 8
        send = torch.from_numpy(np.concatenate([o.reshape(-1), ml.reshape(-1)]))
        assert send.numel() == pd_dist.packed_size(layout)
        recv = torch.empty(world * send.numel(), dtype=send.dtype)
        dist.all_gather_into_tensor(recv, send)
        stride = pd_dist.packed_size(layout)
        packed = recv.numpy().reshape(world, stride)
        shard_o = packed[:, : rows * 64].reshape(world, rows, 64)
        shard_ml = packed[:, rows * 64:].reshape(world, rows, 2)
        out = np.zeros((rows, 64))
        for r in range(rows):
            parts = [(shard_ml[s, r, 0], shard_ml[s, r, 1], shard_ml[s, r, 1] * shard_o[s, r])
                     for s in range(world)]
            # merge_partials works in natural-log units; the packed m is base 2
            parts = [(m / LOG2E, l, n) for m, l, n in parts]
            out[r] = paged_oracle.merge_partials(parts)
        expected = paged_oracle.dense_attention(q, k, v, table, lengths).reshape(rows, 64)
        result_q.put((rank, float(np.abs(out - expected).max())))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, f"error: {exc!r}"))


def _run_ranks(target, world, *args, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q, *args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + timeout
    while len(results) < world and time.time() < deadline:
        try:
            rank, value = q.get(timeout=1)
            results[rank] = value
        except Exception:  # noqa: BLE001 - queue.Empty
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
    return results


def test_sequence_sharded_merge_over_gloo_matches_dense():
    results = _run_ranks(_sequence_worker, 2)
    assert set(results) == {0, 1}, results
    for rank, err in results.items():
        assert not isinstance(err, str), err
        assert err < 1e-12


def _failing_worker(rank, world, port, result_q, mode):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1 and mode == "never_joins":
        result_q.put((rank, "absent"))
        return
    start = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        if rank == 1 and mode == "raises":
            raise RuntimeError("rank 1 failed before the collective")
        x = torch.ones(4)
        out = torch.empty(4 * world)
        dist.all_gather_into_tensor(out, x)
        result_q.put((rank, "completed"))
    except Exception as exc:  # noqa: BLE001
        result_q.put((rank, ("error", type(exc).__name__, round(time.time() - start, 1))))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


@pytest.mark.parametrize("mode", ["raises", "never_joins"])
def test_peer_failure_ends_the_other_rank_with_an_error(mode):
    start = time.time()
    results = _run_ranks(_failing_worker, 2, mode, timeout=90)
    assert 0 in results, results
    outcome = results[0]
    assert isinstance(outcome, tuple) and outcome[0] == "error", outcome
    assert time.time() - start < 90
