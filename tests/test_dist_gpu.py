"""Multi-GPU parity: KV-head and sequence sharding on 2 GPUs against the FP64 oracle.

Two processes (spawned, one per GPU, NCCL with a short timeout) build the same
global workload from one seed, take their shard, and decode.  Rank outputs
are compared with dense attention on the unsharded inputs.  Skipped when
fewer than 2 GPUs are visible.
"""
import datetime
import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
if torch.cuda.device_count() < 2:
    pytest.skip("needs 2 GPUs", allow_module_level=True)

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out, mode):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "paged-decode-lab_b200"), str(root)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from oracle.c_oracle import dense_attention
    from paged_decode import dist as pd_dist
    from paged_decode.layout import Layout
    from paged_decode.workload import make_metadata, make_tensors
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        # "_mqa" modes: 32 query heads on one KV head, the tcgen05 kernel's shape;
        # "_pair": 64 equal sequences, so each rank's plan pairs CTAs in clusters
        kv_heads = 1 if mode.endswith("_mqa") or mode.endswith("_pair") else 8
        batch = 64 if mode.endswith("_pair") else 3
        if mode.endswith("_pair"):
            layout, table, lengths = make_metadata(batch, 32, 1, 128, 1024, 32, seed=5, ragged=False)
        else:
            layout, table, lengths = make_metadata(batch, 32, kv_heads, 128, 3000, 32, seed=5)
        q, k, v = make_tensors(layout, device=f"cuda:{rank}", seed=6)
        if mode == "kv_head":
            plan = pd_dist.KVHeadShardedPlan(layout, table, lengths, rank=rank, world=world,
                                             device=f"cuda:{rank}")
            ql, kl, vl = pd_dist.shard_kv_heads(layout, q, k, v, rank, world)
            out = plan.run(ql, kl, vl).cpu().numpy()
            lo, hi = plan.query_heads
        else:
            lt, ll, _ = pd_dist.shard_sequence_metadata(table, lengths, 32, rank, world)
            ltab, ids = pd_dist.localize_pages(lt, ll, 32)
            loc = Layout(batch, 32, kv_heads, 128, 32, max(1, len(ids)))
            idx = torch.as_tensor(ids, device=q.device)
            kl, vl = k[idx].contiguous(), v[idx].contiguous()
            exchange = "peer" if mode.startswith("sequence_peer") else "nccl"
            plan = pd_dist.SequenceShardedPlan(loc, ltab, ll, device=f"cuda:{rank}", exchange=exchange)
            if mode.endswith("_mqa") or mode.endswith("_pair"):
                assert plan.plan.info.engine == 1   # the tcgen05 kernel
            if mode.endswith("_pair"):
                assert plan.plan.info.cluster_ctas == 2   # (m, l) of pair plans feed the NCCL merge
            first = plan.run(q, kl, vl).clone()
            for _ in range(7):      # alternate exchange parities; every step the same bits
                again = plan.run(q, kl, vl)
                assert torch.equal(again, first)
            out = first.cpu().numpy()
            assert plan.plan.read_errors() == 0
            plan.close()
            lo, hi = 0, 32
        torch.cuda.synchronize()
        ref = dense_attention(*(t.cpu().numpy() for t in (q, k, v)), table, lengths)[:, lo:hi]
        err = float(np.abs(out - ref).max())
        ok = np.allclose(out, ref, atol=2e-3, rtol=1e-3)
        dist.barrier()
        dist.destroy_process_group()
        q_out.put((rank, ok, err))
    except Exception as exc:  # noqa: BLE001
        q_out.put((rank, False, f"{type(exc).__name__}: {exc}"))


@pytest.mark.parametrize("mode", ["kv_head", "sequence", "sequence_peer", "sequence_mqa", "sequence_peer_mqa",
                                  "sequence_pair"])
def test_two_gpu_sharding_matches_oracle(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 240
    while len(results) < 2 and time.time() < deadline:
        try:
            rank, ok, err = q.get(timeout=2)
            results[rank] = (ok, err)
        except Exception:  # noqa: BLE001
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert set(results) == {0, 1}, results
    for rank, (ok, err) in results.items():
        assert ok, (rank, err)
