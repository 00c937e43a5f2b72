"""Multi-GPU decode plans: one process per GPU, torch.distributed for plumbing.

The reference never ran on more than one GPU.  The path partitions in two
natural ways:

* ``KVHeadShardedPlan`` -- rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N), the
  query heads that read them and its own cache shard [P, T, Hkv/N, D].  Each
  rank runs an ordinary DecodePlan on ``Layout(B, Hq/N, Hkv/N, D, T, P)``; the
  output stays sharded by head (the usual tensor-parallel attention layout),
  so there is no collective at all.

* ``SequenceShardedPlan`` -- rank r owns a contiguous run of the logical pages
  of every sequence (with those pages resident in its own cache).  Its rows
  (normalised o, m, l per (b, h)) from all ranks are merged with the
  max-corrected merge, the same algebra the reference uses across context
  partitions (src/paged_decode/oracle.py:88-96).  By default one kernel per
  rank does it all: decode, store the rows into every rank's exchange buffer
  over NVLink, wait for the other ranks, merge (``pd_decode_exchange``).  The
  alternative is ``run_with_stats`` + NCCL ``all_gather_into_tensor`` +
  ``pd_merge_shards``.  NVLink bytes per step per rank: (N-1) * B*Hq*(D+2)*4
  received.

The pure functions (``kv_head_range``, ``query_head_range``,
``shard_sequence_metadata``, ``packed_size``) carry the sharding logic and are
tested on CPU with gloo ranks; the plan classes add the GPU work.
"""
from __future__ import annotations

import ctypes
import datetime

import numpy as np

from . import _native
from .layout import Layout, validate_metadata
from .runtime import DecodePlan

__all__ = ["kv_head_range", "query_head_range", "shard_kv_heads", "shard_sequence_metadata",
           "localize_pages", "packed_size", "KVHeadShardedPlan", "SequenceShardedPlan",
           "init_process_group"]


# ---------------------------------------------------------------------- host logic
def kv_head_range(kv_heads: int, rank: int, world: int):
    """KV heads [lo, hi) owned by ``rank`` under KV-head sharding."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if kv_heads % world:
        raise ValueError("kv_heads must be divisible by the number of ranks")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def query_head_range(layout: Layout, rank: int, world: int):
    """Query heads [lo, hi) that read the KV heads of ``rank`` (head h reads KV head h // G)."""
    lo, hi = kv_head_range(layout.kv_heads, rank, world)
    return lo * layout.group, hi * layout.group


def shard_kv_heads(layout: Layout, q, k, v, rank: int, world: int):
    """Slice full q / k / v tensors to ``rank``'s KV-head shard (contiguous copies)."""
    klo, khi = kv_head_range(layout.kv_heads, rank, world)
    qlo, qhi = query_head_range(layout, rank, world)
    return (q[:, qlo:qhi].contiguous(), k[:, :, klo:khi].contiguous(), v[:, :, klo:khi].contiguous())


def shard_sequence_metadata(table, lengths, page_size: int, rank: int, world: int):
    """Rank ``rank``'s logical pages of every sequence under sequence sharding.

    The table's logical pages [0, W) are cut into ``world`` contiguous runs
    (rank r: [r*W//N, (r+1)*W//N)).  Returns (local_table, local_lengths,
    (first_page, end_page)): the local table holds that run of each row (so the
    same physical page ids, -1 padding kept), and the local length of sequence
    b is how many of its tokens fall in the run.  Attention over a set of keys
    does not depend on their order, so the runs' results merge exactly.
    """
    table = np.asarray(table)
    lengths = np.asarray(lengths, dtype=np.int64)
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    width = table.shape[1]
    lo, hi = rank * width // world, (rank + 1) * width // world
    local_len = np.clip(lengths - lo * page_size, 0, (hi - lo) * page_size).astype(np.int32)
    local_table = np.ascontiguousarray(table[:, lo:hi], dtype=np.int32)
    if local_table.shape[1] == 0:
        local_table = np.full((table.shape[0], 1), -1, dtype=np.int32)
    return local_table, local_len, (lo, hi)


def localize_pages(table, lengths, page_size: int):
    """Compact a rank's page table onto a local cache holding only its pages.

    Returns (local_table, global_page_ids): local_table renumbers the live
    pages 0..n-1 (padding stays -1) and global_page_ids[i] is the physical page
    of the full cache that local page i holds, so a rank can build its cache
    shard as k_full[global_page_ids].
    """
    table = np.asarray(table)
    lengths = np.asarray(lengths, dtype=np.int64)
    live = np.arange(table.shape[1])[None, :] < (-(-lengths // page_size))[:, None]
    ids = np.unique(table[live])
    local = np.full(table.shape, -1, dtype=np.int32)
    local[live] = np.searchsorted(ids, table[live]).astype(np.int32)
    return local, ids.astype(np.int64)


def packed_size(layout: Layout) -> int:
    """Floats per rank in the all-gathered buffer: B*Hq*D outputs then B*Hq*2 (m, l)."""
    return layout.batch * layout.query_heads * (layout.head_dim + 2)


def init_process_group(backend="nccl", timeout_s=60.0, device=None):
    """Initialise torch.distributed from the torchrun environment with a short timeout,
    so that ranks waiting for a missing peer fail instead of hanging."""
    import torch
    import torch.distributed as dist
    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl" and device is not None:
        kwargs["device_id"] = torch.device(device)
    dist.init_process_group(backend, **kwargs)
    return dist.get_rank(), dist.get_world_size()


# ---------------------------------------------------------------------- plans
class KVHeadShardedPlan:
    """KV-head sharding: rank r decodes its own heads with an ordinary plan; no collective."""

    def __init__(self, layout: Layout, table, lengths, *, rank: int, world: int, device="cuda",
                 split_tokens=256, merge="serial", num_ctas=None):
        self.kv_heads = kv_head_range(layout.kv_heads, rank, world)
        self.query_heads = query_head_range(layout, rank, world)
        self.rank, self.world = rank, world
        self.global_layout = layout
        self.local_layout = Layout(layout.batch, layout.query_heads // world, layout.kv_heads // world,
                                   layout.head_dim, layout.page_size, layout.physical_pages)
        self.plan = DecodePlan(self.local_layout, table, lengths, device=device,
                               split_tokens=split_tokens, merge=merge, num_ctas=num_ctas)

    def run(self, q_local, k_local, v_local):
        """Decode this rank's heads: q [B, Hq/N, D], k/v [P, T, Hkv/N, D] -> FP32 [B, Hq/N, D]."""
        return self.plan.run(q_local, k_local, v_local)


class SequenceShardedPlan:
    """Sequence sharding: local split-K over this rank's pages, exchange, merge.

    ``table``/``lengths`` are this rank's local metadata (see
    ``shard_sequence_metadata``) over its own cache shard of ``physical_pages``
    pages.  ``run`` returns the full FP32 [B, Hq, D] output on every rank.

    ``exchange="peer"`` (default, up to 8 ranks on one node): one kernel per
    rank and step decodes, stores its rows into every rank's exchange buffer
    over NVLink (CUDA IPC peer mappings, no multicast) with a per-row launch
    tag, and merges each output row once every rank's copy of it has arrived
    (bounded wait; ``pd_decode_exchange``).  ``exchange="nccl"``:
    ``run_with_stats``, NCCL ``all_gather_into_tensor``, ``pd_merge_shards``.
    Every rank must call ``run`` once per step; call ``close`` on every rank
    (it synchronises them) before the process group goes away.
    """

    def __init__(self, layout: Layout, table, lengths, *, group=None, device="cuda",
                 split_tokens=256, merge="serial", num_ctas=None, exchange="peer"):
        import torch
        import torch.distributed as dist
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.layout = layout
        self.exchange = exchange
        table, lengths = validate_metadata(layout, table, lengths)
        if num_ctas is None and exchange == "peer":
            # one CTA per SM: the exchange kernel takes no CTA-pair plans
            num_ctas = torch.cuda.get_device_properties(torch.device(device)).multi_processor_count
        self.plan = DecodePlan(layout, table, lengths, device=device, split_tokens=split_tokens,
                               merge=merge, num_ctas=num_ctas)
        self.device = self.plan.device
        rows = layout.batch * layout.query_heads
        self._rows = rows
        self._out = torch.empty((layout.batch, layout.query_heads, layout.head_dim), dtype=torch.float32,
                                device=self.device)
        self._lib = _native.load()
        self._buffer = None
        self._peers = []
        if exchange == "peer":
            if self.world > 8:
                raise ValueError("peer exchange supports at most 8 ranks")
            self._setup_peer()
        else:
            self._send = torch.empty(packed_size(layout), dtype=torch.float32, device=self.device)
            self._recv = torch.empty(self.world * packed_size(layout), dtype=torch.float32,
                                     device=self.device)
            D = layout.head_dim
            self._local_out = self._send[: rows * D].view(layout.batch, layout.query_heads, D)
            self._local_stats = self._send[rows * D:].view(layout.batch, layout.query_heads, 2)

    def _setup_peer(self):
        import torch.distributed as dist
        lib, dev = self._lib, self.device.index
        # one buffer per rank, opened by every other rank
        nbytes = int(lib.pd_exchange_bytes(self.plan._native[_native.PD_FLOAT16].handle, self.world))
        buffer, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        _native.check(lib.pd_exchange_alloc(dev, nbytes, ctypes.byref(buffer), handle), "exchange")
        self._buffer = buffer
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=self.group)
        ptrs = []
        for s, h in enumerate(handles):
            if s == self.rank:
                ptrs.append(buffer.value)
                continue
            peer = ctypes.c_void_p()
            _native.check(lib.pd_exchange_open(dev, ctypes.create_string_buffer(h, 64), ctypes.byref(peer)),
                          "exchange")
            self._peers.append(peer)
            ptrs.append(peer.value)
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=self.group)

    @property
    def nvlink_bytes_per_step(self):
        """Bytes each rank receives from its peers per decode step."""
        return (self.world - 1) * packed_size(self.layout) * 4

    def run(self, q, k_local, v_local):
        import torch
        import torch.distributed as dist
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self.exchange == "peer":
            dtype = self.plan._check_inputs(q, k_local, v_local)
            _native.check(self._lib.pd_decode_exchange(
                self.plan._native[dtype].handle, q.data_ptr(), k_local.data_ptr(), v_local.data_ptr(), dtype,
                self._ptrs, self.rank, self.world, self._out.data_ptr(), None, stream), "decode")
            return self._out
        self.plan.run_with_stats(q, k_local, v_local, self._local_out, self._local_stats)
        dist.all_gather_into_tensor(self._recv, self._send, group=self.group)
        D = self.layout.head_dim
        stride = packed_size(self.layout)
        base = self._recv.data_ptr()
        _native.check(self._lib.pd_merge_shards(
            base, base + self._rows * D * 4, self.world, stride, self._rows, D, self._out.data_ptr(),
            stream), "merge_shards")
        return self._out

    def close(self):
        """Unmap the peers' buffers and free this rank's, once every rank is done with them."""
        import torch
        import torch.distributed as dist
        if self._buffer is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for peer in self._peers:
            self._lib.pd_exchange_close(self.device.index, peer)
        self._peers = []
        dist.barrier(group=self.group)
        self._lib.pd_exchange_free(self.device.index, self._buffer)
        self._buffer = None
