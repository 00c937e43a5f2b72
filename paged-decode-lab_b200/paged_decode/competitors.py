"""The CSR paged-KV metadata format, both ways, and the FlashInfer comparison adapter.

``paged_csr`` turns a page table into the CSR form that FlashInfer's paged
decode takes (ensigncode/paged-decode-lab src/paged_decode/competitors.py:8-18):
``indptr [B+1]`` (prefix sums of each row's live page count), ``indices``
(the live physical page ids, row after row) and ``last_page_len [B]`` (tokens
in each row's last page).  Same accepted inputs, same errors, int32 outputs.

``csr_to_table`` is the inverse, so that CSR metadata can feed a
``DecodePlan`` directly (``DecodePlan.from_csr``): row b's pages become table
row b (padded with -1 to the longest row) and its length is
``(pages - 1) * page_size + last_page_len`` (0 for a row without pages).

``FlashInferPlan`` runs FlashInfer's own batch decode on the same NHD caches,
without copying them (the reference's measured competitor,
competitors.py:21-62), and ``DenseSDPAPlan`` the dense baseline the reference
reports (src/paged_decode/reference.py:7-46): gather the live pages into
zero-padded [B, Hkv, L, D] tensors, then PyTorch's scaled_dot_product_attention
with a length mask.  Comparison harness only, never on this package's decode
path.
"""
from __future__ import annotations

import math

import numpy as np

from .layout import Layout, validate_metadata

__all__ = ["paged_csr", "csr_to_table", "FlashInferPlan", "DenseSDPAPlan"]


def paged_csr(layout: Layout, table, lengths):
    """(indptr, indices, last_page_len), all int32, of a validated page table."""
    table, lengths = validate_metadata(layout, table, lengths)
    if (lengths == 0).any():
        raise ValueError("FlashInfer comparison requires nonempty contexts")
    pages = -(-lengths.astype(np.int64) // layout.page_size)
    indptr = np.zeros(len(pages) + 1, dtype=np.int64)
    np.cumsum(pages, out=indptr[1:])
    if indptr[-1] > np.iinfo(np.int32).max:
        raise ValueError("CSR page list exceeds int32 capacity")
    live = np.arange(table.shape[1])[None, :] < pages[:, None]
    indices = table[live]                      # row-major: row 0's pages, then row 1's, ...
    last = (lengths.astype(np.int64) - 1) % layout.page_size + 1
    return indptr.astype(np.int32), indices.astype(np.int32), last.astype(np.int32)


def csr_to_table(layout: Layout, indptr, indices, last_page_len):
    """(table [B, W] int32 with -1 padding, lengths [B] int32) of CSR metadata.

    Rows with no pages have length 0 (the CSR form itself cannot express an
    empty row with a page; ``last_page_len`` of such rows is ignored).  The
    result is validated like any page table.
    """
    indptr = np.asarray(indptr)
    indices = np.asarray(indices)
    last = np.asarray(last_page_len)
    if indptr.shape != (layout.batch + 1,) or last.shape != (layout.batch,) or indices.ndim != 1:
        raise ValueError("CSR metadata must be indptr [batch+1], indices [n], last_page_len [batch]")
    if indptr.dtype.kind not in "iu" or indices.dtype.kind not in "iu" or last.dtype.kind not in "iu":
        raise TypeError("metadata must contain integers")
    counts = np.diff(indptr.astype(np.int64))
    if indptr[0] != 0 or (counts < 0).any() or indptr[-1] != len(indices):
        raise ValueError("indptr must start at 0, not decrease, and end at len(indices)")
    if ((counts > 0) & ((last < 1) | (last > layout.page_size))).any():
        raise ValueError("last_page_len must be in [1, page_size] for rows with pages")
    width = max(1, int(counts.max(initial=0)))
    table = np.full((layout.batch, width), -1, dtype=np.int64)
    rows = np.repeat(np.arange(layout.batch), counts)
    cols = np.arange(len(indices)) - np.repeat(indptr[:-1].astype(np.int64), counts)
    table[rows, cols] = indices
    lengths = np.where(counts > 0, (counts - 1) * layout.page_size + last.astype(np.int64), 0)
    return validate_metadata(layout, table, lengths)


class FlashInferPlan:
    """FlashInfer's batch decode over the same NHD k/v tensors (FP16 only).

    Plan construction, metadata upload and its 1 GiB workspace stay outside
    any timing (its tensor-core path at B256 x 64 query heads overflows the
    usual 128 MiB).  FlashInfer writes FP16 output; this package's decode
    writes FP32.
    """

    def __init__(self, layout: Layout, table, lengths, *, device="cuda", tensor_cores=False, backend="auto"):
        import flashinfer
        import torch
        indptr, indices, last = paged_csr(layout, table, lengths)
        self.version = flashinfer.__version__
        self.tensor_cores = tensor_cores
        self.backend = backend
        self.workspace = torch.zeros(2**30, dtype=torch.uint8, device=device)
        self.indptr = torch.tensor(indptr, device=device)
        self.indices = torch.tensor(indices, device=device)
        self.last = torch.tensor(last, device=device)
        self.out = torch.empty((layout.batch, layout.query_heads, layout.head_dim),
                               dtype=torch.float16, device=device)
        self.wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
            self.workspace, "NHD", use_cuda_graph=True, use_tensor_cores=tensor_cores,
            paged_kv_indptr_buffer=self.indptr, paged_kv_indices_buffer=self.indices,
            paged_kv_last_page_len_buffer=self.last, backend=backend)
        self.wrapper.plan(self.indptr, self.indices, self.last, layout.query_heads, layout.kv_heads,
                          layout.head_dim, layout.page_size, q_data_type=torch.float16,
                          kv_data_type=torch.float16, pos_encoding_mode="NONE",
                          sm_scale=1 / math.sqrt(layout.head_dim))

    def run(self, q, k, v):
        import torch
        if q.dtype != torch.float16 or k.dtype != q.dtype or v.dtype != q.dtype:
            raise TypeError("FlashInfer comparison adapter requires FP16 inputs")
        return self.wrapper.run(q, (k, v), out=self.out)


class DenseSDPAPlan:
    """Gather the pages into dense K/V, then ``torch.nn.functional.scaled_dot_product_attention``.

    The gather indices (physical page, slot) and the length mask are built
    once; ``run`` does the gather (one indexed copy per cache) and the SDPA
    call, both timed as the step.  Query heads share their KV head through
    SDPA's GQA support, so the dense tensors are not repeated per query head.
    All-empty rows come out as zeros (the reference's convention).
    """

    def __init__(self, layout: Layout, table, lengths, *, device="cuda"):
        import torch
        table, lengths = validate_metadata(layout, table, lengths)
        self.layout = layout
        span = max(1, int(lengths.max(initial=0)))
        pos = np.arange(span)
        live = pos[None, :] < lengths[:, None]
        page_idx = np.where(live, pos[None, :] // layout.page_size, 0)
        phys = np.take_along_axis(np.maximum(table, 0), page_idx, axis=1)
        self.pages = torch.tensor(np.where(live, phys, 0), dtype=torch.long, device=device)
        self.slots = torch.tensor(np.where(live, pos[None, :] % layout.page_size, 0), dtype=torch.long,
                                  device=device)
        self.mask = torch.tensor(live, device=device)[:, None, None, :]   # [B, 1, 1, L]
        self.empty = torch.tensor(lengths == 0, device=device)[:, None, None]

    def run(self, q, k, v):
        import torch
        import torch.nn.functional as F
        dense_k = k[self.pages, self.slots].permute(0, 2, 1, 3)       # [B, Hkv, L, D]
        dense_v = v[self.pages, self.slots].permute(0, 2, 1, 3)
        out = F.scaled_dot_product_attention(q.unsqueeze(2), dense_k, dense_v, attn_mask=self.mask,
                                             enable_gqa=True).squeeze(2)
        return torch.where(self.empty, torch.zeros_like(out), out)
