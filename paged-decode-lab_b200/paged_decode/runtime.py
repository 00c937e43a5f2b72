"""Validated, allocation-free decode plans over the sm_100a kernel library.

``DecodePlan`` keeps the reference's surface (src/paged_decode/runtime.py:23-90):
same constructor arguments, the same attributes (``layout``, ``split_tokens``,
``splits``, ``max_context``, ``merge``, ``merge_implementation``, ``device``,
``workspace_bytes``), the same exceptions, and ``run`` returning the borrowed
FP32 [batch, query_heads, head_dim] output.  Underneath, the plan is built by
the C ABI (include/paged_decode.h): metadata is validated, the pages of all
(sequence, KV head) groups are balanced across one persistent CTA per SM, and
metadata plus split-K workspace live in one device buffer that this class
allocates through PyTorch.  ``run`` allocates nothing and never synchronises,
so it can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _native
from .layout import Layout, validate_metadata

__all__ = ["DecodePlan", "inspect_plan", "load_extension"]


def load_extension():
    """Load the prebuilt native library (the reference JIT-compiles here, runtime.py:9-20)."""
    return _native.load()


def _check_limits(layout, split_tokens, merge):
    if merge not in ("serial", "shared"):
        raise ValueError("merge must be 'serial' or 'shared'")
    if layout.head_dim not in (64, 128):
        raise ValueError("head_dim must be 64 or 128")
    if layout.page_size not in (16, 32):
        raise ValueError("page_size must be 16 or 32")
    if layout.batch > 65535 or layout.query_heads > 65535:
        raise ValueError("batch/head count exceeds CUDA grid limits")
    if isinstance(split_tokens, bool) or not isinstance(split_tokens, int) or \
            not 1 <= split_tokens <= 1048576:
        raise ValueError("split_tokens must be an integer in [1,1048576]")


def _native_plan(layout, table, lengths, split_tokens, merge, dtype_code, device_index, num_ctas,
                 max_lengths=None):
    lib = _native.load()
    c_layout = _native.Layout(layout.batch, layout.query_heads, layout.kv_heads, layout.head_dim,
                              layout.page_size, layout.physical_pages)
    table = np.ascontiguousarray(table, dtype=np.int32)
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    handle = ctypes.c_void_p()
    if max_lengths is None:
        status = lib.pd_plan_create(ctypes.byref(c_layout), table.ctypes.data, table.shape[1],
                                    lengths.ctypes.data, split_tokens, int(merge == "shared"),
                                    dtype_code, device_index, num_ctas or 0, ctypes.byref(handle))
    else:
        max_lengths = np.ascontiguousarray(max_lengths, dtype=np.int32)
        status = lib.pd_plan_create_dynamic(ctypes.byref(c_layout), table.ctypes.data, table.shape[1],
                                            lengths.ctypes.data, max_lengths.ctypes.data, split_tokens,
                                            int(merge == "shared"), dtype_code, device_index,
                                            num_ctas or 0, ctypes.byref(handle))
    _native.check(status, "plan")
    return handle


def _worklist(lib, handle):
    info = _native.PlanInfo()
    _native.check(lib.pd_plan_get_info(handle, ctypes.byref(info)))
    segs = np.empty((info.num_segments, 4), dtype=np.int32)
    groups = np.empty((info.num_groups, 8), dtype=np.int32)
    offsets = np.empty(info.num_ctas + 1, dtype=np.int32)
    _native.check(lib.pd_plan_copy_worklist(handle, segs.ctypes.data, groups.ctypes.data,
                                            offsets.ctypes.data))
    return info, segs, groups, offsets


_DTYPE_CODES = {"float16": _native.PD_FLOAT16, "float32": _native.PD_FLOAT32}


def inspect_plan(layout: Layout, table, lengths, *, split_tokens=256, num_ctas=148, dtype="float16",
                 max_lengths=None):
    """Build a host-only plan (no GPU needed) for one input dtype and return its work list.

    Returns a dict with ``info`` (pd_plan_info fields), ``segments``
    [n, 4] = (group, first_page, end_page, first partial slot or -1),
    ``groups`` [g, 8] = (batch, first_kv_head, query_head_offset, query_heads,
    length, first partial slot or -1, segments, 0) and ``cta_offsets``
    [num_ctas + 1].
    """
    _check_limits(layout, split_tokens, "serial")
    table, lengths = validate_metadata(layout, table, lengths)
    lib = _native.load()
    handle = _native_plan(layout, table, lengths, split_tokens, "serial", _DTYPE_CODES[dtype], -1, num_ctas,
                          max_lengths)
    try:
        info, segs, groups, offsets = _worklist(lib, handle)
    finally:
        lib.pd_plan_destroy(handle)
    return {"info": {name: getattr(info, name) for name, _ in info._fields_},
            "segments": segs, "groups": groups, "cta_offsets": offsets}


def _align256(n):
    return (int(n) + 255) // 256 * 256


class _NativePlan:
    """One C-ABI plan (one input dtype); ``DecodePlan`` binds it to device memory."""

    def __init__(self, lib, layout, table, lengths, split_tokens, merge, dtype_code, device, num_ctas,
                 max_lengths=None):
        self._lib = lib
        self.handle = _native_plan(layout, table, lengths, split_tokens, merge, dtype_code,
                                   device.index, num_ctas, max_lengths)
        self.info, self.segments, self.groups, self.cta_offsets = _worklist(lib, self.handle)
        self.metadata_bytes = int(lib.pd_plan_metadata_bytes(self.handle))
        self.workspace_bytes = int(lib.pd_plan_workspace_bytes(self.handle))

    def __del__(self):
        handle = getattr(self, "handle", None)
        if handle:
            self._lib.pd_plan_destroy(handle)
            self.handle = None


class DecodePlan:
    """A decode plan for one batch's fixed metadata, reusable across steps.

    The constructor validates the layout and the CPU page table / lengths,
    keeps its own copies of them, and lays out everything a decode step needs
    on the device: a balanced work list and one split-K workspace.  Between
    runs only the contents of q, k and v may change; new lengths or pages
    need a new plan (or a dynamic plan, ``max_lengths``).  ``run`` hands back
    the plan's own FP32 output tensor, which the next run overwrites.  Launch
    a plan from one stream at a time; concurrent streams need a plan each.

    ``merge`` is accepted for compatibility: the B200 path always merges
    split partials the same way (inside the decode kernel after a grid
    barrier, or in a dependent merge kernel), and ``merge_implementation``
    keeps the reference's classification ("serial", "shared" or
    "serial_fallback", runtime.py:54).  ``num_ctas`` (extension) overrides
    the persistent grid size, which by default is one CTA per SM.

    Each input dtype has its own native plan (page tiles are sized per
    dtype).  Both live in one device buffer: their metadata side by side and
    one shared split-K workspace of the larger size, since a plan's launches
    stay in one stream order and a workspace carries nothing between them.
    """

    def __init__(self, layout: Layout, table, lengths, *, device="cuda", split_tokens=256,
                 merge="serial", num_ctas=None, max_lengths=None):
        import torch
        _check_limits(layout, split_tokens, merge)
        table, lengths = validate_metadata(layout, table, lengths)
        if max_lengths is not None:
            max_lengths = np.asarray(max_lengths)
            if max_lengths.shape != lengths.shape or max_lengths.dtype.kind not in "iu":
                raise ValueError("max_lengths must be integers of shape [batch]")
            if (max_lengths < lengths).any() or (max_lengths > table.shape[1] * layout.page_size).any():
                raise ValueError("max_lengths must lie between lengths and the page table capacity")
            max_lengths = max_lengths.astype(np.int32)
        self.max_lengths = max_lengths
        if table.shape[1] > 65536:
            raise ValueError("page table width must not exceed 65536")
        self.max_context = int(lengths.max(initial=0))
        if self.max_context > 1048576:
            raise ValueError("this implementation supports at most 1M context tokens")
        self.splits = max(1, math.ceil(self.max_context / split_tokens))
        if self.splits > 65535:
            raise ValueError("too many context splits")
        self.layout, self.split_tokens = layout, split_tokens
        self.merge = merge
        self.merge_implementation = (("shared" if self.splits * 4 <= 4096 else "serial_fallback")
                                     if merge == "shared" else "serial")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DecodePlan requires a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._table_cpu, self._lengths_cpu = table, lengths
        self._lib = _native.load()
        # one native plan per input dtype (page tiles are sized per dtype), in one
        # buffer: [FP16 metadata][FP32 metadata][shared split-K workspace]
        self._native = {code: _NativePlan(self._lib, layout, table, lengths, split_tokens, merge, code,
                                          self.device, num_ctas, max_lengths)
                        for code in (_native.PD_FLOAT16, _native.PD_FLOAT32)}
        metas = [_align256(n.metadata_bytes) for n in self._native.values()]
        ws = _align256(max(n.workspace_bytes for n in self._native.values()))
        self._buffer = torch.empty(max(sum(metas) + ws, 256), dtype=torch.uint8, device=self.device)
        base = self._buffer.data_ptr()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        offset = 0
        for plan, meta in zip(self._native.values(), metas):
            _native.check(self._lib.pd_plan_bind_split(plan.handle, base + offset, meta,
                                                       base + sum(metas) if ws else None, ws, stream), "bind")
            offset += meta
        self._out = torch.empty((layout.batch, layout.query_heads, layout.head_dim),
                                dtype=torch.float32, device=self.device)
        self.barrier = "plain"

    @classmethod
    def from_csr(cls, layout: Layout, indptr, indices, last_page_len, **kwargs):
        """A plan from CSR paged metadata (FlashInfer's indptr / indices /
        last_page_len form, see ``competitors.csr_to_table``)."""
        from .competitors import csr_to_table
        table, lengths = csr_to_table(layout, indptr, indices, last_page_len)
        return cls(layout, table, lengths, **kwargs)

    @property
    def info(self):
        """pd_plan_info of the FP16 plan (see ``native_info`` for FP32)."""
        return self._native[_native.PD_FLOAT16].info

    def native_info(self, dtype):
        import torch
        return self._native[_native.PD_FLOAT16 if dtype == torch.float16 else _native.PD_FLOAT32].info

    @property
    def workspace_bytes(self):
        """Bytes of split-K workspace one run uses: the partial outputs o
        (FP32 [slots, HG, GT, D]) and their (m, l) pairs, which the FP16 and
        FP32 plans share (the larger of the two)."""
        return max(int(n.info.workspace_bytes) for n in self._native.values())

    @property
    def device_bytes(self):
        """Device bytes the plan holds: both dtypes' metadata and the shared workspace."""
        return int(self._buffer.numel())

    @property
    def num_ctas(self):
        return int(self.info.num_ctas)

    def kernels_per_run(self, dtype=None):
        """CUDA kernels one ``run`` launches: the decode kernel, plus the dependent
        merge kernel when some (sequence, KV-head group) was split or sub-pipelined
        and the decode CTAs do not merge the partials themselves."""
        import torch
        info = self.native_info(dtype if dtype is not None else torch.float16)
        return 1 + int(info.num_pieces > 0 and not info.merge_in_kernel)

    def _check_inputs(self, q, k, v):
        import torch
        layout = self.layout
        expected_q = (layout.batch, layout.query_heads, layout.head_dim)
        expected_k = (layout.physical_pages, layout.page_size, layout.kv_heads, layout.head_dim)
        if tuple(q.shape) != expected_q or tuple(k.shape) != expected_k or tuple(v.shape) != expected_k:
            raise ValueError("input shape does not match plan")
        if q.dtype not in (torch.float16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
            raise TypeError("q/k/v must share float16 or float32 dtype")
        for tensor in (q, k, v):
            if tensor.device != self.device or not tensor.is_contiguous():
                raise ValueError("inputs must be contiguous on the plan device")
            if tensor.requires_grad:
                raise ValueError("inference only: detach tensors requiring gradients")
        return _native.PD_FLOAT16 if q.dtype == torch.float16 else _native.PD_FLOAT32

    def run(self, q, k, v, out=None):
        """Decode one step; returns the plan's borrowed FP32 [B, Hq, D] output, or
        writes into ``out`` (extension: a contiguous FP32 [B, Hq, D] tensor on the
        plan device) and returns it."""
        import torch
        dtype = self._check_inputs(q, k, v)
        if out is None:
            out = self._out
        elif (tuple(out.shape) != tuple(self._out.shape) or out.dtype != torch.float32 or
              out.device != self.device or not out.is_contiguous()):
            raise ValueError("out must be a contiguous FP32 [B,Hq,D] tensor on the plan device")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.check(self._lib.pd_decode(self._native[dtype].handle, q.data_ptr(), k.data_ptr(),
                                          v.data_ptr(), dtype, out.data_ptr(), stream), "decode")
        return out

    def run_with_stats(self, q, k, v, out, stats):
        """Decode into caller buffers: out FP32 [B,Hq,D] and stats FP32 [B,Hq,2] = (m, l).

        m is the maximum of score*log2(e)/sqrt(D) and l the softmax
        denominator relative to it (-inf, 0 for an empty sequence); sequence
        sharding merges such results across GPUs.
        """
        import torch
        dtype = self._check_inputs(q, k, v)
        layout = self.layout
        rows = (layout.batch, layout.query_heads)
        for t, tail in ((out, (layout.head_dim,)), (stats, (2,))):
            if tuple(t.shape) != rows + tail or t.dtype != torch.float32 or \
                    t.device != self.device or not t.is_contiguous():
                raise ValueError("out/stats must be contiguous FP32 [B,Hq,D] / [B,Hq,2] on the plan device")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.check(self._lib.pd_decode_with_stats(
            self._native[dtype].handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), dtype, out.data_ptr(),
            stats.data_ptr(), stream), "decode")
        return out, stats

    def run_dynamic(self, q, k, v, table, lengths, out=None, stats=None):
        """Decode with live metadata in device memory (plans built with ``max_lengths``).

        ``table`` int32 [B, W] (this plan's width) and ``lengths`` int32 [B] are
        CUDA tensors read when the kernel runs, so a decode loop can append
        tokens and pages on the device, inside a CUDA graph, without a new
        plan.  Lengths above ``max_lengths`` are clamped and flag
        PD_DEVERR_LENGTH (``read_errors``).  Returns ``out`` (default: the
        plan's borrowed output).
        """
        import torch
        if self.max_lengths is None:
            raise ValueError("run_dynamic needs a plan built with max_lengths")
        dtype = self._check_inputs(q, k, v)
        layout = self.layout
        width = self._table_cpu.shape[1]
        for t, shape in ((table, (layout.batch, width)), (lengths, (layout.batch,))):
            if not isinstance(t, torch.Tensor) or t.dtype != torch.int32 or tuple(t.shape) != shape or \
                    t.device != self.device or not t.is_contiguous():
                raise ValueError("table/lengths must be contiguous int32 CUDA tensors of shape "
                                 "[batch, table width] / [batch] on the plan device")
        out = self._out if out is None else out
        rows = (layout.batch, layout.query_heads)
        if tuple(out.shape) != rows + (layout.head_dim,) or out.dtype != torch.float32 or \
                out.device != self.device or not out.is_contiguous():
            raise ValueError("out must be contiguous FP32 [B,Hq,D] on the plan device")
        if stats is not None and (tuple(stats.shape) != rows + (2,) or stats.dtype != torch.float32 or
                                  stats.device != self.device or not stats.is_contiguous()):
            raise ValueError("stats must be contiguous FP32 [B,Hq,2] on the plan device")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.check(self._lib.pd_decode_dynamic(
            self._native[dtype].handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), dtype,
            table.data_ptr(), lengths.data_ptr(), out.data_ptr(),
            None if stats is None else stats.data_ptr(), stream), "decode")
        return out

    def gather(self, k, v):
        """Debug: the live K/V rows of every (sequence, KV head) through the kernel's TMA path.

        Returns dense [B, Hkv, max_context (max(max_lengths) for a dynamic plan), D]
        tensors in the cache dtype; rows
        past a sequence's length are zero.
        """
        import torch
        layout = self.layout
        q_stub = torch.empty((layout.batch, layout.query_heads, layout.head_dim), dtype=k.dtype,
                             device=self.device)
        dtype = self._check_inputs(q_stub, k, v)
        span = int(self.max_lengths.max(initial=0)) if self.max_lengths is not None else self.max_context
        shape = (layout.batch, layout.kv_heads, max(span, 1), layout.head_dim)
        dense_k = torch.zeros(shape, dtype=k.dtype, device=self.device)
        dense_v = torch.zeros(shape, dtype=k.dtype, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.check(self._lib.pd_gather_debug(self._native[dtype].handle, k.data_ptr(), v.data_ptr(),
                                                dtype, dense_k.data_ptr(), dense_v.data_ptr(), stream),
                      "gather")
        return dense_k, dense_v

    def set_barrier(self, mode):
        """How the grid barrier before the in-kernel merge is launched (extension;
        see pd_plan_set_barrier): "plain" (default: a plain launch whose CTAs
        leave the barrier when another CTA has not started, the last one then
        merging for them), "cooperative" (all CTAs resident, or the merge
        kernel), or "leave_at_once" (every waiting CTA leaves; tests the fallback)."""
        codes = {"plain": _native.PD_BARRIER_PLAIN, "cooperative": _native.PD_BARRIER_COOPERATIVE,
                 "leave_at_once": _native.PD_BARRIER_LEAVE_AT_ONCE}
        if mode not in codes:
            raise ValueError(f"barrier mode must be one of {sorted(codes)}")
        for plan in self._native.values():
            _native.check(self._lib.pd_plan_set_barrier(plan.handle, codes[mode]))
        self.barrier = mode

    def read_barrier_fallbacks(self):
        """Return and clear the number of launches whose grid barrier fell back to
        merging for CTAs that left (synchronises the current stream)."""
        import torch
        stream = torch.cuda.current_stream(self.device).cuda_stream
        total = 0
        for plan in self._native.values():
            count = ctypes.c_uint32(0)
            _native.check(self._lib.pd_plan_read_barrier_fallbacks(plan.handle, ctypes.byref(count), stream))
            total += int(count.value)
        return total

    def read_errors(self):
        """Return and clear the device error words (synchronises the current stream)."""
        import torch
        stream = torch.cuda.current_stream(self.device).cuda_stream
        total = 0
        for plan in self._native.values():
            word = ctypes.c_uint32(0)
            _native.check(self._lib.pd_plan_read_errors(plan.handle, ctypes.byref(word), stream))
            total |= int(word.value)
        return total

    def worklist(self, dtype=None):
        """(segments, groups, cta_offsets) of the FP16 (or given dtype's) plan, see ``inspect_plan``."""
        import torch
        plan = self._native[_native.PD_FLOAT32 if dtype == torch.float32 else _native.PD_FLOAT16]
        return plan.segments.copy(), plan.groups.copy(), plan.cta_offsets.copy()

    def split_bounds(self, b):
        """The reference's context partitions of sequence b: range(0, max(len,1), split_tokens)."""
        length = int(self._lengths_cpu[b])
        return [(s, min(s + self.split_tokens, length))
                for s in range(0, max(length, 1), self.split_tokens)]
