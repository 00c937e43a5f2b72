#!/usr/bin/env python3
"""Decode-attention benchmark: achieved HBM TB/s and µs per decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3a|c3b|c3c|c4|c5] [--no-cpu-baseline]

One step = one DecodePlan.run over one batch: every live K/V row of every
sequence is read once per KV head.  Default workload
(B32 ragged lengths 0..8192 with a shared 64-page prefix, 32:8 heads, D128,
FP16, page 16, split 256), seeded synthetic data.

N > 1 (torchrun, one rank per GPU, NCCL): by default KV-head sharding with
weak scaling.  Every rank serves the same sequences (same page tables and
lengths) for its own 8 KV heads and their 32 query heads, i.e. rank r owns KV
heads [8r, 8r+8) of an 8N-KV-head model; there is no data-path collective.
--scaling strong splits the chosen config itself: KV heads across ranks, or
(c5, --sharding sequence) contiguous page runs of every sequence with an NCCL
all-gather of (o, m, l) and a merge.  value = all ranks' algorithmic bytes /
max-over-ranks step time.

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
synchronize, device time from CUDA events on the launching stream; each step
is also timed alone for the kernel's average duration (roofline).  Inputs are
larger than L2 for config 2; smaller workloads flush L2 between steps.
e2e: the same step through the public API with host buffers: q copied from
pinned host memory, decode, FP32 output copied back, every step.

--impl reference: the reference's CPU path (FP64 dense attention, our C port
of src/paged_decode/oracle.py:59-71, all host threads) on a bounded sample of
the same workload, plus the reference's own CUDA kernel (built from its
sources for sm_100a) on the same inputs as an extra field.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "paged-decode-lab_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn µs/step + achieved HBM TB/s vs ~8 TB/s peak at 1/2/4/8 B200"
L2_BYTES = 126 * 2**20
DEFAULT_STEPS, DEFAULT_WARMUP = 200, 5
GRAPH_STEPS = 50            # default e2e steps per captured CUDA graph (one GPU; --graph-steps)

# dram__bytes_read.sum + dram__bytes_write.sum of one decode-kernel launch (the
# 4th of `bench.py --workload W --steps 1 --warmup 3`), one ncu capture per
# workload; config 4 (4.8 GB resident) was not captured.
NCU_TRAFFIC_BYTES = {"c1": 67_258_880 + 571_648, "c2": 469_731_072 + 5_400_320,
                     "c3a": 2_150_068_480 + 7_169_792, "c3b": 67_789_056 + 1_476_096,
                     "c3c": 540_718_336 + 4_886_528, "c5": 1_073_953_792 + 3_577_344}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=DEFAULT_STEPS)
    ap.add_argument("--warmup", type=int, default=DEFAULT_WARMUP)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3a", "c3b", "c3c", "c4", "c5"])
    ap.add_argument("--graph-steps", type=int, default=GRAPH_STEPS,
                    help="e2e decode steps (with their copies) per captured CUDA graph on one GPU")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N > 1: weak = KV-head shards of an N x larger model; strong = split this config")
    ap.add_argument("--sharding", choices=["kv_head", "sequence"], default=None,
                    help="strong scaling split (default: sequence for c5, kv_head otherwise)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="sequence sharding: one kernel with NVLink peer stores, or NCCL all-gather + merge")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-competitors", action="store_true",
                    help="skip the FlashInfer decode timed on the same inputs (1 GPU only)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    return ap.parse_args()


# ---------------------------------------------------------------------- helpers
def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


_SAMPLER = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
while True:
    t = time.time()
    print(t, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
          pynvml.nvmlDeviceGetCurrentClocksEventReasons(h), flush=True)
    time.sleep(0.0005)
"""


class ClockSampler:
    """SM clock and throttle reasons sampled while the timed region runs.

    A child process polls NVML (the library nvidia-smi reads) every half
    millisecond, free of this process's GIL; `mark_start`/`mark_end` bracket
    the timed region in wall-clock time and only samples inside it count.
    """
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.t0 = self.t1 = None
        self.rows, self.max_mhz, self.window = [], None, None

    def _physical_index(self):
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        if visible:
            ids = [x.strip() for x in visible.split(",") if x.strip()]
            if self.device_index < len(ids) and ids[self.device_index].isdigit():
                return int(ids[self.device_index])
        return self.device_index

    def start(self):
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, str(self._physical_index())],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            first = self.proc.stdout.readline().split()   # "max <mhz>" once NVML is up
            self.max_mhz = int(first[1]) if len(first) == 2 else None
        except Exception:  # noqa: BLE001 - no NVML: reported as unsampled
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if not self.proc:
            return
        time.sleep(0.002)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        samples = []
        for line in out.splitlines():
            parts = line.split()
            if len(parts) == 3:
                samples.append((float(parts[0]), int(parts[1]), int(parts[2])))
        t0, t1 = self.t0 or 0.0, self.t1 or float("inf")
        self.rows = [(m, r) for t, m, r in samples if t0 <= t <= t1]
        self.window = "timed region"
        if not self.rows:
            # a very short timed region can fall between two polls: use the polls
            # just around it (the GPU runs the same steps back to back there too)
            self.rows = [(m, r) for t, m, r in samples if t0 - 0.05 <= t <= t1 + 0.05]
            self.window = "timed region +- 50 ms"

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted(n for n, bit in self.REASONS.items() if any(r & bit for _, r in self.rows))
        return {"sm_mhz": statistics.median(m for m, _ in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows), "source": "nvml, 0.5 ms",
                "window": self.window}


def algorithmic_bytes(w):
    """Unique live K/V rows of every KV head + q + FP32 out + live table entries."""
    import numpy as np
    L = w.layout
    elt = 2 if w.dtype == "float16" else 4
    slots = []
    entries = 0
    for b in range(L.batch):
        n = int(w.lengths[b])
        entries += -(-n // L.page_size)
        tok = np.arange(n, dtype=np.int64)
        slots.append(w.table[b][tok // L.page_size].astype(np.int64) * L.page_size + tok % L.page_size)
    unique = int(np.unique(np.concatenate(slots)).size) if slots else 0
    return (2 * unique * L.kv_heads * L.head_dim * elt
            + L.batch * L.query_heads * L.head_dim * (elt + 4) + entries * 4)


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        # NCCL may print its banner on stdout while the communicator comes up;
        # keep stdout for the one JSON result line by pointing fd 1 at stderr meanwhile.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    return rank, local, world


def max_over_ranks(value, world):
    import torch
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------- CPU baseline
def cpu_baseline(w, q, k, v, nbytes, budget_s, steps=None):
    """FP64 C port of the reference's dense_attention, all host threads, on the workload.

    Runs whole decode steps until ``budget_s`` seconds of CPU time have passed
    (or ``steps`` times); value = algorithmic bytes per step * steps / seconds.
    """
    from oracle import c_oracle
    threads = os.cpu_count() or 1
    qh, kh, vh = (t.cpu().numpy() for t in (q, k, v))
    done, t0 = 0, time.perf_counter()
    while True:
        c_oracle.dense_attention(qh, kh, vh, w.table, w.lengths, threads=threads)
        done += 1
        elapsed = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and elapsed >= budget_s):
            break
    return {"value": nbytes * done / elapsed / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
            "sample": f"{done} full decode step(s) of {w.name} in {elapsed:.2f} s "
                      f"(FP64 C restatement of oracle.dense_attention, {threads} threads)",
            "s_per_step": elapsed / done}


# ---------------------------------------------------------------------- our implementation
class RankJob:
    """What one rank decodes per step, and how the job's bytes are counted."""

    def __init__(self, args, rank, world):
        import torch
        from paged_decode import dist as pd_dist
        from paged_decode import workload
        from paged_decode.layout import Layout

        w = workload.CONFIGS[args.workload]()
        self.workload = w
        L = w.layout
        self.sharding = "none"
        self.bytes_total = algorithmic_bytes(w)
        self.extra_kernels = 0
        self.close = lambda: None
        self.run_into = lambda q, out: out.copy_(self.run(q))   # sharded plans return their own output
        if world == 1:
            from paged_decode.runtime import DecodePlan
            self.plan = DecodePlan(L, w.table, w.lengths, split_tokens=w.split_tokens)
            self.q, self.k, self.v = w.tensors("cuda")
            self.run = lambda q: self.plan.run(q, self.k, self.v)
            self.run_into = lambda q, out: self.plan.run(q, self.k, self.v, out=out)
            self.decode_plan = self.plan
            self.bytes_rank = self.bytes_total
            return
        mode = args.sharding or ("sequence" if args.workload == "c5" else "kv_head")
        if args.scaling == "weak":
            # KV-head sharding of a model with world x the config's KV heads: every rank
            # serves the same sequences for its own heads (same local geometry as config).
            glob = Layout(L.batch, L.query_heads * world, L.kv_heads * world, L.head_dim, L.page_size,
                          L.physical_pages)
            plan = pd_dist.KVHeadShardedPlan(glob, w.table, w.lengths, rank=rank, world=world,
                                             split_tokens=w.split_tokens)
            w.seed += rank
            self.q, self.k, self.v = w.tensors("cuda")
            self.run = lambda q: plan.run(q, self.k, self.v)
            self.decode_plan = plan.plan
            self.bytes_rank = self.bytes_total
            self.bytes_total *= world
            self.sharding = (f"kv_head, weak: rank r owns KV heads [{L.kv_heads}r, {L.kv_heads}r+{L.kv_heads}) "
                             f"of a {L.kv_heads * world}-KV-head model; same sequences on every rank; "
                             "no collective")
        elif mode == "kv_head":
            plan = pd_dist.KVHeadShardedPlan(L, w.table, w.lengths, rank=rank, world=world,
                                             split_tokens=w.split_tokens)
            loc = plan.local_layout
            local = workload.Workload(w.name, loc, w.table, w.lengths, w.split_tokens, dtype=w.dtype,
                                      std=w.std, seed=w.seed + rank)
            self.q, self.k, self.v = local.tensors("cuda")
            self.run = lambda q: plan.run(q, self.k, self.v)
            self.decode_plan = plan.plan
            self.bytes_rank = algorithmic_bytes(local)
            self.sharding = (f"kv_head, strong: rank r owns KV heads [{loc.kv_heads}r, {loc.kv_heads}(r+1)) "
                             "and their query heads; no collective")
        else:
            lt, ll, (lo, hi) = pd_dist.shard_sequence_metadata(w.table, w.lengths, L.page_size, rank, world)
            ltab, ids = pd_dist.localize_pages(lt, ll, L.page_size)
            loc = Layout(L.batch, L.query_heads, L.kv_heads, L.head_dim, L.page_size, max(1, len(ids)))
            local = workload.Workload(w.name, loc, ltab, ll, w.split_tokens, dtype=w.dtype, std=w.std,
                                      seed=w.seed + rank)
            plan = pd_dist.SequenceShardedPlan(loc, ltab, ll, split_tokens=w.split_tokens,
                                               exchange=args.exchange)
            self.q, self.k, self.v = local.tensors("cuda")
            self.run = lambda q: plan.run(q, self.k, self.v)
            self.close = plan.close
            self.decode_plan = plan.plan
            self.bytes_rank = algorithmic_bytes(local)
            self.nvlink_bytes = plan.nvlink_bytes_per_step
            if args.exchange == "peer":
                self.extra_kernels = -self.decode_plan.kernels_per_run(self.q.dtype) + 1   # one kernel a step
                how = (f"one kernel per rank: decode, NVLink peer stores of {pd_dist.packed_size(loc) * 4} B "
                       "into every rank's buffer, bounded wait for all ranks, max-corrected merge")
            else:
                self.extra_kernels = 1                  # the cross-shard merge (NCCL's own kernel not counted)
                how = f"NCCL all_gather of {pd_dist.packed_size(loc) * 4} B per rank + max-corrected merge"
            self.sharding = f"sequence, strong: rank r owns logical pages [{lo}, {hi}) of every sequence; {how}"

    def kernels_per_step(self):
        return self.decode_plan.kernels_per_run(self.q.dtype) + self.extra_kernels


def run_ours(args, rank, local, world):
    import torch

    job = RankJob(args, rank, world)
    w = job.workload
    q, k, v = job.q, job.k, job.v
    kv_bytes = 2 * k.numel() * k.element_size()
    flush = None
    if kv_bytes < 2 * L2_BYTES:
        # read-only flush: leaves L2 full of clean lines, so the decode never pays
        # for write-backs that a zero-fill flush would leave behind
        flush = torch.ones(2 * L2_BYTES // 2, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        return job.run(q)

    clocks = ClockSampler(local).start()
    for _ in range(max(args.warmup, 0)):
        step()
    barrier(world)

    # (1) K steps.  Inputs larger than L2 run back to back between one pair of
    # events (events between the steps would add their own gaps); smaller
    # inputs flush L2 before every step, and each step then has its own events
    # so that the flushes stay outside the timed time.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    clocks.mark_start()
    t_start.record(stream)
    for i in range(args.steps):
        if flush is not None:
            flush.amax()
            starts[i].record(stream)
        step()
        if flush is not None:
            ends[i].record(stream)
    t_end.record(stream)
    barrier(world)
    clocks.mark_end()
    clocks.stop()
    if flush is not None:
        launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        total_ms = sum(launch_ms)
    else:
        total_ms = t_start.elapsed_time(t_end)
    step_ms = max_over_ranks(total_ms / args.steps, world)
    # the step's kernels (decode, plus the merge kernel when it is separate) per launch
    kernel_ms = total_ms / args.steps
    errors = job.decode_plan.read_errors()
    if errors:
        raise SystemExit(f"device error word {errors:#x}")

    # (2) e2e through the public API with host buffers.  Every step copies its q
    # from pinned host memory and its FP32 output back; the two directions run
    # on their own streams, double-buffered, so step i+1's input and step i-1's
    # output move while step i decodes (on one GPU the decode writes straight
    # into the staging buffer the output is copied back from).  On
    # one GPU, --graph-steps such steps (their copies included) are captured once
    # through the same public calls and replayed, so the host's per-call
    # overhead does not set the pace.
    e2e = None
    if not args.no_e2e:
        copy = torch.cuda.Stream()       # device -> host
        upload = torch.cuda.Stream()     # host -> device
        q_host = [q.cpu().pin_memory() for _ in range(2)]
        out_shape = step().shape
        out_host = [torch.empty(out_shape, dtype=torch.float32).pin_memory() for _ in range(2)]
        q_dev = [torch.empty_like(q) for _ in range(2)]
        stage = [torch.empty(out_shape, dtype=torch.float32, device=q.device) for _ in range(2)]
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        computed = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]

        def e2e_step(i, main, fresh=False):
            # fresh: the first two steps of a capture, whose buffers no earlier step in it used
            b = i % 2
            with torch.cuda.stream(upload):
                if not fresh:
                    upload.wait_event(computed[b])    # q_dev[b] no longer read by step i-2
                q_dev[b].copy_(q_host[b], non_blocking=True)
                h2d_done[b].record(upload)
            main.wait_event(h2d_done[b])
            if not fresh:
                main.wait_event(d2h_done[b])          # stage[b] drained by step i-2's copy
            job.run_into(q_dev[b], stage[b])
            computed[b].record(main)
            with torch.cuda.stream(copy):
                copy.wait_event(computed[b])
                out_host[b].copy_(stage[b], non_blocking=True)
                d2h_done[b].record(copy)

        for i in range(max(args.warmup, 2)):
            e2e_step(i, stream)
        torch.cuda.synchronize()
        graph, reps = None, args.steps
        if world == 1:
            graph = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(stream)
            with torch.cuda.graph(graph, stream=cap):
                copy.wait_stream(cap)
                upload.wait_stream(cap)
                for i in range(args.graph_steps):
                    if flush is not None:
                        flush.amax()
                    e2e_step(i, cap, fresh=i < 2)
                cap.wait_stream(copy)
                cap.wait_stream(upload)
            reps = -(-args.steps // args.graph_steps)
            graph.replay()
            torch.cuda.synchronize()
        timed = reps * args.graph_steps if graph is not None else args.steps
        barrier(world)
        t0 = time.perf_counter()
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if graph is not None:
            for _ in range(reps):
                graph.replay()
        else:
            for i in range(args.steps):
                if flush is not None:
                    flush.amax()
                e2e_step(i, stream)
        stream.wait_stream(copy)
        stream.wait_stream(upload)
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / timed
        if flush is not None:                     # take out the flushes' own time
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(timed):
                flush.amax()
            f1.record(stream)
            torch.cuda.synchronize()
            e2e_ms -= f0.elapsed_time(f1) / timed
        del graph
        e2e_ms = max_over_ranks(e2e_ms, world)
        e2e = {"value": job.bytes_total / (e2e_ms * 1e-3) / 1e12, "unit": "TB/s",
               "us_per_step": e2e_ms * 1e3,
               "h2d_bytes_per_step": q.numel() * q.element_size(),
               "d2h_bytes_per_step": out_host[0].numel() * 4,
               "wall_s": time.perf_counter() - t0,
               "steps": timed,
               "path": ("public API run() (ctypes -> C ABI pd_decode"
                        + (", out= the staging buffer" if world == 1 else "")
                        + "); pinned host q in and FP32 out back "
                        "every step, each direction on its own stream, double-buffered"
                        + (f"; {args.graph_steps} steps captured once as a CUDA graph and replayed"
                           if world == 1 else ""))}

    peak, peak_kind = measured_peak()
    achieved = job.bytes_rank / (kernel_ms * 1e-3) / 1e9
    traffic = NCU_TRAFFIC_BYTES.get(args.workload) if world == 1 else None
    info = job.decode_plan.native_info(q.dtype)
    line = {
        "metric": METRIC,
        "value": job.bytes_total / (step_ms * 1e-3) / 1e12,
        "unit": "TB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "us_per_step": step_ms * 1e3,
        "higher_is_better": True,
        "scaling": "weak" if (world == 1 or args.scaling == "weak") else "strong",
        "vs_baseline": None,
        "dtype": "f16" if w.dtype == "float16" else "f32",
        "data": "synthetic: seeded N(0,1) tensors, BASELINE config generators (no dataset exists)",
        "config": {"workload": w.name, "batch": w.layout.batch, "query_heads": w.layout.query_heads,
                   "kv_heads": w.layout.kv_heads, "head_dim": w.layout.head_dim,
                   "page_size": w.layout.page_size, "split_tokens": w.split_tokens,
                   "bytes_per_step_total": job.bytes_total, "bytes_per_step_rank": job.bytes_rank,
                   "sharding": job.sharding,
                   "l2": ("inputs larger than L2" if flush is None else "L2 flushed (read-only) between steps"),
                   "persistent_ctas": int(info.num_ctas),
                   "kv_heads_per_tile": int(info.heads_per_tile)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic,
                     "kernel": "paged_decode_kernel" + ("" if job.kernels_per_step() == 1
                                                        else " (+ merge_partials_kernel)"),
                     "kernel_us": kernel_ms * 1e3,
                     "algorithmic_bytes_per_launch": job.bytes_rank},
        "gpu_launches": args.steps * job.kernels_per_step(),
        "clocks": clocks.summary(),
    }
    if hasattr(job, "nvlink_bytes"):
        line["nvlink_bytes_per_step_per_gpu"] = job.nvlink_bytes
    if e2e:
        line["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, q, k, v, job.bytes_total, args.cpu_seconds)
    if world == 1 and not args.no_competitors:
        line["competitors"] = competitors(w, q, k, v, job, flush, args.steps)
    job.close()
    return line


def competitors(w, q, k, v, job, flush, steps):
    """The reference's comparisons on the same caches, timed like our step.

    FlashInfer's batch decode (FP16 only; empty rows get one token because it
    needs nonempty contexts, so its workload is that much larger, never
    smaller) with and without its tensor-core path, and the dense baseline:
    gather the pages into padded dense K/V and run PyTorch SDPA.
    """
    import torch
    from paged_decode.competitors import DenseSDPAPlan, FlashInferPlan
    table, lengths = w.table.copy(), w.lengths.copy()
    table[lengths == 0, 0] = 0
    lengths[lengths == 0] = 1
    out = {}
    ours = job.decode_plan.run(q, k, v).clone()
    live = torch.as_tensor(w.lengths > 0, device=q.device)   # rows the comparisons all define alike
    entries = [("dense_gather_sdpa", lambda: DenseSDPAPlan(w.layout, w.table, w.lengths, device=q.device))]
    if w.dtype == "float16":
        entries += [("flashinfer", lambda: FlashInferPlan(w.layout, table, lengths, device=q.device)),
                    ("flashinfer_tensor_cores",
                     lambda: FlashInferPlan(w.layout, table, lengths, device=q.device, tensor_cores=True))]
    for key, make in entries:
        try:
            fi = make()
            for _ in range(3):
                fi.run(q, k, v)
            torch.cuda.synchronize()
            if flush is None:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(steps):
                    fi.run(q, k, v)
                b.record()
                torch.cuda.synchronize()
                ms = a.elapsed_time(b) / steps
            else:
                times = []
                for _ in range(steps):
                    flush.amax()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    fi.run(q, k, v)
                    b.record()
                    torch.cuda.synchronize()
                    times.append(a.elapsed_time(b))
                ms = sum(times) / steps
            result = fi.run(q, k, v)
            torch.cuda.synchronize()
            out[key] = {"version": getattr(fi, "version", torch.__version__), "us_per_step": ms * 1e3,
                        "value": job.bytes_total / (ms * 1e-3) / 1e12, "unit": "TB/s",
                        "max_abs_vs_ours": float((result.float() - ours)[live].abs().max()),
                        "timing": "same as value (back to back, or L2 flushed per step)"}
            del fi
        except Exception as exc:  # noqa: BLE001 - reported, never fatal
            out[key] = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    return out


# ---------------------------------------------------------------------- reference arm
def run_reference(args, rank, local, world):
    import torch
    from paged_decode import workload

    if rank != 0:
        return None
    w = workload.CONFIGS[args.workload]()
    q, k, v = w.tensors("cuda")
    nbytes = algorithmic_bytes(w)
    samples = []
    t0 = time.perf_counter()
    for _ in range(max(args.warmup, 0)):
        cpu_baseline(w, q, k, v, nbytes, 0, steps=1)
    for _ in range(args.steps):
        samples.append(cpu_baseline(w, q, k, v, nbytes, 0, steps=1))
    s_per_step = statistics.mean(s["s_per_step"] for s in samples)
    value = nbytes / s_per_step / 1e12
    base = samples[0]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": s_per_step * 1e3,
        "us_per_step": s_per_step * 1e6, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: seeded N(0,1) tensors, BASELINE config generators (no dataset exists)",
        "config": {"workload": w.name, "bytes_per_step_per_gpu": nbytes},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": base["cores"], "kind": "port",
                         "sample": f"{args.steps} timed full decode steps of {w.name} (FP64 C restatement "
                                   f"of the reference oracle.dense_attention, {base['cores']} threads)"},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0,
    }
    # The reference's own CUDA kernel on this B200 (built from its sources), same inputs.
    try:
        from oracle import ref_kernel
        if ref_kernel.SO_PATH.exists():
            ref = {}
            for merge in ("serial", "shared"):
                plan = ref_kernel.RefPlan(w.layout, w.table, w.lengths, device=q.device,
                                          split_tokens=w.split_tokens, merge=merge)
                for _ in range(3):
                    plan.run(q, k, v)
                torch.cuda.synchronize()
                times = []
                for _ in range(10):
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    plan.run(q, k, v)
                    e.record()
                    e.synchronize()
                    times.append(s.elapsed_time(e))
                ms = statistics.median(times)
                ref[merge] = {"us_per_step": ms * 1e3, "TB/s": nbytes / (ms * 1e-3) / 1e12}
            line["ref_cuda_b200"] = ref
    except Exception as exc:  # noqa: BLE001 - reported, not fatal: the CPU arm is the line's value
        line["ref_cuda_b200"] = {"unavailable": f"{type(exc).__name__}: {exc}"}
    return line


def main():
    args = parse_args()
    if args.steps < 1 or args.warmup < 0:
        raise SystemExit("--steps >= 1 and --warmup >= 0 required")
    if args.impl == "reference" and int(os.environ.get("RANK", "0")) != 0:
        return                      # the reference arm runs on rank 0 only
    if args.impl == "reference":
        os.environ["WORLD_SIZE"] = "1"
        args.gpus = 1
    rank, local, world = dist_setup(args)
    try:
        line = (run_reference if args.impl == "reference" else run_ours)(args, rank, local, world)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
