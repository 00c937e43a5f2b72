#!/usr/bin/env python3
"""Decode-attention benchmark: µs per decode step and achieved HBM TB/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3a|c3b|c3c|c4|c5] [--windows R]
                    [--scaling strong|weak] [--sharding kv_head|sequence]

One step = one decode of one batch: every live K/V row of every sequence is
read once per KV head.  Default workload: BASELINE config 4 (B256, Llama-3-70B
heads 64:8, D128, FP16 N(0, 0.5), page 16, lengths uniform in [1024, 8192],
pages a random permutation of the pool), seeded synthetic data.

N > 1 (torchrun, one rank per GPU): strong scaling of the chosen config.  KV
heads are split across ranks (config 4: 8/4/2/1 KV heads per GPU with their
8-query-head groups, no collective); config 5 splits every sequence into
contiguous page runs, and the ranks' (o, m, l) rows are merged over NVLink
(one kernel per rank with peer stores, or --exchange nccl: all-gather +
merge).  Every rank draws the full config's tensors from the same seed and
keeps its shard.  --scaling weak instead gives every rank its own copy of the
config (an N-times larger model).  value = all ranks' algorithmic bytes /
max-over-ranks step time.

Timing (the reference's protocol, docs/BENCHMARKING.md:49-53, with graph
replay): W untimed warm-up steps; K steps captured once as a CUDA graph
through the public DecodePlan.run; R timed windows, each one replay of the K
steps between CUDA events on the launching stream, all R bracketed by barrier
+ synchronize.  Window means give median (the reported step time), min and
interpolated p95; max over ranks per window.  Inputs larger than L2 run as
they are; smaller ones rotate over enough identical K/V copies that each step
reads a copy the previous steps left out of L2.  Sequence sharding runs the
K steps eagerly (its exchange kernel is a cooperative launch).

Gate (the cpu_baseline leg): the FP64 C oracle on the same tensors checks the
timed output (FP16 max-abs 2e-3 / rel 1e-3, FP32 1e-5); a failure exits 1.
e2e: the same steps through the public API with host buffers: q copied from
pinned host memory, decode, FP32 output copied back, every step.

--impl reference: the reference's CPU path (FP64 dense attention, our C port
of src/paged_decode/oracle.py:59-71, all host threads) on a bounded sample of
the same workload's sequences, plus the reference's own CUDA kernel (built
from its sources for sm_100a) on the full workload as an extra field.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
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
DEFAULT_STEPS, DEFAULT_WARMUP, DEFAULT_WINDOWS = 200, 5, 10
GRAPH_STEPS = 50            # default e2e steps per captured CUDA graph (one GPU; --graph-steps)
TOL = {"float16": (2e-3, 1e-3), "float32": (1e-5, 1e-5)}   # BASELINE gate (atol, rtol)

# dram__bytes_read.sum + dram__bytes_write.sum of one decode-kernel launch (the
# 4th of `bench.py --workload W --steps 1 --warmup 3`), one ncu capture per
# workload.  Config 4 (4.8 GB resident) is captured as its 32-sequence subset
# "c4s" and scaled by the ratio of algorithmic bytes (see NCU_SCALED).
NCU_TRAFFIC_BYTES = {"c1": 67_258_880 + 571_648, "c2": 469_731_072 + 5_400_320,
                     "c3a": 2_150_068_480 + 7_169_792, "c3b": 67_789_056 + 1_476_096,
                     "c3c": 540_718_336 + 4_886_528, "c5": 1_073_953_792 + 3_577_344}
NCU_TRAFFIC_BYTES["c4s"] = 580_584_448 + 4_443_648
NCU_SCALED = {"c4": ("c4s", NCU_TRAFFIC_BYTES["c4s"])}   # workload -> (captured workload, its traffic)
# the same for plans on the tcgen05 kernel (paged_decode_mqa_kernel)
NCU_TRAFFIC_BYTES_TCGEN05 = {"c3b": 67_764_736 + 709_120}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=DEFAULT_STEPS)
    ap.add_argument("--warmup", type=int, default=DEFAULT_WARMUP)
    ap.add_argument("--windows", type=int, default=DEFAULT_WINDOWS,
                    help="timed windows of --steps steps each (median / min / p95 over windows)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c4", choices=["c1", "c2", "c3a", "c3b", "c3c", "c4", "c4s", "c5"])
    ap.add_argument("--graph-steps", type=int, default=GRAPH_STEPS,
                    help="e2e decode steps (with their copies) per captured CUDA graph on one GPU")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong",
                    help="N > 1: strong = split this config across ranks; weak = a copy per rank")
    ap.add_argument("--sharding", choices=["kv_head", "sequence"], default=None,
                    help="strong scaling split (default: sequence for c5, kv_head otherwise)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="sequence sharding: one kernel with NVLink peer stores, or NCCL all-gather + merge")
    ap.add_argument("--timing", choices=["graph", "eager"], default=None,
                    help="how the K steps of a window are launched (default: graph, eager for sequence sharding)")
    ap.add_argument("--l2", choices=["rotate", "flush"], default="rotate",
                    help="inputs smaller than L2: rotate over K/V copies (default) or flush L2 before each step")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the oracle timing and the gate")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-competitors", action="store_true",
                    help="skip FlashInfer / dense SDPA timed on the same inputs (1 GPU only)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    return ap.parse_args()


# ---------------------------------------------------------------------- helpers
def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def percentile(xs, p):
    """Linearly interpolated percentile (numpy's default method)."""
    xs = sorted(xs)
    pos = (len(xs) - 1) * p / 100.0
    lo = int(math.floor(pos))
    hi = min(lo + 1, len(xs) - 1)
    return xs[lo] + (xs[hi] - xs[lo]) * (pos - lo)


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


def max_over_ranks(values, world):
    """Element-wise maximum over ranks of a list of floats (a float for a float)."""
    import torch
    scalar = not isinstance(values, (list, tuple))
    vals = [values] if scalar else list(values)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor(vals, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.tolist()
    return vals[0] if scalar else vals


def all_ranks_ok(ok, world):
    import torch
    if world == 1:
        return ok
    import torch.distributed as dist
    t = torch.tensor([0 if ok else 1], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t.item()) == 0


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------- CPU baseline leg
def cpu_baseline(w, q, k, v, nbytes, budget_s, steps=None, threads=None):
    """FP64 C port of the reference's dense_attention, all host threads, on the workload.

    Runs whole decode steps until ``budget_s`` seconds of CPU time have passed
    (or ``steps`` times); value = algorithmic bytes per step * steps / seconds.
    Returns the summary and the oracle's output of the last step.
    """
    from oracle import c_oracle
    threads = threads or os.cpu_count() or 1
    qh, kh, vh = (t.cpu().numpy() if hasattr(t, "cpu") else t for t in (q, k, v))
    done, t0 = 0, time.perf_counter()
    while True:
        ref = c_oracle.dense_attention(qh, kh, vh, w.table, w.lengths, threads=threads)
        done += 1
        elapsed = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and elapsed >= budget_s):
            break
    return {"value": nbytes * done / elapsed / 1e12, "unit": "TB/s", "cores": threads, "kind": "port",
            "sample": f"{done} full decode step(s) of {w.name} in {elapsed:.2f} s "
                      f"(FP64 C restatement of oracle.dense_attention, {threads} threads)",
            "s_per_step": elapsed / done}, ref


def gate(out, ref, dtype):
    """The BASELINE tolerance applied as assert_allclose(atol, rtol); returns the record."""
    import numpy as np
    atol, rtol = TOL[dtype]
    got = out.cpu().numpy().astype(np.float64)
    err = np.abs(got - ref)
    ok = bool(np.all(err <= atol + rtol * np.abs(ref)) and np.isfinite(got).all())
    return {"max_abs": float(err.max(initial=0.0)), "atol": atol, "rtol": rtol,
            "oracle": "FP64 C restatement of oracle.dense_attention", "gate": "pass" if ok else "fail"}


# ---------------------------------------------------------------------- our implementation
class RankJob:
    """What one rank decodes per step, and how the job's bytes are counted.

    ``step(i, out=None)`` launches step i (K/V copy i % copies); ``check``
    holds (workload, q, k, v) on the host-facing side of the gate for the
    output this rank produces, or None when another rank checks it.
    """

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
        self.graphable = True
        self.check = None
        if world == 1:
            from paged_decode.runtime import DecodePlan
            plan = DecodePlan(L, w.table, w.lengths, split_tokens=w.split_tokens)
            self.q, k, v = w.tensors("cuda")
            self._run = lambda q, k, v, out: plan.run(q, k, v, out=out)
            self.decode_plan = plan
            self.bytes_rank = self.bytes_total
            self.check = (w, self.q, k, v)
        elif args.scaling == "weak":
            # every rank serves its own copy of the config (an N-times larger model)
            glob = Layout(L.batch, L.query_heads * world, L.kv_heads * world, L.head_dim, L.page_size,
                          L.physical_pages)
            plan = pd_dist.KVHeadShardedPlan(glob, w.table, w.lengths, rank=rank, world=world,
                                             split_tokens=w.split_tokens)
            w.seed += rank
            self.q, k, v = w.tensors("cuda")
            self._run = lambda q, k, v, out: plan.plan.run(q, k, v, out=out)
            self.decode_plan = plan.plan
            self.bytes_rank = self.bytes_total
            self.bytes_total *= world
            self.check = (w, self.q, k, v)
            self.sharding = (f"kv_head, weak: rank r owns KV heads [{L.kv_heads}r, {L.kv_heads}r+{L.kv_heads}) "
                             f"of a {L.kv_heads * world}-KV-head model; same sequences on every rank; "
                             "no collective")
        elif (args.sharding or ("sequence" if args.workload == "c5" else "kv_head")) == "kv_head":
            plan = pd_dist.KVHeadShardedPlan(L, w.table, w.lengths, rank=rank, world=world,
                                             split_tokens=w.split_tokens)
            loc = plan.local_layout
            qf, kf, vf = w.tensors("cuda")          # the full config, same seed on every rank
            self.q, k, v = pd_dist.shard_kv_heads(L, qf, kf, vf, rank, world)
            del qf, kf, vf
            torch.cuda.empty_cache()
            local = workload.Workload(w.name, loc, w.table, w.lengths, w.split_tokens, dtype=w.dtype,
                                      std=w.std, seed=w.seed)
            self._run = lambda q, k, v, out: plan.plan.run(q, k, v, out=out)
            self.decode_plan = plan.plan
            self.bytes_rank = algorithmic_bytes(local)
            self.check = (local, self.q, k, v)
            self.sharding = (f"kv_head, strong: rank r owns KV heads [{loc.kv_heads}r, {loc.kv_heads}(r+1)) "
                             f"and their {loc.query_heads} query heads of the config; no collective")
        else:
            lt, ll, (lo, hi) = pd_dist.shard_sequence_metadata(w.table, w.lengths, L.page_size, rank, world)
            ltab, ids = pd_dist.localize_pages(lt, ll, L.page_size)
            loc = Layout(L.batch, L.query_heads, L.kv_heads, L.head_dim, L.page_size, max(1, len(ids)))
            local = workload.Workload(w.name, loc, ltab, ll, w.split_tokens, dtype=w.dtype, std=w.std,
                                      seed=w.seed)
            plan = pd_dist.SequenceShardedPlan(loc, ltab, ll, split_tokens=w.split_tokens,
                                               exchange=args.exchange)
            qf, kf, vf = w.tensors("cuda")          # the full config, same seed on every rank
            index = torch.as_tensor(ids if len(ids) else [0], device=kf.device)
            self.q = qf
            k, v = kf.index_select(0, index).contiguous(), vf.index_select(0, index).contiguous()
            if rank == 0:
                self.check = (w, qf, kf, vf)      # the merged output is the whole config's
            else:
                del kf, vf
            torch.cuda.empty_cache()
            # the plan writes its merged output into its own buffer (self.out below)
            self._run = lambda q, k, v, out: (plan.run(q, k, v) if out is plan._out
                                              else out.copy_(plan.run(q, k, v)))
            self.out = plan._out
            self.close = plan.close
            self.decode_plan = plan.plan
            self.bytes_rank = algorithmic_bytes(local)
            self.nvlink_bytes = plan.nvlink_bytes_per_step
            self.graphable = False
            if args.exchange == "peer":
                self.extra_kernels = -self.decode_plan.kernels_per_run(self.q.dtype) + 1   # one kernel a step
                how = (f"one kernel per rank: decode, NVLink peer stores of {pd_dist.packed_size(loc) * 4} B "
                       "into every rank's buffer, bounded wait for all ranks, max-corrected merge")
            else:
                self.extra_kernels = 1      # the cross-shard merge (NCCL's own kernel not counted)
                how = f"NCCL all_gather of {pd_dist.packed_size(loc) * 4} B per rank + max-corrected merge"
            self.sharding = f"sequence, strong: rank r owns logical pages [{lo}, {hi}) of every sequence; {how}"
        self.kv = [(k, v)]
        if not hasattr(self, "out"):
            self.out = torch.empty(self.out_shape(), dtype=torch.float32, device=self.q.device)

    def out_shape(self):
        L = self.decode_plan.layout
        return (L.batch, L.query_heads, L.head_dim)

    def add_copies(self, n):
        """Identical K/V copies, so that step i reads copy i % n."""
        k, v = self.kv[0]
        self.kv += [(k.clone(), v.clone()) for _ in range(n - 1)]

    def step(self, i, q=None, out=None):
        k, v = self.kv[i % len(self.kv)]
        return self._run(self.q if q is None else q, k, v, self.out if out is None else out)

    def kernels_per_step(self):
        return self.decode_plan.kernels_per_run(self.q.dtype) + self.extra_kernels


def time_windows(job, args, stream, flush):
    """R windows of K steps; returns the per-step device ms of every window.

    Graph timing captures the K steps once through the public run() and
    replays them; eager timing launches them from Python.  With --l2 flush
    each step is bracketed by its own events after an L2 flush.
    """
    import torch
    K, R = args.steps, args.windows
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731
    if flush is not None:
        times = []
        for _ in range(R):
            total = 0.0
            for i in range(K):
                flush.amax()
                a, b = ev(), ev()
                a.record(stream)
                job.step(i)
                b.record(stream)
                b.synchronize()
                total += a.elapsed_time(b)
            times.append(total / K)
        return times, "eager, L2 flushed before each step, per-step events"
    graph = None
    if args.timing == "graph" and job.graphable:
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        # thread-local capture: other threads (NCCL's watchdog at N > 1) keep working
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):
            for i in range(K):
                job.step(i)
        stream.wait_stream(cap)
        graph.replay()                     # one untimed replay
        torch.cuda.synchronize()
    starts, ends = [ev() for _ in range(R)], [ev() for _ in range(R)]
    for r in range(R):
        starts[r].record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(K):
                job.step(i)
        ends[r].record(stream)
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) / K for s, e in zip(starts, ends)]
    del graph
    how = ("CUDA graph of the K steps (captured once via DecodePlan.run), one replay per window"
           if args.timing == "graph" and job.graphable else "K eager steps per window")
    return times, how


def run_ours(args, rank, local, world):
    import torch

    job = RankJob(args, rank, world)
    w = job.workload
    q = job.q
    k, v = job.kv[0]
    kv_bytes = 2 * k.numel() * k.element_size()
    flush, l2 = None, "inputs larger than L2 (each step reads more than 2x L2)"
    if kv_bytes < 2 * L2_BYTES:
        if args.l2 == "flush":
            # read-only flush: leaves L2 full of clean lines, so the decode never pays
            # for write-backs that a zero-fill flush would leave behind
            flush = torch.ones(2 * L2_BYTES // 2, dtype=torch.float16, device="cuda")
            l2 = "L2 flushed (read-only pass over 252 MB) before each step"
        else:
            copies = max(2, math.ceil(4 * L2_BYTES / kv_bytes))
            job.add_copies(copies)
            l2 = (f"{copies} identical K/V copies ({copies * kv_bytes / 2**20:.0f} MiB > 4x the 126 MiB L2) "
                  "rotated step by step: each step reads a copy the previous steps did not")
    if args.timing is None:
        args.timing = "graph" if job.graphable else "eager"
    stream = torch.cuda.current_stream()

    clocks = ClockSampler(local).start()
    for i in range(max(args.warmup, 0)):
        job.step(i)
    barrier(world)

    # (1) R timed windows of K steps each, bracketed by barrier + synchronize.
    clocks.mark_start()
    t_wall = time.perf_counter()
    window_ms, how = time_windows(job, args, stream, flush)
    barrier(world)
    timed_s = time.perf_counter() - t_wall
    clocks.mark_end()
    clocks.stop()
    window_ms = max_over_ranks(window_ms, world)
    step_ms = statistics.median(window_ms)
    errors = job.decode_plan.read_errors()
    if errors:
        raise SystemExit(f"device error word {errors:#x}")
    timed_out = job.out.clone()             # the timed steps' output (every step writes the same)

    # (2) e2e through the public API with host buffers.  Every step copies its q
    # from pinned host memory and its FP32 output back; the two directions run
    # on their own streams, double-buffered, so step i+1's input and step i-1's
    # output move while step i decodes (the decode writes straight into the
    # staging buffer the output is copied back from).  On one GPU,
    # --graph-steps such steps (their copies included) are captured once
    # through the same public calls and replayed, so the host's per-call
    # overhead does not set the pace.
    e2e = None
    if not args.no_e2e:
        copy = torch.cuda.Stream()       # device -> host
        upload = torch.cuda.Stream()     # host -> device
        q_host = [q.cpu().pin_memory() for _ in range(2)]
        out_shape = job.out_shape()
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
            if flush is not None:
                flush.amax()
            job.step(i, q=q_dev[b], out=stage[b])
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
               "path": ("public API run() (ctypes -> C ABI pd_decode, out= the staging buffer); pinned host q "
                        "in and FP32 out back every step, each direction on its own stream, double-buffered"
                        + (f"; {args.graph_steps} steps captured once as a CUDA graph and replayed"
                           if world == 1 else ""))}

    peak, peak_kind = measured_peak()
    kernel_ms = statistics.median(window_ms)
    achieved = job.bytes_rank / (kernel_ms * 1e-3) / 1e9
    traffic, traffic_note = None, None
    info = job.decode_plan.native_info(q.dtype)
    tcgen05 = int(info.engine) == 1
    if world == 1 or args.scaling == "weak":
        if tcgen05:
            traffic = NCU_TRAFFIC_BYTES_TCGEN05.get(args.workload)
        elif args.workload in NCU_TRAFFIC_BYTES:
            traffic = NCU_TRAFFIC_BYTES[args.workload]
        elif args.workload in NCU_SCALED:
            from paged_decode import workload as wl
            src, src_traffic = NCU_SCALED[args.workload]
            ratio = job.bytes_rank / algorithmic_bytes(wl.CONFIGS[src]())
            traffic = int(src_traffic * ratio)
            traffic_note = (f"ncu capture of workload {src} ({src_traffic} B) scaled by the ratio of "
                            f"algorithmic bytes {ratio:.3f}")
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
        "data": "synthetic: seeded N(0,1)-scaled tensors, BASELINE config generators (no dataset exists)",
        "config": {"workload": w.name, "batch": w.layout.batch, "query_heads": w.layout.query_heads,
                   "kv_heads": w.layout.kv_heads, "head_dim": w.layout.head_dim,
                   "page_size": w.layout.page_size, "split_tokens": w.split_tokens,
                   "bytes_per_step_total": job.bytes_total, "bytes_per_step_rank": job.bytes_rank,
                   "sharding": job.sharding, "l2": l2, "timing": how,
                   "persistent_ctas": int(info.num_ctas),
                   "kv_heads_per_tile": int(info.heads_per_tile),
                   "engine": "tcgen05" if tcgen05 else "warp",
                   "cluster_ctas": int(info.cluster_ctas)},
        "windows": {"count": args.windows, "steps_each": args.steps,
                    "median_us": step_ms * 1e3, "min_us": min(window_ms) * 1e3,
                    "p95_us": percentile(window_ms, 95) * 1e3,
                    "raw_us": [round(x * 1e3, 3) for x in window_ms],
                    "timed_region_s": timed_s, "per_window": "max over ranks"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic,
                     "kernel": ("paged_decode_mqa_kernel" if tcgen05 else "paged_decode_kernel")
                               + ("" if job.kernels_per_step() == 1 else " (+ merge_partials_kernel)"),
                     "kernel_us": kernel_ms * 1e3,
                     "algorithmic_bytes_per_launch": job.bytes_rank},
        "gpu_launches": args.windows * args.steps * job.kernels_per_step(),
        "clocks": clocks.summary(),
    }
    if traffic_note:
        line["roofline"]["traffic_note"] = traffic_note
    if hasattr(job, "nvlink_bytes"):
        line["nvlink_bytes_per_step_per_gpu"] = job.nvlink_bytes
    if e2e:
        line["e2e"] = e2e

    # (3) The cpu_baseline leg: the FP64 oracle timed on rank 0 at N = 1, and on
    # every rank that owns an output, the gate on the timed output.
    if not args.no_cpu_baseline:
        ok = True
        if job.check is not None:
            cw, cq, ck, cv = job.check
            threads = max(1, (os.cpu_count() or 1) // world)
            if world == 1:
                base, ref = cpu_baseline(cw, cq, ck, cv, job.bytes_total, args.cpu_seconds)
                line["cpu_baseline"] = base
            else:
                _, ref = cpu_baseline(cw, cq, ck, cv, 0, 0, steps=1, threads=threads)
            result = gate(timed_out, ref, cw.dtype)
            ok = result["gate"] == "pass"
            line["gate"] = dict(result, checked_by=("rank 0 (full merged output)" if world > 1 and
                                                     job.sharding.startswith("sequence")
                                                     else "every rank, its own heads" if world > 1 else "rank 0"))
        if not all_ranks_ok(ok, world):
            line["gate"] = dict(line.get("gate", {}), gate="fail")
    if world == 1 and not args.no_competitors:
        line["competitors"] = competitors(w, q, job, flush, args.steps)
    job.close()
    return line


def competitors(w, q, job, flush, steps):
    """The reference's comparisons on the same caches, timed like our step.

    FlashInfer's batch decode (FP16 only; empty rows get one token because it
    needs nonempty contexts, so its workload is that much larger, never
    smaller) with and without its tensor-core path, and the dense baseline:
    gather the pages into padded dense K/V and run PyTorch SDPA.  Each
    rotates over the same K/V copies as our steps (or flushes L2 the same way).
    """
    import torch
    from paged_decode.competitors import DenseSDPAPlan, FlashInferPlan
    table, lengths = w.table.copy(), w.lengths.copy()
    table[lengths == 0, 0] = 0
    lengths[lengths == 0] = 1
    out = {}
    ours = job.out.clone()
    live = torch.as_tensor(w.lengths > 0, device=q.device)   # rows the comparisons all define alike
    entries = [("dense_gather_sdpa", lambda: DenseSDPAPlan(w.layout, w.table, w.lengths, device=q.device))]
    if w.dtype == "float16":
        entries += [("flashinfer", lambda: FlashInferPlan(w.layout, table, lengths, device=q.device)),
                    ("flashinfer_tensor_cores",
                     lambda: FlashInferPlan(w.layout, table, lengths, device=q.device, tensor_cores=True))]
    n = len(job.kv)
    for key, make in entries:
        try:
            fi = make()
            for i in range(3):
                fi.run(q, *job.kv[i % n])
            torch.cuda.synchronize()
            if flush is None:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for i in range(steps):
                    fi.run(q, *job.kv[i % n])
                b.record()
                torch.cuda.synchronize()
                ms = a.elapsed_time(b) / steps
            else:
                times = []
                for _ in range(steps):
                    flush.amax()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    fi.run(q, *job.kv[0])
                    b.record()
                    torch.cuda.synchronize()
                    times.append(a.elapsed_time(b))
                ms = sum(times) / steps
            result = fi.run(q, *job.kv[0])
            torch.cuda.synchronize()
            out[key] = {"version": getattr(fi, "version", torch.__version__), "us_per_step": ms * 1e3,
                        "value": job.bytes_total / (ms * 1e-3) / 1e12, "unit": "TB/s",
                        "max_abs_vs_ours": float((result.float() - ours)[live].abs().max()),
                        "timing": "eager back to back over the same K/V copies (or L2 flushed per step)"}
            del fi
        except Exception as exc:  # noqa: BLE001 - reported, never fatal
            out[key] = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    return out


# ---------------------------------------------------------------------- reference arm
def sample_workload(w, rows):
    """The first ``rows`` sequences of ``w`` (same caches): a bounded CPU sample."""
    from paged_decode import workload
    from paged_decode.layout import Layout
    L = w.layout
    lay = Layout(rows, L.query_heads, L.kv_heads, L.head_dim, L.page_size, L.physical_pages)
    return workload.Workload(w.name, lay, w.table[:rows], w.lengths[:rows], w.split_tokens, dtype=w.dtype,
                             std=w.std, seed=w.seed)


def run_reference(args, rank, local, world):
    import torch
    from paged_decode import workload

    if rank != 0:
        return None
    w = workload.CONFIGS[args.workload]()
    q, k, v = w.tensors("cuda")
    nbytes = algorithmic_bytes(w)
    t0 = time.perf_counter()
    qh, kh, vh = (t.cpu().numpy() for t in (q, k, v))     # host copies, made once
    # Size the per-step sample: whole steps when one takes at most ~0.3 s on
    # the host, else the first sequences of the batch up to that much work.
    first, _ = cpu_baseline(w, qh, kh, vh, nbytes, 0, steps=1)
    rows = w.layout.batch
    if first["s_per_step"] > 0.3:
        rows = max(1, int(w.layout.batch * 0.3 / first["s_per_step"]))
    sw = sample_workload(w, rows)
    sq = qh[:rows].copy()
    sbytes = algorithmic_bytes(sw)
    for _ in range(max(args.warmup - 1, 0)):
        cpu_baseline(sw, sq, kh, vh, sbytes, 0, steps=1)
    samples = [cpu_baseline(sw, sq, kh, vh, sbytes, 0, steps=1)[0] for _ in range(args.steps)]
    s_per_step = statistics.mean(s["s_per_step"] for s in samples)
    value = sbytes / s_per_step / 1e12
    base = samples[0]
    what = (f"{'every' if rows == w.layout.batch else f'the first {rows} of {w.layout.batch}'} sequences "
            f"of {w.name} per step ({sbytes} algorithmic bytes)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": s_per_step * 1e3,
        "us_per_step": s_per_step * 1e6, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: seeded N(0,1)-scaled tensors, BASELINE config generators (no dataset exists)",
        "config": {"workload": w.name, "bytes_per_step_total": nbytes, "sample_bytes_per_step": sbytes,
                   "sample_sequences": rows},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": base["cores"], "kind": "port",
                         "sample": f"{args.steps} timed steps, each {what} (FP64 C restatement of the "
                                   f"reference oracle.dense_attention, {base['cores']} threads)"},
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
    if args.steps < 1 or args.warmup < 0 or args.windows < 1:
        raise SystemExit("--steps >= 1, --warmup >= 0 and --windows >= 1 required")
    if args.impl == "reference" and int(os.environ.get("RANK", "0")) != 0:
        return                      # the reference arm runs on rank 0 only
    if args.impl == "reference":
        os.environ["WORLD_SIZE"] = "1"
        args.gpus = 1
    rank, local, world = dist_setup(args)
    failed = False
    try:
        line = (run_reference if args.impl == "reference" else run_ours)(args, rank, local, world)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
        failed = line is not None and line.get("gate", {}).get("gate") == "fail"
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if failed:
        raise SystemExit("correctness gate failed: the timed output differs from the FP64 oracle")


if __name__ == "__main__":
    main()
