#!/usr/bin/env python3
"""Benchmark of the row-sharded eager-op workload on 1..8 B200s (one process per GPU).

Workload (the multi-GPU configuration of the hot path): X float32 [262144, 8192] ~ N(0, 1)
(seed 4), rows split into contiguous blocks across the ranks, and r float32 [1, 8192] ~ U(-1, 1)
(seed 4, stream 1) on every rank. One step:
    Y = (X - r) * r          bit-identical to ctorch's sub then mul
    s = sum(Y)               float64 partial per rank, exchanged between ranks, rank-order sum
    k = argmin(Y, dim=1)     per row, first index on ties
computed by one kernel launch per rank (ctb_chain_rows_allsum): one pass over the rank's rows
with a row-argmin and float64-sum epilogue, whose last CTA stores the rank's partial into every
rank's workspace over NVLink, waits for the others' and adds them in rank order. The same step
with the partials all-gathered through NCCL instead, as three kernels (chain, sum, argmin), and
as ctorch's eager op sequence (sub, mul, sum, argmin) is timed too and reported beside it. Total work is fixed as GPUs are added (strong scaling). `value` is elements of X processed per
second by the whole job, device-timed with CUDA events, max over ranks. Inputs (8 GiB in total)
are larger than the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

--impl reference times ctorch's own CPU implementation of the same step (its public front-doors,
compiled from its sources into oracle/_ref/) on a bounded row sample, on rank 0 only.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS, COLS = 262144, 8192
SEED = 4
METRIC = "HBM GB/s per op vs ~8 TB/s peak; elements/sec at 1/2/4/8 B200 vs ctorch CPU"
UNIT = "elements/s"
WORKLOAD = ("row-sharded Y=(X-r)*r, sum(Y), argmin(Y,1); X f32[262144,8192] ~N(0,1) seed 4, "
            "r f32[1,8192] ~U(-1,1)")
FALLBACK_HBM_GBS = 6650.0


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def base_config(world):
    return {"workload": WORKLOAD, "rows": ROWS, "cols": COLS, "parallelism": f"rows{world}",
            "l2": "inputs larger than L2 (no flush)", "data": "synthetic, seeded splitmix64"}


# ------------------------------------------------------------------------------- CPU (ctorch)

def host_synth():
    """ctorch_b200/synth.py loaded as a standalone module (numpy only), so that the CPU legs never
    import the package, whose import loads the CUDA kernel library: the reference arm's process
    maps ctorch's code (oracle/_ref) and nothing of this backend."""
    import importlib.util

    name = "_ctb_host_synth"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "ctorch_b200", "synth.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def host_inputs(rows):
    sy = host_synth()
    x = sy.host_fill((rows, COLS), "float32", sy.NORMAL, SEED, 0, 0.0, 1.0)
    r = sy.host_fill((1, COLS), "float32", sy.UNIFORM, SEED, 1, -1.0, 1.0)
    return x, r


def ctorch_cpu_step(ref, x, r):
    """ctorch's public CPU front-doors: sub, mul (src/ops/binary_ops_cpu.cpp:251-254), sum
    (reduction_ops_cpu.cpp:463), argmin (:497)."""
    t = ref.binary("sub", x, r)
    y = ref.binary("mul", t, r)
    s = ref.reduce("sum", y)
    k = ref.arg("argmin", y, 1)
    return s, k


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def time_ctorch_cpu(rows, steps, warmup, threads=1):
    """ctorch's CPU front-doors on `rows` rows of the workload, the rows split into contiguous
    blocks over `threads` host threads. Each thread runs the whole step (sub, mul, sum, argmin)
    on its block: ctorch's CPU kernels are single-threaded (`#pragma omp simd` only, no threading
    runtime), so a row split is the only way its code uses more than one core, and it is the same
    split the GPU ranks use. The blocks' float32 sums are then added in block order (in double) and
    the row argmins stay per block. ctypes releases the GIL inside each call, and ctorch's CPU pool
    allocator keeps one cache per thread. Returns (elements per second, seconds per step)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import ref as get_ref

    ref = get_ref()
    xh, rh = host_inputs(rows)
    threads = max(1, min(int(threads), rows))
    bounds = [(rows * t // threads, rows * (t + 1) // threads) for t in range(threads)]
    xs = [ref.tensor(xh[a:b]) for a, b in bounds]
    r = ref.tensor(rh)
    del xh
    pool = ThreadPoolExecutor(max_workers=threads) if threads > 1 else None

    def step():
        if pool is None:
            ctorch_cpu_step(ref, xs[0], r)
            return
        parts = list(pool.map(lambda x: ctorch_cpu_step(ref, x, r), xs))
        total = 0.0
        for s_block, _ in parts:
            total += float(s_block.numpy())
        return total

    try:
        for _ in range(warmup):
            step()
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            step()
            ts.append(time.perf_counter() - t0)
    finally:
        if pool is not None:
            pool.shutdown()
    per_step = statistics.mean(ts)
    return rows * COLS / per_step, per_step


def calibrate_rows(budget_s, n_steps, threads, probe_rows=1024):
    """Rows per CPU step (a power of two, 512..65536) so that n_steps on `threads` threads fit in
    budget_s, from a one-thread probe."""
    _, t = time_ctorch_cpu(probe_rows, 1, 0, 1)
    per_row = t / probe_rows
    rows = max(512, min(65536, int(budget_s / max(1, n_steps) / per_row * threads)))
    p = 512
    while p * 2 <= rows:
        p *= 2
    return p


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    threads = host_threads()
    rows = args.cpu_rows or calibrate_rows(150.0, args.steps + args.warmup, threads)
    value, per_step = time_ctorch_cpu(rows, args.steps, args.warmup, threads)
    sample = (f"{rows} of {ROWS} rows per step ({rows * COLS} elements), ctorch front-doors "
              f"sub, mul, sum, argmin on CPU tensors, rows split in {threads} blocks over {threads} "
              f"host threads (ctorch's CPU kernels are single-threaded each)")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": base_config(world), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock and throttle-reason samples every 50 ms, each stamped with the host time it
    arrived, so that stop() keeps only the samples taken inside the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n_devices=1):
        self.n_devices = n_devices
        self.proc = None
        self.lines = []
        self.reader = None

    def start(self):
        """Samples the GPUs the job's ranks use (local ranks 0..n-1 on devices 0..n-1 of the
        visible list), not the node's other GPUs, which may be idle."""
        import threading

        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        ids = vis.split(",")[: self.n_devices] if vis else [str(i) for i in range(self.n_devices)]
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
               "-i", ",".join(i.strip() for i in ids)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def read():
            for line in self.proc.stdout:
                self.lines.append((time.time(), line))

        self.reader = threading.Thread(target=read, daemon=True)
        self.reader.start()

    def stop(self, t0=None, t1=None):
        """Median SM clock, max clock and the throttle reasons seen in the samples that arrived
        between t0 and t1 (host time.time(); all samples when none did, `in_window` false)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        time.sleep(0.12)  # the sample taken at t1 arrives a little later
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        if self.reader is not None:
            self.reader.join(timeout=5)
        lines = self.lines
        in_window = True
        if t0 is not None and t1 is not None:
            sel = [ln for ts, ln in lines if t0 <= ts <= t1 + 0.1]
            if not sel:
                sel, in_window = [ln for _, ln in lines], False
        else:
            sel = [ln for _, ln in lines]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO("".join(sel))):
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                smax.append(float(row[2]))
            except ValueError:
                continue
            for nm, val in zip(names, row[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "in_window": in_window}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(rows):
    """DRAM bytes (read + write) of one launch of the one-pass kernel over `rows` rows, from the
    committed ncu capture (profiles/ncu_traffic.json): the read bytes per row times the rows, plus
    the algorithmic writes per row times the rows, less the constant part of Y still dirty in L2
    when the kernel ends (which the captured launch did not write back). None if absent."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        n = float(d["rows"])
        read_per_row = float(d["dram_read"]) / n
        write_per_row = (float(d["dram_write"]) + float(d["l2_write_tail"])) / n
        return read_per_row * rows + write_per_row * rows - float(d["l2_write_tail"])
    except (OSError, KeyError, ValueError, ZeroDivisionError):
        return None


# ------------------------------------------------------------------------------- GPU arm

PLUGIN_CHECK = os.path.join(ROOT, "ctorch_b200", "ctorch_plugin", "_build", "plugin_check")


def plugin_bench(reps=50, timeout=600):
    """The hot-path ops through ctorch's own API with this backend linked in (plugin_check
    --bench): per op, dispatch::call into preallocated outputs, the public front-door (allocation
    + Storage zero-fill + kernel) and the zero-fill alone. A list of dicts, or None when the
    plugin was not built (no ctorch sources at build time)."""
    if not os.path.exists(PLUGIN_CHECK):
        return None
    r = subprocess.run([PLUGIN_CHECK, "--bench", str(reps)], capture_output=True, text=True, timeout=timeout)
    out = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    if r.returncode != 0:
        out.append({"error": f"plugin_check --bench exited {r.returncode}", "stderr": r.stderr[-400:]})
    return out

def run_b200(args):
    import datetime

    import torch
    import torch.distributed as dist

    import ctorch_b200 as cb
    from ctorch_b200.sharded import PeerStep, ShardedSum, row_shard, sharded_step_fused
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    rank, world, local = env_rank()
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def check_exchange():
        """Every one-launch step so far completed its cross-GPU exchange, on every rank (a wait
        that ran out leaves NaN as the sum and is recorded in the rank's workspace)."""
        done, failed = peer.status()
        bad = max_over_ranks(float(failed != 0 or done != peer.epoch))
        if bad:
            raise cb.CommTimeoutError(f"rank {rank}: a cross-GPU exchange timed out (status {done}, {failed}; "
                                      f"{peer.epoch} calls)")

    shard = row_shard(ROWS, rank, world)
    x = torch.empty((shard.rows, COLS), dtype=torch.float32, device=dev)
    r = torch.empty((1, COLS), dtype=torch.float32, device=dev)
    device_fill(x, NORMAL, SEED, 0, 0.0, 1.0, first=shard.start * COLS)
    device_fill(r, UNIFORM, SEED, 1, -1.0, 1.0)
    summer = ShardedSum(dev, world)
    # the step: one launch per rank that also exchanges the sum's partials over NVLink
    peer = PeerStep(dev, rank, world)
    y_buf = torch.empty_like(x)
    k_buf = torch.empty(shard.rows, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()

    def step():
        return peer(x, r, y_buf, k_buf)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()

    K = args.steps
    # The kernel's own duration (for the roofline) comes from events around every tenth step only:
    # an event recorded between two launches keeps the second from starting as a programmatic
    # dependent of the first, so the other steps run back to back as in production.
    sampled = [i for i in range(K) if i % 10 == 0]
    ev = {i: [torch.cuda.Event(enable_timing=True) for _ in range(2)] for i in sampled}
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(int(os.environ.get("LOCAL_WORLD_SIZE", world)))
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    cb.launch_count_reset()
    t_region0 = time.time()
    start.record()
    for i in range(K):
        if i in ev:
            ev[i][0].record()
        step()
        if i in ev:
            ev[i][1].record()
    end.record()
    torch.cuda.synchronize()
    t_region1 = time.time()
    barrier()
    launches = cb.launch_count()
    clocks = sampler.stop(t_region0, t_region1) if rank == 0 else None
    check_exchange()
    # where a step's time goes on each rank (kernel-side timestamps of the last timed calls)
    step_trace = PeerStep.trace_summary(peer.trace(min(K, 64)))
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, step_trace)
    else:
        gathered = [step_trace]
    elapsed = max_over_ranks(start.elapsed_time(end))
    fused_ms = max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in ev.values()))
    total_launches = int(sum_over_ranks(launches))

    def time_steps(fn, n):
        fn()  # warm-up (first-call allocations)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1)) / n

    def three_kernels():
        y = cb.binary_chain("sub", "mul", x, r, r)
        summer(y)
        cb.argmin(y, 1)

    def eager_ops():
        y = cb.mul(cb.sub(x, r), r)
        summer(y)
        cb.argmin(y, 1)

    def nccl_step():
        sharded_step_fused(x, r, summer)

    n_cmp = min(K, 20)
    nccl_ms = time_steps(nccl_step, n_cmp)
    three_kernel_ms = time_steps(three_kernels, n_cmp)
    eager_ms = time_steps(eager_ops, n_cmp)

    # end to end: pinned host input -> device, step, device -> pinned host results
    e2e = None
    xd = rd = None
    if not args.no_e2e:
        xh = torch.empty((shard.rows, COLS), dtype=torch.float32, pin_memory=True)
        xh.copy_(x)
        rh = torch.empty((1, COLS), dtype=torch.float32, pin_memory=True)
        rh.copy_(r)
        kh = torch.empty((shard.rows,), dtype=torch.int64, pin_memory=True)
        sh = torch.empty((), dtype=torch.float32, pin_memory=True)
        xd = torch.empty_like(x)
        rd = torch.empty_like(r)

        def e2e_step():
            xd.copy_(xh, non_blocking=True)
            rd.copy_(rh, non_blocking=True)
            y, s, k = peer(xd, rd, y_buf, k_buf)
            sh.copy_(s, non_blocking=True)
            kh.copy_(k, non_blocking=True)

        e2e_steps = max(2, min(K, 5))
        e2e_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(e2e_steps):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(a0.elapsed_time(a1)) / e2e_steps
        check_exchange()
        e2e = {"value": ROWS * COLS / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": ROWS * COLS * 4 + world * COLS * 4,
               "d2h_bytes_per_step": ROWS * 8 + world * 4, "ms_per_step": e2e_ms,
               "path": "pinned host X, r -> HBM; one launch per rank: chain + row argmin + float64 "
                       "partial, partials exchanged over NVLink and combined (ctb_chain_rows_allsum); "
                       "s and k -> pinned host"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        rows = args.cpu_rows or 32768
        v, per_step = time_ctorch_cpu(rows, 2, 1, threads)
        v1, per_step1 = time_ctorch_cpu(min(rows, 4096), 2, 1, 1)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "reference",
               "sample": f"{rows} of {ROWS} rows ({rows * COLS} elements) through ctorch's CPU "
                         f"front-doors sub, mul, sum, argmin, rows split over {threads} host threads; "
                         f"mean of 2 steps after 1 warm-up, {per_step:.3f} s per step",
               "one_thread": {"value": v1, "unit": UNIT, "cores": 1,
                              "sample": f"{min(rows, 4096)} rows on one thread, {per_step1:.3f} s per step"}}

    per_op, plugin = None, None
    if rank == 0 and world == 1 and not args.no_per_op:
        xd = rd = None  # noqa: F841 (the e2e buffers: 8 GiB)
        torch.cuda.empty_cache()
        per_op = []
        sub = argparse.Namespace(steps=min(K, 50), warmup=3, no_cpu_baseline=args.no_cpu_baseline)
        run_suite(sub, sink=per_op)
        torch.cuda.empty_cache()
        plugin = plugin_bench(reps=min(K, 50))

    if rank == 0:
        peak, peak_kind = measured_peak()
        fused_bytes = shard.rows * COLS * 4 * 2 + COLS * 4 + shard.rows * 8
        achieved = fused_bytes / (fused_ms / 1e3) / 1e9
        traffic = ncu_traffic(shard.rows)
        ms_per_step = elapsed / K
        line = {
            "metric": METRIC,
            "value": ROWS * COLS * K / (elapsed / 1e3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": base_config(world),
            "gbs": (ROWS * COLS * 4 * 2 + ROWS * 8) / (ms_per_step / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "kernel": "fused_rows_kernel (ctb_chain_rows_allsum: (X - r) * r, row argmin, "
                                   "float64 sum exchanged across ranks in the same launch)",
                         "algorithmic_bytes": fused_bytes,
                         "traffic": traffic,
                         "traffic_note": "ncu DRAM bytes of a 65536-row launch, per row, less the constant "
                                         "L2 write-back tail (profiles/ncu_traffic.json)"},
            "kernels_ms": {"chain_rows_allsum": fused_ms,
                           "timed_launches": len(ev),
                           "note": "CUDA events around every tenth timed step, max over ranks of the mean"},
            "step_trace_by_rank": gathered,
            "nccl_step_ms_per_step": nccl_ms,
            "three_kernel_ms_per_step": three_kernel_ms,
            "eager_ms_per_step": eager_ms,
            "gpu_launches": total_launches,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "per_op": per_op,
            "plugin_ops": plugin,
        }
        print(json.dumps(line), flush=True)
    del summer
    peer.close()
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------- profiling cases

def run_case(args):
    """Launches one kernel of the hot path a few times on a reduced input, for an ncu capture
    (e.g. `ncu --set full --clock-control none -k regex:ew_rows -c 3 python bench.py --case chain
    --rows 4096 --warmup 0 --steps 3`, after the same command has run without ncu). Inputs stay
    larger than L2 at the default sizes. Prints nothing to time."""
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.sharded import ShardedSum
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    dev = torch.device("cuda", 0)
    rows = args.rows
    t = lambda shape, dt=torch.float32: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
    case = args.case
    if case in ("chain", "sum", "argmin", "sub", "chain_rows", "step"):
        from ctorch_b200.sharded import PeerStep

        x = device_fill(t((rows, COLS)), NORMAL, SEED, 0, 0.0, 1.0)
        r = device_fill(t((1, COLS)), UNIFORM, SEED, 1, -1.0, 1.0)
        y = cb.binary_chain("sub", "mul", x, r, r)
        summer = ShardedSum(dev, 1)
        if case == "step":  # the bench's own step: one launch (world of one)
            peer = PeerStep(dev, 0, 1)
            k = torch.empty(rows, dtype=torch.int64, device=dev)
            fn = lambda: peer(x, r, y, k)  # noqa: E731
        else:
            fn = {"chain": lambda: cb.binary_chain("sub", "mul", x, r, r), "sub": lambda: cb.sub(x, r),
                  "sum": lambda: summer(y), "argmin": lambda: cb.argmin(y, 1),
                  "chain_rows": lambda: cb.chain_rows("sub", "mul", x, r, r, out_sum=summer.partial)}[case]
    elif case in ("add", "relu"):
        a = device_fill(t((4096, 4096)), UNIFORM, 0, 0, -1.0, 1.0)
        b = device_fill(t((1, 4096)), UNIFORM, 0, 1, -1.0, 1.0)
        fn = (lambda: cb.add(a, b)) if case == "add" else (lambda: cb.relu(a))
    elif case in ("sum_rows", "argmax_cols", "max_cols", "prod_rows", "sum_cols"):
        x = device_fill(t((8192, 8192)), NORMAL, 1, 0, 0.0, 1.0)
        fn = {"sum_rows": lambda: cb.sum(x, [1], True), "prod_rows": lambda: cb.prod(x, [1]),
              "argmax_cols": lambda: cb.argmax(x, 0), "max_cols": lambda: cb.max(x, 0),
              "sum_cols": lambda: cb.sum(x, [0])}[case]
    elif case == "cols_bulk":  # rows of 4096 floats, too narrow for 148 strips: the bulk column kernel
        x = device_fill(t((16384, 4096)), NORMAL, 1, 0, 0.0, 1.0)
        fn = lambda: cb.argmax(x, 0)  # noqa: E731
    elif case == "cols_narrow":  # 256-byte rows: the flat narrow column kernel
        x = device_fill(t((1_000_000, 64)), NORMAL, 1, 0, 0.0, 1.0)
        fn = lambda: cb.argmax(x, 0)  # noqa: E731
    elif case == "cols_outer":  # rows of 8190 floats (not a whole number of 16-byte chunks): the register kernel
        x = device_fill(t((8192, 8190)), NORMAL, 1, 0, 0.0, 1.0)
        fn = lambda: cb.max(x, 0)  # noqa: E731
    elif case == "rows_short":  # rows of 64 floats with a broadcast row: the short-row elementwise kernel
        a = device_fill(t((1_048_576, 64)), UNIFORM, 0, 0, -1.0, 1.0)
        b = device_fill(t((1, 64)), UNIFORM, 0, 1, -1.0, 1.0)
        fn = lambda: cb.add(a, b)  # noqa: E731
    elif case == "tiled_f64":  # float64 operand read transposed: the 64x64 shared-memory tile kernel
        a = device_fill(t((32, 1024, 1024), torch.float64), UNIFORM, 3, 0, -1.0, 1.0)
        b = device_fill(t((32, 1024, 1024), torch.float64), UNIFORM, 3, 1, -1.0, 1.0)
        fn = lambda: cb.mul(a, b.permute(0, 2, 1))  # noqa: E731
    elif case == "ew_general":  # two operands permuted two different ways: the per-element decode kernel
        a = device_fill(t((1024, 1024, 64)), UNIFORM, 3, 0, -1.0, 1.0)
        b = device_fill(t((64, 1024, 1024)), UNIFORM, 3, 1, -1.0, 1.0)
        fn = lambda: cb.add(a.permute(2, 0, 1), b.transpose(1, 2))  # noqa: E731
    elif case == "red_runs":  # sum over dims 0 and 2 of [64, 1024, 1024]: packs along the reduced runs
        x = device_fill(t((64, 1024, 1024)), NORMAL, 1, 0, 0.0, 1.0)
        fn = lambda: cb.sum(x, [0, 2])  # noqa: E731
    elif case == "red_general":  # the same over [64, 1024, 1023]: runs of 1023 floats, per-element decode
        x = device_fill(t((64, 1024, 1023)), NORMAL, 1, 0, 0.0, 1.0)
        fn = lambda: cb.sum(x, [0, 2])  # noqa: E731
    elif case == "argmin_rows":
        y = device_fill(t((rows, COLS)), NORMAL, SEED, 0, 0.0, 1.0)
        fn = lambda: cb.argmin(y, 1)  # noqa: E731
    elif case == "gather_general":  # rows gathered from a transposed source: the strided gather kernel
        x = device_fill(t((8192, 8192)), NORMAL, 2, 0, 0.0, 1.0)
        idx = device_fill(t((4096,), torch.int64), UNIFORM, 2, 2, 0, 8191)
        fn = lambda: cb.index_select_async(x.t(), 0, idx)  # noqa: E731
    elif case == "index_select":
        tab = device_fill(t((1_000_000, 256)), NORMAL, 2, 0, 0.0, 1.0)
        idx = device_fill(t((rows * 16,), torch.int64), UNIFORM, 2, 2, 0, 999_999)
        fn = lambda: cb.index_select_async(tab, 0, idx)  # noqa: E731
    elif case in ("mul_t", "div_b"):
        i = device_fill(t((64, 512, 1024), torch.int32), UNIFORM, 3, 0, -1000, 1000)
        f = device_fill(t((64, 1024, 512)), UNIFORM, 3, 1, -1.0, 1.0)
        d = device_fill(t((1, 512, 1), torch.float64), UNIFORM, 3, 2, 0.5, 2.0)
        p = cb.mul(i, f.permute(0, 2, 1))
        fn = (lambda: cb.mul(i, f.permute(0, 2, 1))) if case == "mul_t" else (lambda: cb.div(p, d))
    else:
        raise SystemExit(f"unknown case {case}")
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    return 0


# ------------------------------------------------------------------------------- per-op suite

def run_suite(args, sink=None):
    """Per-op device time and GB/s for every op of the five configurations, one JSON line per op
    (appended to `sink` instead when it is a list: the default run's `per_op` key).

    Each op is captured 8 times back to back in a CUDA graph (configuration 1, whose working set is
    about the size of L2, as 2 rounds over 4 separate copies of its inputs), and the graph is
    replayed `--steps` times back to back between CUDA events on the replay stream; the op's time
    is the elapsed time per call, each call following another as in a stream of eager ops. The inputs touched between two calls on the same data exceed the 126 MB L2, so no flush
    is needed, and no host (Python / ctypes) time falls inside the measurement. ctorch's own CPU
    path (oracle/_ref, its public front-doors, one thread) is timed on the same inputs, or on a
    stated sample of them, unless --no-cpu-baseline is given."""
    import torch

    import ctorch_b200 as cb
    from ctorch_b200.sharded import ShardedSum
    from ctorch_b200.synth import NORMAL, UNIFORM, device_fill

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = measured_peak()
    t = lambda shape, dt=torch.float32: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
    ref = None
    if not args.no_cpu_baseline:
        from oracle.oracle import ref as get_ref

        ref = get_ref()

    def graph_ms(fns):
        # 8 calls per graph (rounds of fns), so that each call follows another as in a stream of
        # eager ops: every kernel is launched as a programmatic dependent of the one before it
        fns = list(fns) * max(1, 8 // len(fns))
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                for fn in fns:
                    fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for fn in fns:
                fn()
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / (args.steps * len(fns))

    def cpu_ms(fn, reps=1):
        if ref is None:
            return None
        fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps * 1e3

    def emit(config, op, fn, nbytes, elems, cpu=None, cpu_elems=None, note=""):
        ms = graph_ms(fn if isinstance(fn, list) else [fn])
        line = {"config": config, "op": op, "ms": ms, "gbs": nbytes / ms / 1e6,
                "frac_of_measured_peak": nbytes / ms / 1e6 / peak, "peak_gbs": peak,
                "peak_kind": peak_kind, "algorithmic_bytes": nbytes, "elements_per_s": elems / ms * 1e3}
        if cpu is not None and ref is not None:
            cms = cpu_ms(cpu)
            ce = cpu_elems or elems
            line["cpu"] = {"ms": cms, "elements": ce, "elements_per_s": ce / cms * 1e3, "threads": 1,
                           "speedup": (elems / ms) / (ce / cms)}
        if note:
            line["note"] = note
        if sink is not None:
            sink.append(line)
        else:
            print(json.dumps(line), flush=True)

    def rt(x):  # ctorch CPU tensor of a device tensor's values
        return ref.tensor(x.cpu().numpy()) if ref is not None else None

    # config 1: 4 copies of the inputs, used in turn (4 x 134 MB > L2)
    a = device_fill(t((4096, 4096)), UNIFORM, 0, 0, -1.0, 1.0)
    b = device_fill(t((1, 4096)), UNIFORM, 0, 1, -1.0, 1.0)
    c = cb.add(a, b)
    ra, rb, rc = rt(a), rt(b), rt(c)
    copies = [(a.clone(), b.clone(), c.clone()) for _ in range(4)]
    rot = "4 copies of the inputs used in turn (536 MB > L2)"
    emit(1, "add", [lambda q=q: cb.add(q[0], q[1]) for q in copies], 134234112, 4096 * 4096,
         lambda: ref.binary("add", ra, rb), note=rot)
    emit(1, "relu", [lambda q=q: cb.relu(q[2]) for q in copies], 134217728, 4096 * 4096,
         lambda: ref.unary("relu", rc), note=rot)
    emit(1, "relu(add) one pass", [lambda q=q: cb.binary_unary("add", "relu", q[0], q[1]) for q in copies],
         134234112, 4096 * 4096, lambda: ref.unary("relu", ref.binary("add", ra, rb)), note=rot)
    del a, b, c, ra, rb, rc, copies
    # config 2
    x = device_fill(t((8192, 8192)), NORMAL, 1, 0, 0.0, 1.0)
    u = device_fill(t((8192, 8192)), UNIFORM, 1, 1, -1.0, 1.0)
    xp = cb.add(cb.mul(u, torch.tensor(0.001, device=dev)), torch.tensor(1.0, device=dev))
    del u
    rx, rxp = rt(x), rt(xp)
    rd = 268435456
    emit(2, "sum dim=1 keepdim", lambda: cb.sum(x, [1], True), rd + 32768, 8192 * 8192,
         lambda: ref.reduce("sum", rx, [1], True))
    emit(2, "mean dim=1 keepdim", lambda: cb.mean(x, [1], True), rd + 32768, 8192 * 8192,
         lambda: ref.reduce("mean", rx, [1], True))
    emit(2, "max dim=0 (values+indices)", lambda: cb.max(x, 0, False), rd + 32768 + 65536, 8192 * 8192,
         lambda: ref.reduce_idx("max", rx, 0))
    emit(2, "argmax dim=0", lambda: cb.argmax(x, 0, False), rd + 65536, 8192 * 8192,
         lambda: ref.arg("argmax", rx, 0))
    emit(2, "prod dim=1", lambda: cb.prod(xp, [1], False), rd + 32768, 8192 * 8192,
         lambda: ref.reduce("prod", rxp, [1], False))
    del x, xp, rx, rxp
    torch.cuda.empty_cache()
    # config 3 (the CPU leg gathers a 1/16 sample of the indices)
    idx = device_fill(t((4_194_304,), torch.int64), UNIFORM, 2, 2, 0, 999_999)
    for dt, name in ((torch.float32, "float32"), (torch.int32, "int32")):
        if dt == torch.float32:
            tab = device_fill(t((1_000_000, 256)), NORMAL, 2, 0, 0.0, 1.0)
        else:
            tab = device_fill(t((1_000_000, 256), torch.int32), UNIFORM, 2, 1, -(2**30), 2**30 - 1)
        rtab = rt(tab)
        ridx = ref.tensor(idx[:262144].cpu().numpy()) if ref is not None else None
        emit(3, f"index_select {name}", lambda: cb.index_select_async(tab, 0, idx), 8623489024,
             4_194_304 * 256, lambda: ref.index_select(rtab, 0, ridx), 262144 * 256,
             note="CPU leg: the first 262144 of the 4194304 indices")
        del tab, rtab
        torch.cuda.empty_cache()
    del idx
    # config 4
    i4 = device_fill(t((64, 512, 1024), torch.int32), UNIFORM, 3, 0, -1000, 1000)
    f4 = device_fill(t((64, 1024, 512)), UNIFORM, 3, 1, -1.0, 1.0)
    d4 = device_fill(t((1, 512, 1), torch.float64), UNIFORM, 3, 2, 0.5, 2.0)
    p4 = cb.mul(i4, f4.permute(0, 2, 1))
    ri, rf, rdd, rp = rt(i4), rt(f4), rt(d4), rt(p4)
    rft = rf.permute([0, 2, 1]) if ref is not None else None
    emit(4, "mul int32 x float32^T -> float32", lambda: cb.mul(i4, f4.permute(0, 2, 1)), 402653184,
         64 * 512 * 1024, lambda: ref.binary("mul", ri, rft),
         note="CPU leg: ctorch's front-door casts the int32 operand on the host first")
    emit(4, "div float32 / float64[1,512,1] -> float64", lambda: cb.div(p4, d4), 402657280,
         64 * 512 * 1024, lambda: ref.binary("div", rp, rdd))
    del i4, f4, d4, p4, ri, rf, rdd, rp, rft
    torch.cuda.empty_cache()
    # config 5, one GPU, the kernels of the step (the CPU leg runs on 32768 of the 262144 rows)
    x5 = device_fill(t((ROWS, COLS)), NORMAL, SEED, 0, 0.0, 1.0)
    r5 = device_fill(t((1, COLS)), UNIFORM, SEED, 1, -1.0, 1.0)
    y5 = cb.binary_chain("sub", "mul", x5, r5, r5)
    summer = ShardedSum(dev, 1)
    xs = ref.tensor(x5[:32768].cpu().numpy()) if ref is not None else None
    rr = rt(r5)
    ys = ref.binary("mul", ref.binary("sub", xs, rr), rr) if ref is not None else None
    n5 = ROWS * COLS
    emit(5, "sub (eager)", lambda: cb.sub(x5, r5), n5 * 8 + COLS * 4, n5, lambda: ref.binary("sub", xs, rr), 32768 * COLS)
    emit(5, "(X-r)*r one pass", lambda: cb.binary_chain("sub", "mul", x5, r5, r5), n5 * 8 + COLS * 4, n5,
         lambda: ref.binary("mul", ref.binary("sub", xs, rr), rr), 32768 * COLS)
    emit(5, "sum whole (float64 partial)", lambda: summer(y5), n5 * 4, n5, lambda: ref.reduce("sum", ys), 32768 * COLS)
    emit(5, "argmin dim=1", lambda: cb.argmin(y5, 1), n5 * 4 + ROWS * 8, n5, lambda: ref.arg("argmin", ys, 1), 32768 * COLS)
    emit(5, "chain + row argmin + sum, one pass", lambda: cb.chain_rows("sub", "mul", x5, r5, r5, out_sum=summer.partial),
         n5 * 8 + COLS * 4 + ROWS * 8, n5, lambda: (ref.reduce("sum", ys), ref.arg("argmin", ys, 1)), 32768 * COLS,
         note="CPU leg: sum and argmin of the precomputed Y sample")
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-rows", type=int, default=0, help="rows per CPU step (0 = auto)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-per-op", action="store_true",
                    help="skip the per-op table (every op of the five configurations) and the ctorch-API "
                         "timings that the default one-GPU run adds to its line")
    ap.add_argument("--case", default=None,
                    help="profiling mode: launch one kernel (chain_rows, chain, sub, sum, argmin, step, add, relu, "
                         "sum_rows, prod_rows, argmax_cols, max_cols, sum_cols, cols_bulk, cols_narrow, cols_outer, argmin_rows, "
                         "rows_short, tiled_f64, ew_general, red_runs, red_general, gather_general, index_select, mul_t, div_b) --warmup + --steps "
                         "times")
    ap.add_argument("--rows", type=int, default=16384, help="rows of X for --case (default 16384: 512 MiB)")
    ap.add_argument("--suite", action="store_true",
                    help="per-op device time, GB/s and ctorch CPU time for every op of the five configurations")
    args = ap.parse_args()
    if args.case:
        return run_case(args)
    if args.suite:
        return run_suite(args)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
