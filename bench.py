"""Benchmark: kernels emitted by compile.py on B200, against the roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --suite            # every workload once, one line each

Headline workload (one "step"): the full-reduction pair of the benchmark
configs -- sum and mean of x: f32[2^26] ~ U(-1, 1) -- each compiled from its
Kernel IR by ``compile.py``'s pipeline and launched through ``libemmyrt``.
Inputs (256 MiB) are larger than the 126 MB L2, so no flush is needed.
With N GPUs (torchrun, one process per GPU) every rank reduces its own 2^26
shard and the library's fold kernel (emmy_rt_fold_f32: peer stores over NVLink)
sums the two scalars over the ranks, giving the global sum and mean (weak
scaling); ``--collective nccl`` uses an NCCL all-reduce instead.

Printed JSON: ``value`` = algorithmic GB/s of the whole job (device-resident
inputs, CUDA events, max over ranks); ``e2e`` = the same through the C ABI with
host buffers (H2D + launches + D2H in the timed region); ``roofline`` for the
dominant kernel against the measured HBM copy bandwidth; ``cpu_baseline`` =
PyTorch CPU of the same expressions. At N = 1 ``per_config`` adds one entry per
benchmark configuration (pointwise add, sum, mean, RMSNorm, softmax, L2-norm,
both matmuls, both attentions): CUDA-event median per launch with L2 flushed
(or a working set above twice L2), fraction of the roofline, compile ms, the
kernel's error word, its largest error against an fp64 result of the same
inputs, and PyTorch CPU of the same expression.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "emmy-ir-to-ptx_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "per-kernel % of B200 roofline (HBM GB/s or TC TFLOP/s); compile ms/kernel"
N_REDUCE = 1 << 26
PER_KERNEL = 10               # steps of the per-kernel (event-bracketed) timing pass
HBM_NOMINAL_GBS = 8000.0      # B200 HBM3e nominal bandwidth, for context beside the measured peak
RES_SLOTS = 4                 # result slots: an all-reduce may lag its step by 3 steps
FOLD_SLOTS = 64               # result slots with the fold (a fold may lag its step by 63 steps)
FALLBACK_HBM_GBS = 6650.0
REF_STEP_S = 0.15             # reference arm: seconds of CPU work per step
E2E_STEPS = 30                # e2e: timed steps (median)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def ncu_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/ncu_traffic.txt)."""
    p = ROOT / "profiles" / "ncu_traffic.txt"
    if not p.is_file():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and not line.startswith("#") and parts[0] == kernel \
                and parts[1] == workload:
            return int(parts[2])
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self):
        return time.time()

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = []
        for ts, line in self.lines:
            if t0 - 0.25 <= ts <= t1 + 0.25:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].lower() in ("active", "1")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "power_w": statistics.median(pw) if pw else None, "samples": len(rows)}


# ---------------------------------------------------------------------------
# compile the workload kernels
# ---------------------------------------------------------------------------

def compile_workload(make, *, repeats=5):
    """(ptx, template, meta, kernel_meta, median in-process compile ms)."""
    from emmyptx.emit import compile_payload
    payload, meta = make()
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        ptx, template, _ = compile_payload(payload, meta)
        times.append((time.perf_counter() - t0) * 1e3)
    return ptx, template, meta, meta["kernels"][0], statistics.median(times)


def compile_process_ms(make, repeats=5):
    """Median wall time of ``python compile.py <kernel>.ir.json`` (a fresh interpreter per
    compile, as the reference contract runs it), IR and meta.json written to a temp folder."""
    import subprocess
    import tempfile
    payload, meta = make()
    with tempfile.TemporaryDirectory() as d:
        ir_path = Path(d) / f"{meta['kernels'][0]['entry']}.ir.json"
        ir_path.write_text(json.dumps(payload))
        (Path(d) / "meta.json").write_text(json.dumps(meta))
        times = []
        for _ in range(repeats + 1):
            t0 = time.perf_counter()
            subprocess.run([sys.executable, str(ROOT / "compile.py"), str(ir_path)], check=True,
                           stdout=subprocess.DEVNULL)
            times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times[1:])


# ---------------------------------------------------------------------------
# reference arm: the CPU evaluation of the same expressions
# ---------------------------------------------------------------------------

def run_reference(args, rank, world):
    """The reference arm: PyTorch CPU of the same expressions (x.sum(), x.mean()) on all host
    cores, on rank 0 only. A step is a bounded sample of the workload: back-to-back passes
    over the full x for about REF_STEP_S seconds (the same measurement as ``cpu_baseline``,
    split into ``--steps`` parts), after ``--warmup`` untimed steps."""
    if rank != 0:
        return 0
    from oracle import cpu_baseline as cb
    cores = cb.threads()
    x = cb.reduce_inputs(N_REDUCE)
    bytes_step = 2 * (4 * N_REDUCE) + 4 + 4 + 4
    for _ in range(max(args.warmup, 1)):
        cb.reduce_rate(x, REF_STEP_S)
    per_step, passes = [], 0
    for _ in range(args.steps):
        sec, n = cb.reduce_rate(x, REF_STEP_S)
        per_step.append(sec)
        passes += n
    sec = statistics.mean(per_step)
    gbs = bytes_step / sec / 1e9
    line = {
        "metric": METRIC, "impl": "reference", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config(world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"torch CPU x.sum() and x.mean() of the full x f32[2^26]: "
                                   f"{args.steps} steps of ~{REF_STEP_S} s, {passes} passes"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _config(world, grid=None, collective="fold"):
    return {"workload": "full reductions f32: sum and mean of x[2^26] ~ U(-1,1) per GPU "
                        "(benchmark config 'Full reductions in f32')",
            "n_per_gpu": N_REDUCE, "block": 256, "grid": grid,
            "l2": "inputs larger than L2 (256 MiB per pass); no flush",
            "parallelism": (f"x sharded over {world} GPU(s); the 2 scalars summed over ranks "
                            + ("by emmy_rt_fold_f32 (peer stores over NVLink)"
                               if collective == "fold" else "by an NCCL all-reduce"))
            if world > 1 else "single GPU"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def cpu_baseline_leg():
    from oracle import cpu_baseline as cb
    cores = cb.threads()
    x = cb.reduce_inputs(N_REDUCE)
    bytes_step = 2 * (4 * N_REDUCE) + 12
    sec, n = cb.reduce_rate(x, 3.0)
    return {"value": round(bytes_step / sec / 1e9, 3), "unit": "GB/s", "cores": cores,
            "kind": "port",
            "sample": f"torch CPU x.sum() and x.mean() of the full x f32[2^26], {n} steps "
                      f"(~3 s)"}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from emmyptx import runtime, workloads

    torch.cuda.set_device(local_rank)
    runtime.init(local_rank)
    dev = torch.device("cuda", local_rank)

    grid = args.grid or 4 * workloads.SM_COUNT
    ptx_s, _, _, k_s, c_s = compile_workload(
        lambda: workloads.full_reduce(N_REDUCE, "sum", grid=grid))
    # the mean divides by the global count so the all-reduce sum of shard results is the mean
    ptx_m, _, meta_m, k_m, c_m = compile_workload(
        lambda: workloads.full_reduce(N_REDUCE, "mean", grid=grid))
    mod_s = runtime.Module(ptx_s, k_s["entry"], local_rank)
    mod_m = runtime.Module(ptx_m, k_m["entry"], local_rank)

    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    x = torch.empty(N_REDUCE, device=dev, dtype=torch.float32).uniform_(-1, 1, generator=g)
    count = torch.tensor([float(N_REDUCE * world)], device=dev, dtype=torch.float32)
    fold = None
    fold_note = None
    if world > 1 and args.collective == "fold":
        fold, fold_note = _peer_fold(rank, world)
    # result slots: step i writes slot i % slots, so the exchange of step i overlaps the
    # kernels of the next steps; before a slot is written again the exchange that read it
    # has completed (an all-reduce is waited for on the stream; a fold's completion event is
    # waited for unless it has already fired), and all are settled before the stop event
    slots = FOLD_SLOTS if fold is not None else RES_SLOTS
    res = torch.zeros(slots, 2, device=dev, dtype=torch.float32)
    tot = torch.zeros(slots, 2, device=dev, dtype=torch.float32) if fold is not None else res
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    # the fold runs on a stream of its own, after an event behind each step's mean: in the
    # stream of overlapped reductions it would sit between the mean and the next sum, whose
    # writes would then wait for the slowest rank's flag (measured on 4 GPUs, us per step,
    # two boxes: no exchange 72.0 / 72.0, fold in the stream 76.0 / 73.6, fold on its own
    # stream 72.5 / 72.5; an event wait between two overlapped launches cost nothing, 72.0)
    side = torch.cuda.Stream(device=dev) if fold is not None else None
    mean_done = [torch.cuda.Event() for _ in range(slots)] if fold is not None else None
    fold_ev = [torch.cuda.Event() for _ in range(slots)] if fold is not None else None
    fold_done = [None] * slots
    grid3, block3 = k_s["grid"], k_s["block"]
    p_sum = [[x.data_ptr(), res[i].data_ptr()] for i in range(slots)]
    p_mean = [[x.data_ptr(), count.data_ptr(), res[i].data_ptr() + 4] for i in range(slots)]
    assert [a["name"] for a in k_m["args"]] == ["x", "mean_keepdim_count", "mean"]
    pending = [None] * slots
    last_fold = [None]
    align = torch.zeros(2, device=dev, dtype=torch.float32)    # the untimed aligning exchange
    overlap_ok = world == 1 or fold is not None

    def drain():
        """Every exchange issued so far completes before what is enqueued next on the stream."""
        for i, h in enumerate(pending):
            if h is not None:
                h.wait()
                pending[i] = None
        if last_fold[0] is not None:
            stream.wait_event(last_fold[0])
            last_fold[0] = None

    def step(i, ev=None, collective=True, lead=False):
        """One step: sum and mean kernels, then (N > 1) the sum of the two scalars over ranks.
        Untimed heat-up and tail steps, whose count follows the wall clock and so differs
        between ranks, skip it: every rank issues the same collectives in the same order.

        Without ``ev`` the kernels are launched to overlap their predecessor on the stream
        (programmatic stream serialization): a kernel may start once every thread of the
        previous one has streamed 7/8 of x. It reads the front of x, which the previous
        kernel read more than an L2's worth of bytes earlier, so it fills the SMs that finish
        first without sharing any line with its predecessor: x is read from HBM by each
        kernel (268 MB, twice L2).
        With N > 1 the fold kernel (emmy_rt_fold_f32, one warp) sums the scalars over ranks
        through peer stores into every rank's mailbox, on its own stream once the step's mean
        has completed; it takes no SM room the reductions need. The NCCL
        alternative (--collective nccl) runs with plain launches and an async all-reduce:
        measured at N = 2 (us per step), plain launches with it 85.5, overlapped launches with
        it 102.6 (its kernel competes for SMs with the overlapped reductions).
        With ``ev`` (the per-kernel timing pass) they are plain launches between events.
        ``lead``: the first step after the start event, whose sum starts only once everything
        before the event has completed."""
        slot = i % slots
        if pending[slot] is not None:
            pending[slot].wait()
            pending[slot] = None
        if fold_done[slot] is not None:
            if not fold_done[slot].query():          # the fold that read this slot
                stream.wait_event(fold_done[slot])
            fold_done[slot] = None
        if ev:
            ev[0].record(stream)
        overlap = not ev and overlap_ok
        mod_s.launch(grid3, block3, 0, p_sum[slot], sh, overlap=overlap and not lead)
        if ev:
            ev[1].record(stream)
        mod_m.launch(grid3, block3, 0, p_mean[slot], sh, overlap=overlap)
        if ev:
            ev[2].record(stream)
        if world > 1 and collective:
            if fold is not None:
                mean_done[slot].record(stream)
                side.wait_event(mean_done[slot])
                fold.launch(res[slot].data_ptr(), 2, tot[slot].data_ptr(), side.cuda_stream,
                            overlap=False)
                fold_done[slot] = last_fold[0] = fold_ev[slot]
                fold_done[slot].record(side)
            else:
                pending[slot] = dist.all_reduce(res[slot], async_op=True)

    # correctness of this run's result against the fp64 sum of the device data
    if world > 1:
        dist.barrier()          # the first fold: every rank's mailbox is mapped by now
    step(0)
    drain()
    torch.cuda.synchronize()
    got = tot[0].clone()
    if world > 1:
        xs = x.double().sum()
        dist.all_reduce(xs)
        want = torch.stack([xs, xs / (N_REDUCE * world)]).float()
    else:
        xs = x.double().sum()
        want = torch.stack([xs, xs / N_REDUCE]).float()
    rel = float((got.double() - want.double()).abs().max() / want.double().abs().max())
    err_word = mod_s.error_word() | mod_m.error_word()

    with ClockSampler(local_rank) as clocks:
        t_heat = time.time()
        n = 0
        while time.time() - t_heat < 0.6:           # untimed: heat up + let the sampler start
            step(n, collective=False)
            n += 1
        # per-kernel pass (untimed for `value`): plain launches, each between two events
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(PER_KERNEL)]
        for i in range(PER_KERNEL):
            step(i, evs[i], collective=False)
        if world > 1:
            dist.barrier()          # ranks enter the first fold together
        for i in range(args.warmup):
            step(i)
        drain()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        t0 = clocks.mark()
        if world > 1:
            # ranks leave the host barrier tens of microseconds apart, and the first timed
            # exchange would charge that skew to the ranks that started early: one untimed
            # exchange on the stream lines the ranks up on the device (every rank leaves it
            # within one NVLink flag round trip) and the start event follows it
            if fold is not None:
                fold.launch(res[0].data_ptr(), 2, align.data_ptr(), sh, overlap=False)
            else:
                dist.all_reduce(align)
        start.record(stream)
        h0 = time.perf_counter()
        for i in range(args.steps):
            step(i, lead=i == 0)
        host_us_step = (time.perf_counter() - h0) / args.steps * 1e6   # enqueue time only
        drain()
        stop.record(stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t1 = clocks.mark()
        # keep the GPU busy briefly so trailing samples still see load
        t_tail = time.time()
        n = 0
        while time.time() - t_tail < 0.3:
            step(n, collective=False)
            n += 1
        torch.cuda.synchronize()
    ms = ms_local = start.elapsed_time(stop)
    sum_us = [e[0].elapsed_time(e[1]) * 1e3 for e in evs]
    mean_us = [e[1].elapsed_time(e[2]) * 1e3 for e in evs]
    rank_ms = [ms]
    if world > 1:
        t = torch.zeros(world, device=dev, dtype=torch.float64)
        t[rank] = ms
        dist.all_reduce(t)                  # every rank's timed region, max taken below
        rank_ms = [round(float(v), 5) for v in t.tolist()]
        ms = max(rank_ms)
    ms_step = ms / args.steps

    bytes_sum = 4 * N_REDUCE + 4
    bytes_mean = 4 * N_REDUCE + 4 + 4
    bytes_step = (bytes_sum + bytes_mean) * world
    value = bytes_step / (ms_step * 1e-3) / 1e9

    peaks = measured_peaks()
    avg_sum_us = statistics.mean(sum_us)
    # the timed region runs 2 launches per step of the same template over the same bytes
    # (the mean reads 4 more): its average launch duration is this rank's time / launches
    launch_us = ms_local / args.steps / 2 * 1e3
    achieved = bytes_sum / (launch_us * 1e-6) / 1e9
    traffic = ncu_traffic("k_sum_1_reduce", "sum_2^26")

    # e2e through the C ABI with host buffers (H2D + launch + D2H timed per step)
    e2e = _e2e(runtime, ptx_s, k_s, ptx_m, k_m, local_rank, world, dev, fold)
    fold_err = fold.error_word() if fold is not None else 0      # every fold of this run
    if world > 1:
        # a fold whose wait ran out returns at once from then on: the timed steps of that
        # rank then exchanged nothing, so the run has no valid number on any rank
        fe = torch.tensor([float(fold_err)], device=dev, dtype=torch.float64)
        dist.all_reduce(fe, op=dist.ReduceOp.MAX)
        fold_err = int(fe.item())

    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": _config(world, grid, "fold" if fold is not None else "nccl"),
        "roofline": {"bound": "hbm", "kernel": "k_sum_1_reduce",
                     "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic, "algorithmic_bytes": bytes_sum,
                     "launch_us": round(launch_us, 3),
                     "nominal_peak": HBM_NOMINAL_GBS,
                     "frac_of_nominal": round(achieved / HBM_NOMINAL_GBS, 4),
                     "note": "peak is a read+write copy; this kernel only reads",
                     "duration": ("timed region / launches in it (each launch starts when its "
                                  "predecessor has streamed 7/8 of x; no line is read by both)")
                     if overlap_ok
                     else "timed region / launches in it (plain launches)",
                     "peak_source": f"{peaks['source']} hbm_gbs (burst copy)"},
        "kernels": {                 # plain launches, each between two events
            "k_sum_1_reduce": {"us": round(avg_sum_us, 3),
                               "gbs": round(bytes_sum / avg_sum_us / 1e3, 2),
                               "frac": round(bytes_sum / avg_sum_us / 1e3 / peaks["hbm_gbs"], 4),
                               "compile_ms": round(c_s, 2)},
            "k_mean_reduce": {"us": round(statistics.mean(mean_us), 3),
                              "gbs": round(bytes_mean / statistics.mean(mean_us) / 1e3, 2),
                              "frac": round(bytes_mean / statistics.mean(mean_us) / 1e3
                                            / peaks["hbm_gbs"], 4),
                              "compile_ms": round(c_m, 2)},
        },
        "check": {"rel_err_vs_fp64": rel, "error_word": err_word,
                  **({"fold_error_word": fold_err} if fold is not None else {}),
                  **({"fold_unavailable": fold_note} if fold_note else {})},
        "host_enqueue_us_per_step": round(host_us_step, 2),
        "rank_ms": rank_ms,          # each rank's timed region (device events); value uses the max
        "gpu_launches": (3 if fold is not None else 2) * args.steps,
        "e2e": e2e,
        "clocks": clocks.summary(t0, t1),
    }
    if fold_err:
        result["value"] = None
        result["invalid"] = (f"emmy_rt_fold_f32 error word {fold_err:#x}: a fold's bounded wait "
                             "ran out, so later steps exchanged nothing between ranks")
    if rank == 0 and world == 1:
        result["per_config"] = per_config(args, peaks, local_rank)
        result["cpu_baseline"] = cpu_baseline_leg()
    if rank == 0:
        print(json.dumps(result), flush=True)
    mod_s.close()
    mod_m.close()
    if fold is not None:
        fold.close()
    return 1 if fold_err else 0


def _e2e(runtime, ptx_s, k_s, ptx_m, k_m, local_rank, world, dev, fold=None):
    """End to end through the C ABI with a pinned host buffer: every step copies x (and the
    count) host -> device once (emmy_rt_memcpy_htod), launches the sum and the mean kernels on
    it (emmy_rt_launch), with N > 1 sums the two scalars over the ranks (emmy_rt_fold_f32,
    when the fold is set up), and reads both results back (emmy_rt_memcpy_dtoh, which waits
    for the kernels). Wall-clock median over the steps; max over ranks. Every rank runs the
    same number of steps, so the folds pair up."""
    import ctypes

    import numpy as np
    n = N_REDUCE
    lib = runtime.lib()
    hp = ctypes.c_void_p()
    runtime.check(lib.emmy_rt_host_alloc(4 * n + 4, ctypes.byref(hp)))
    d_x = runtime.DeviceBuffer(4 * n)
    d_cnt = runtime.DeviceBuffer(4)
    d_res = runtime.DeviceBuffer(8)
    d_tot = runtime.DeviceBuffer(8)
    ms = runtime.Module(ptx_s, k_s["entry"], local_rank)
    mm = runtime.Module(ptx_m, k_m["entry"], local_rank)
    try:
        host = np.ctypeslib.as_array((ctypes.c_float * (n + 1)).from_address(hp.value))
        host[:n] = np.random.default_rng(7).uniform(-1, 1, n).astype(np.float32)
        host[n] = float(n * world)
        res = np.zeros(2, np.float32)
        grid, block = k_s["grid"], k_s["block"]

        def step():
            runtime.check(lib.emmy_rt_memcpy_htod(d_x.ptr, hp.value, 4 * n))
            runtime.check(lib.emmy_rt_memcpy_htod(d_cnt.ptr, hp.value + 4 * n, 4))
            ms.launch(grid, block, 0, [d_x.ptr, d_res.ptr])
            mm.launch(grid, block, 0, [d_x.ptr, d_cnt.ptr, d_res.ptr + 4])
            if fold is not None:
                fold.launch(d_res.ptr, 2, d_tot.ptr, 0, overlap=False)
                runtime.check(lib.emmy_rt_memcpy_dtoh(res.ctypes.data, d_tot.ptr, 8))
            else:
                runtime.check(lib.emmy_rt_memcpy_dtoh(res.ctypes.data, d_res.ptr, 8))

        if world > 1:
            import torch.distributed as dist
            dist.barrier()      # pinned allocation and fill take different times per rank
        for _ in range(2):
            step()
        times = []
        for _ in range(E2E_STEPS):
            t0 = time.perf_counter()
            step()
            times.append((time.perf_counter() - t0) * 1e6)
        want = float(np.sum(host[:n], dtype=np.float64))
        n_sum = n
        if fold is not None:             # every rank streamed the same host data
            want *= world
            n_sum *= world
        # the reduction tolerance of the tests: 1e-5 relative plus 1e-5 * sqrt(terms), the
        # scale of f32 rounding over n terms of magnitude <= 1 (this x sums to about -159)
        tol = 1e-5 * max(abs(want), 1.0) + 1e-5 * n_sum ** 0.5
        err = abs(float(res[0]) - want)
        ok = err <= tol
    finally:
        ms.close()
        mm.close()
        for b in (d_x, d_cnt, d_res, d_tot):
            b.free()
        lib.emmy_rt_host_free(hp)
    us = statistics.median(times)
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.tensor([us], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
    bytes_step = (2 * 4 * n + 12) * world
    return {"value": round(bytes_step / (us * 1e-6) / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": 4 * n + 4, "d2h_bytes_per_step": 8,
            "api": "C ABI: emmy_rt_memcpy_htod (pinned host buffer, one copy of x per step for "
                   "both kernels) + 2 x emmy_rt_launch"
                   + (" + emmy_rt_fold_f32 (sum over ranks)" if fold is not None else "")
                   + " + emmy_rt_memcpy_dtoh",
            "e2e_us": round(us, 3), "result_check": bool(ok),
            "result_abs_err": float(f"{err:.3g}"), "result_tol": float(f"{tol:.3g}")}


# ---------------------------------------------------------------------------
# per configuration: every benchmark workload once (device-resident, L2 flushed)
# ---------------------------------------------------------------------------

TENSOR_DENOM = "bf16_tflops / 2 / 3"   # dense TF32 is half the bf16 rate; 3xTF32 = 3 products
# workload -> its row in profiles/ncu_traffic.txt (DRAM bytes per launch from one ncu capture)
TRAFFIC_KEY = {"add": "add_2^20", "sum": "sum_2^26", "mean": "mean_2^26",
               "rmsnorm": "rmsnorm_8192x4096", "softmax": "softmax_8192x4096",
               "l2norm": "l2norm_8192x4096", "matmul_sq": "matmul_4096",
               "matmul_rect": "matmul_8192x2048x4096"}


def tf32x3_ceiling(peaks):
    """The contraction roofline: the measured dense bf16 GEMM rate / 2 (TF32) / 3 (3xTF32)."""
    return peaks["bf16_tflops"] / 2.0 / 3.0


def _algorithmic(name, k):
    """(work per launch, unit, bound) of a benchmark workload from its argument shapes."""
    import numpy as np
    shp = {a["name"]: a["shape"] for a in k["args"]}
    if name.startswith("matmul"):
        (M, K_), (_, N) = shp["x0"], shp["x1"]
        return 2.0 * M * N * K_, "FLOP", "tensor"
    if name.startswith("attention"):
        Bq, Hq, Sq, D = shp["q"]
        return 4.0 * Bq * Hq * Sq * shp["kt"][-1] * D, "FLOP", "tensor"
    return float(sum(4 * int(np.prod(a.get("shape") or [1])) for a in k["args"])), "B", "hbm"


def fp64_error(name, inputs, got, device):
    """Largest error of ``got`` against the fp64 result of the same inputs, computed on the GPU
    in float64 with torch (a checker beside the measurement, not part of the timed path).

    Row normalisations and sums: the largest element-wise relative error |got - ref| / |ref|
    (bound 1e-5). Contractions: the largest |got - ref| / (|ref| + row max|ref|) (bound 1e-4).
    Pointwise add: the number of elements that differ from the f32 sum (bound 0)."""
    import numpy as np
    import torch

    def t64(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device, torch.float64)
    g = t64(got)
    if name == "add":
        want = torch.from_numpy(inputs["x0"] + inputs["x1"]).to(device)
        diff = int((torch.from_numpy(got).to(device) != want).sum().item())
        return {"form": "elements differing from f32 x0 + x1", "value": diff, "bound": 0,
                "ok": diff == 0}
    if name in ("sum", "mean", "rmsnorm", "softmax", "l2norm"):
        x = t64(inputs["x"])
        if name == "sum":
            ref = x.sum().reshape(1)
        elif name == "mean":
            ref = x.mean().reshape(1)
        elif name == "rmsnorm":
            ref = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6) * t64(inputs["w"])
        elif name == "softmax":
            ref = torch.softmax(x, -1)
        else:
            ref = x / torch.clamp(x.norm(dim=-1, keepdim=True), min=1e-12)
        g = g.reshape(ref.shape)
        err = float(((g - ref).abs() / ref.abs()).max().item())
        return {"form": "max |got - ref| / |ref| (element-wise)", "value": float(f"{err:.3e}"),
                "bound": 1e-5, "ok": err <= 1e-5}
    if name.startswith("matmul"):
        ref = t64(inputs["x0"]) @ t64(inputs["x1"])
        refs = [(g.reshape(ref.shape), ref)]
    else:
        c = float(inputs["div_c1"].reshape(-1)[0])
        q, kt, v = inputs["q"], inputs["kt"], inputs["v"]
        g = g.reshape(q.shape)
        refs = []
        for b in range(q.shape[0]):       # one batch entry (all heads) at a time
            s_ = torch.softmax((t64(q[b]) @ t64(kt[b])) / c, -1)
            refs.append((g[b], s_ @ t64(v[b])))
    err = 0.0
    for gb, rb in refs:
        rowmax = rb.abs().amax(-1, keepdim=True)
        err = max(err, float(((gb - rb).abs() / (rb.abs() + rowmax)).max().item()))
    return {"form": "max |got - ref| / (|ref| + row max|ref|)", "value": float(f"{err:.3e}"),
            "bound": 1e-4, "ok": err <= 1e-4}


def measure_config(name, args, peaks, l2, flush, *, device=0, compile_repeats=5,
                   process_repeats=3, cpu=True, check=True):
    """One benchmark workload: compile it (in-process median and ``python compile.py``
    process time), run it once on the seeded inputs for the fp64 check, then time ``steps``
    launches with CUDA events (L2 flushed by a 256 MiB memset before each launch unless the
    working set is above twice L2, in which case it streams from HBM anyway)."""
    import numpy as np
    from emmyptx import runtime, workloads
    from emmyptx.inputs import kernel_inputs
    ptx, template, meta, k, cms = compile_workload(workloads.WORKLOADS[name],
                                                   repeats=compile_repeats)
    proc_ms = compile_process_ms(workloads.WORKLOADS[name], repeats=process_repeats) \
        if process_repeats else None
    mod = runtime.Module(ptx, k["entry"], device)
    inputs = kernel_inputs(k)
    bufs, outs, footprint = [], {}, 0
    for a in k["args"]:
        shape = tuple(a.get("shape") or (1,))
        nbytes = 4 * int(np.prod(shape))
        footprint += nbytes
        if a.get("output"):
            b = runtime.DeviceBuffer(nbytes)
            b.zero()
            outs[a["name"]] = (b, shape)
        else:
            b = runtime.DeviceBuffer.from_array(inputs[a["name"]])
        bufs.append(b)
    ptrs = [b.ptr for b in bufs]
    work, unit, bound = _algorithmic(name, k)
    entry = {"entry": k["entry"], "template": template, "grid": k["grid"][0],
             "block": k["block"][0], "smem_bytes": k.get("smem_bytes", 0),
             "registers": mod.attrs()["registers"]}
    try:
        if check:
            mod.launch(k["grid"], k["block"], k.get("smem_bytes", 0), ptrs)
            runtime.sync()
            (b, shape), = outs.values()
            got = b.download(np.zeros(shape, np.float32))
            entry["fp64_check"] = fp64_error(name, inputs, got, f"cuda:{device}")
        do_flush = footprint < 2 * l2
        ms = mod.time(k["grid"], k["block"], k.get("smem_bytes", 0), ptrs,
                      iters=args.steps, warmup=args.warmup,
                      flush_ptr=flush.ptr if do_flush else 0,
                      flush_bytes=flush.nbytes if do_flush else 0)
        entry["error_word"] = mod.error_word()
        maps = mod.tensor_maps()
        if maps["maps"]:
            # which tile loads the timed launches used: bit 0 TMA, bit 1 registers
            word = mod.path_word()
            entry["tile_loads"] = {1: "tma", 2: "registers"}.get(word, f"mixed {word:#x}")
    finally:
        mod.close()
        for b in bufs:
            b.free()
    us = statistics.median(ms) * 1e3
    entry.update({"us_median": round(us, 3), "us_min": round(min(ms) * 1e3, 3),
                  "launches": args.steps, "l2_flush": do_flush,
                  "compile_ms": round(cms, 2)})
    if "griddepcontrol.launch_dependents" in ptx:
        ov = _overlapped(ptx, k, inputs, footprint, l2, device, max(4 * args.steps, 50))
        ov["frac"] = round(ov["gbs"] / peaks["hbm_gbs"], 4)
        entry["overlapped"] = ov
    if proc_ms is not None:
        entry["compile_process_ms"] = round(proc_ms, 1)
    traffic = ncu_traffic(k["entry"], TRAFFIC_KEY.get(name, name))
    if bound == "hbm":
        gbs = work / (us * 1e-6) / 1e9
        entry["roofline"] = {"bound": "hbm", "algorithmic_bytes": int(work), "traffic": traffic,
                             "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                             "peak_source": f"{peaks['source']} hbm_gbs (burst copy)"}
    else:
        tfl = work / (us * 1e-6) / 1e12
        ceil = tf32x3_ceiling(peaks)
        entry["roofline"] = {"bound": "tensor", "algorithmic_flops": work, "traffic": traffic,
                             "achieved": round(tfl, 2), "peak": round(ceil, 1),
                             "unit": "TFLOP/s", "frac": round(tfl / ceil, 4),
                             "peak_source": f"{peaks['source']} {TENSOR_DENOM}"}
    if cpu:
        from oracle import cpu_baseline as cb
        entry["cpu_baseline"] = cb.workload_baseline(
            name, inputs, algorithmic=work, unit="GB/s" if bound == "hbm" else "TFLOP/s")
    return entry


def _overlapped(ptx, k, inputs, footprint, l2, device, launches):
    """Back-to-back launches of a kernel that takes overlapped launches (pointwise, rows, full
    sums) with programmatic stream serialization (``EMMY_RT_LAUNCH_OVERLAP``): each launch may
    be scheduled while the previous one runs and orders its memory accesses after it
    (``griddepcontrol.wait``). The launches cycle over enough copies of the buffers to cover
    twice L2, so every launch reads its inputs from HBM. Time per launch = the event-timed
    region over the launches."""
    import numpy as np
    import torch
    from emmyptx import runtime
    sets = max(2, -(-2 * l2 // footprint))
    smem = k.get("smem_bytes", 0)
    mod = runtime.Module(ptx, k["entry"], device)
    bufs = []
    try:
        ptr_sets = []
        for _ in range(sets):
            ptrs = []
            for a in k["args"]:
                if a.get("output"):
                    b = runtime.DeviceBuffer(4 * int(np.prod(a.get("shape") or [1])))
                else:
                    b = runtime.DeviceBuffer.from_array(inputs[a["name"]])
                bufs.append(b)
                ptrs.append(b.ptr)
            ptr_sets.append(ptrs)
        stream = torch.cuda.current_stream(device)
        sh = stream.cuda_stream
        for i in range(2 * sets):                              # warm-up
            mod.launch(k["grid"], k["block"], smem, ptr_sets[i % sets], sh, overlap=True)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(launches):
            mod.launch(k["grid"], k["block"], smem, ptr_sets[i % sets], sh, overlap=True)
        e1.record(stream)
        torch.cuda.synchronize(device)
        us = e0.elapsed_time(e1) * 1e3 / launches
        err = mod.error_word()
    finally:
        mod.close()
        for b in bufs:
            b.free()
    return {"us_per_launch": round(us, 3), "launches": launches, "rotating_sets": sets,
            "gbs": round(footprint / (us * 1e-6) / 1e9, 1), "error_word": err,
            "note": "back-to-back launches with programmatic stream serialization over "
                    f"{sets} buffer sets (> 2 x L2): launch cost overlapped, inputs from HBM"}


def per_config(args, peaks, device=0):
    """Every benchmark configuration once on this GPU (``measure_config``)."""
    from emmyptx import runtime, workloads
    l2 = runtime.device_info(device)["l2_bytes"]
    flush = runtime.DeviceBuffer(256 << 20)
    out = {}
    try:
        for name in workloads.WORKLOADS:
            out[name] = measure_config(name, args, peaks, l2, flush, device=device)
    finally:
        flush.free()
    return out


# ---------------------------------------------------------------------------
# suite: one line per workload (device-resident, L2 flushed between launches)
# ---------------------------------------------------------------------------

def run_suite(args):
    """One line per workload: ``measure_config`` (timing, roofline, compile ms, fp64 check,
    CPU baseline), plus the fixed cost of an empty kernel under the same launch for the
    memory-bound ones and the reference compiler's PTX of the same computation."""
    from emmyptx import runtime, workloads
    runtime.init(0)
    ref_variants = _reference_ptx_variants()
    peaks = measured_peaks()
    l2 = runtime.device_info(0)["l2_bytes"]
    flush = runtime.DeviceBuffer(256 << 20)
    names = args.only.split(",") if args.only else list(workloads.WORKLOADS)
    for name in names:
        line = {"workload": name}
        line.update(measure_config(name, args, peaks, l2, flush, compile_repeats=20,
                                   process_repeats=5, cpu=not args.no_cpu))
        if line["roofline"]["bound"] == "hbm":
            k = workloads.WORKLOADS[name]()[1]["kernels"][0]
            line["launch_floor_us"] = round(_empty_kernel_us(k, len(k["args"]), args, flush), 3)
        if name in ref_variants:
            line["reference_ptx"] = _time_reference_ptx(ref_variants[name], line["us_median"],
                                                        args, flush, l2)
        print(json.dumps(line), flush=True)


def run_suite_sharded(args, rank, world, local_rank):
    """``--suite`` under torchrun: every rank runs its shard of each workload (the IR at the
    shard's extent, see emmyptx/shard.py) on its own GPU; a workload's time is the slowest
    rank's median, and its throughput the whole configuration's work over that time (strong
    scaling: the problem stays the configuration's as N grows). The sum and mean add the
    measured exchange of their scalar, the one exchange those shards need: the peer-memory
    fold (emmy_rt_fold_f32) or, with --collective nccl, an NCCL all-reduce."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from emmyptx import runtime, shard, workloads
    from emmyptx.emit import compile_payload
    from emmyptx.inputs import kernel_inputs
    torch.cuda.set_device(local_rank)
    runtime.init(local_rank)
    dev = torch.device("cuda", local_rank)
    peaks = measured_peaks()
    l2 = runtime.device_info(local_rank)["l2_bytes"]
    flush = runtime.DeviceBuffer(256 << 20)
    names = args.only.split(",") if args.only else list(workloads.WORKLOADS)
    fold = None
    if args.collective == "fold":
        fold, _ = _peer_fold(rank, world)
        fold_buf = torch.zeros(2, device=dev)
    for name in names:
        sh = shard.shard_workload(name, world, rank)
        ptx, template, _ = compile_payload(sh.payload, sh.meta)
        k = sh.meta["kernels"][0]
        mod = runtime.Module(ptx, k["entry"], local_rank)
        inputs = kernel_inputs(k)
        bufs, total = [], 0
        for a in k["args"]:
            nbytes = 4 * int(np.prod(a.get("shape") or [1]))
            total += nbytes
            b = runtime.DeviceBuffer(nbytes)
            if a.get("output"):
                b.zero()
            else:
                b.upload(inputs[a["name"]])
            bufs.append(b)
        do_flush = total < 2 * l2
        dist.barrier()
        ms = mod.time(k["grid"], k["block"], k.get("smem_bytes", 0), [b.ptr for b in bufs],
                      iters=args.steps, warmup=args.warmup,
                      flush_ptr=flush.ptr if do_flush else 0,
                      flush_bytes=flush.nbytes if do_flush else 0)
        us = statistics.median(ms) * 1e3
        err = mod.error_word()
        path = mod.path_word() if mod.tensor_maps()["maps"] else 0
        mod.close()
        for b in bufs:
            b.free()
        combine_us = 0.0
        if sh.combine == "sum":                   # the scalar exchange, timed on its own
            t = torch.zeros(1, device=dev)
            cs = torch.cuda.current_stream(dev).cuda_stream

            def combine():
                if fold is not None:         # plain launches: each waits for every rank
                    fold.launch(fold_buf.data_ptr(), 1, fold_buf.data_ptr() + 4, cs,
                                overlap=False)
                else:
                    dist.all_reduce(t)
            for _ in range(3):
                combine()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                combine()
            e1.record()
            torch.cuda.synchronize()
            combine_us = e0.elapsed_time(e1) * 1e3 / 20
        stats = torch.tensor([us + combine_us, us, combine_us, float(err), float(path)],
                             device=dev, dtype=torch.float64)
        every = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(every, stats)
        if rank != 0:
            continue
        per_rank = [float(v[0]) for v in every]
        t_us = max(per_rank)
        whole = workloads.WORKLOADS[name]()[1]["kernels"][0]
        line = {"workload": name, "n_gpus": world, "scaling": "strong", "template": template,
                "us_max_over_ranks": round(t_us, 3),
                "us_per_rank": [round(v, 3) for v in per_rank],
                "kernel_us_per_rank": [round(float(v[1]), 3) for v in every],
                "combine_us": round(float(every[0][2]), 3) if sh.combine else None,
                "combine": (("emmy_rt_fold_f32" if fold is not None else "NCCL all-reduce")
                            if sh.combine else None),
                "error_words": [int(v[3]) for v in every],
                **({"tile_loads_per_rank": [{1: "tma", 2: "registers"}.get(int(v[4]), int(v[4]))
                                            for v in every]} if any(int(v[4]) for v in every)
                   else {}),
                "shard_units": list(sh.units), "l2_flush": do_flush}
        shp = {a["name"]: a["shape"] for a in whole["args"]}
        if name.startswith("matmul") or name.startswith("attention"):
            if name.startswith("matmul"):
                (M, K_), (_, N) = shp["x0"], shp["x1"]
                flops = 2.0 * M * N * K_
            else:
                Bq, Hq, Sq, D = shp["q"]
                flops = 4.0 * Bq * Hq * Sq * shp["kt"][-1] * D
            line.update({"algorithmic_flops": flops,
                         "tflops_aggregate": round(flops / (t_us * 1e-6) / 1e12, 2)})
        else:
            alg = sum(4 * int(np.prod(a.get("shape") or [1])) for a in whole["args"])
            gbs = alg / (t_us * 1e-6) / 1e9
            line.update({"algorithmic_bytes": alg, "gbs_aggregate": round(gbs, 1),
                         "frac_of_n_hbm": round(gbs / (world * peaks["hbm_gbs"]), 4)})
        print(json.dumps(line), flush=True)
    if fold is not None:
        fold_err = fold.error_word()
        dist.barrier()
        fold.close()
        if fold_err:
            raise RuntimeError(f"emmy_rt_fold_f32 error word {fold_err} on rank {rank}")
    return 0


def _peer_fold(rank, world):
    """(PeerFold, None), or (None, reason) on every rank alike when some rank could not make
    or map a mailbox; the caller then sums the scalars with the NCCL all-reduce."""
    import torch.distributed as dist
    from emmyptx.fold import FoldUnavailable, PeerFold

    def gather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out
    try:
        return PeerFold(rank, world, gather), None
    except FoldUnavailable as e:
        return None, str(e)


def _distributed(local_rank, fn):
    """Run ``fn`` inside an NCCL process group bound to this rank's GPU."""
    import datetime

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    try:
        return fn()
    finally:
        dist.destroy_process_group()


REF_PTX_DIR = ROOT / "tests" / "golden" / "ref_ptx"


def run_fixtures(args):
    """One line per fixture (the reference's own problems): our PTX and the reference
    compiler's PTX (JIT-compiled for this GPU) timed under the fixture's meta.json launch on
    the same buffers, L2 flushed before each launch (the fixtures are far smaller than L2)."""
    import numpy as np
    from emmyptx import runtime
    from emmyptx.emit import PTXEmitter
    from emmyptx.inputs import kernel_inputs
    runtime.init(0)
    flush = runtime.DeviceBuffer(256 << 20)
    problems = ROOT / "tests" / "golden" / "problems"
    for pdir in sorted(p for p in problems.iterdir() if (p / "meta.json").is_file()):
        meta = json.loads((pdir / "meta.json").read_text())
        k = meta["kernels"][0]
        em = PTXEmitter()
        t0 = time.perf_counter()
        ours = em.compile_ptx(str(pdir / f"{k['entry']}.ir.json"))
        cms = (time.perf_counter() - t0) * 1e3
        template = em.last_template
        inputs = kernel_inputs(k)
        bufs = []
        for a in k["args"]:
            shape = tuple(a.get("shape") or (1,))
            b = runtime.DeviceBuffer(4 * int(np.prod(shape)))
            if a.get("output"):
                b.zero()
            else:
                b.upload(inputs[a["name"]])
            bufs.append(b)
        times = {}
        for tag, ptx in (("ours", ours), ("reference", (REF_PTX_DIR / f"{pdir.name}.ptx")
                                          .read_text())):
            mod = runtime.Module(ptx, k["entry"])
            ms = mod.time(k["grid"], k["block"], k.get("smem_bytes", 0), [b.ptr for b in bufs],
                          iters=max(args.steps, 20), warmup=args.warmup, flush_ptr=flush.ptr,
                          flush_bytes=flush.nbytes)
            times[tag] = statistics.median(ms) * 1e3
            mod.close()
        for b in bufs:
            b.free()
        print(json.dumps({"fixture": pdir.name, "entry": k["entry"], "template": template,
                          "grid": k["grid"][0], "block": k["block"][0],
                          "us_ours": round(times["ours"], 3),
                          "us_reference_ptx": round(times["reference"], 3),
                          "speedup": round(times["reference"] / times["ours"], 2),
                          "compile_ms": round(cms, 2)}), flush=True)
    return 0


def _empty_kernel_us(k, nparams, args, flush):
    """Median event-timed duration of an empty kernel with the same launch geometry and
    the same L2 flush: the fixed cost (launch, CTA dispatch, events) inside every number
    of this suite, which dominates the small configurations."""
    from emmyptx import runtime
    params = ", ".join(f".param .u64 p{i}" for i in range(nparams))
    ptx = (".version 8.8\n.target sm_100a\n.address_size 64\n"
           f".visible .entry k_empty({params})\n{{\nret;\n}}\n")
    mod = runtime.Module(ptx, "k_empty")
    ms = mod.time(k["grid"], k["block"], k.get("smem_bytes", 0), [0] * nparams,
                  iters=max(20, args.steps), warmup=3, flush_ptr=flush.ptr,
                  flush_bytes=flush.nbytes)
    mod.close()
    return statistics.median(ms) * 1e3


def _reference_ptx_variants():
    """benchmark workload -> (variant name, its manifest entry) for the reference compiler's
    PTX of the same computation (in the form its lowerers accept)."""
    path = REF_PTX_DIR / "MANIFEST.json"
    if not path.is_file():
        return {}
    entries = json.loads(path.read_text())["entries"]
    return {e["mirrors"]: (n, e) for n, e in entries.items() if e["source"] == "workload"}


def _time_reference_ptx(variant, our_us, args, flush, l2):
    """Time the reference compiler's PTX (JIT-compiled for this GPU) on its variant of the
    workload. The rank-2 attention slice covers one (batch, head); its time is multiplied by
    the number of heads of the benchmark configuration."""
    import numpy as np
    from emmyptx import runtime, workloads
    from emmyptx.inputs import kernel_inputs
    name, e = variant
    fn, a, kw = e["call"]
    _, meta = getattr(workloads, fn)(*a, **kw)
    k = meta["kernels"][0]
    mod = runtime.Module((REF_PTX_DIR / f"{name}.ptx").read_text(), k["entry"])
    inputs = kernel_inputs(k)
    bufs, alg = [], 0
    for arg in k["args"]:
        shape = tuple(arg.get("shape") or (1,))
        nbytes = 4 * int(np.prod(shape))
        alg += nbytes
        b = runtime.DeviceBuffer(nbytes)
        if arg.get("output"):
            b.zero()
        else:
            b.upload(inputs[arg["name"]])
        bufs.append(b)
    do_flush = alg < 2 * l2
    iters = max(3, min(args.steps, 10))
    ms = mod.time(k["grid"], k["block"], k.get("smem_bytes", 0), [b.ptr for b in bufs],
                  iters=iters, warmup=1, flush_ptr=flush.ptr if do_flush else 0,
                  flush_bytes=flush.nbytes if do_flush else 0)
    mod.close()
    for b in bufs:
        b.free()
    per_launch = statistics.median(ms) * 1e3
    launches = 1
    if fn == "attention_rows":
        mq = workloads.WORKLOADS[e["mirrors"]]()[1]["kernels"][0]
        shape = next(x["shape"] for x in mq["args"] if x["name"] == "q")
        launches = shape[0] * shape[1]
    total = per_launch * launches
    return {"variant": name, "us": round(total, 3), "us_per_launch": round(per_launch, 3),
            "launches": launches, "speedup": round(total / our_us, 2),
            "note": "reference compile.py PTX (.target sm_89) JIT-run on this GPU"
                    + (f"; {launches} rank-2 (batch, head) launches" if launches > 1 else "")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--grid", type=int, default=0, help="CTAs of the reduction kernels")
    ap.add_argument("--suite", action="store_true")
    ap.add_argument("--fixtures", action="store_true",
                    help="time every fixture: ours against the reference compiler's PTX")
    ap.add_argument("--only", default="")
    ap.add_argument("--no-cpu", action="store_true",
                    help="--suite: skip the per-workload PyTorch CPU baseline")
    ap.add_argument("--collective", choices=("fold", "nccl"), default="fold",
                    help="N > 1: sum the per-rank scalars with the peer-memory fold kernel "
                         "(overlapped launches) or an async NCCL all-reduce (plain launches)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.fixtures:
        return run_fixtures(args)
    if args.suite:
        if world > 1:
            return _distributed(local_rank, lambda: run_suite_sharded(args, rank, world,
                                                                      local_rank))
        return run_suite(args)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        return _distributed(local_rank, lambda: run_ours(args, rank, world, local_rank))
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
