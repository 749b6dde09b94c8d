#!/usr/bin/env python
"""Throughput benchmark: aligned frames/s of the B200-native CTC aligner.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--mode optimized|conventional]
                    [--impl ours|reference|reference-cuda]

One step = one ``align`` call over one synthetic batch of benchmark
configuration C (default cfg1, the configuration the 1-GPU metric is quoted
on).  Under torchrun each rank aligns its own independent batch of that shape
on its own GPU (records are independent: no collective on the data path;
weak scaling).
With --split every rank draws the same batch and aligns its share of a
length-balanced partition of its records instead (strong scaling: the
multi-GPU configuration's whole-box measurement).

impl=ours            this package: device-resident timing (``value``), an
                     end-to-end host->device->host timing (``e2e``), the live
                     roofline of the DP forward kernel and a CPU baseline.
impl=reference       the reference's own CPU implementation of the path (its
                     corrected C++ comparator, compiled in place into
                     oracle/_ref) on all host threads; rank 0 only.
impl=reference-cuda  the reference's own CUDA extension (oracle/_ref) on the
                     same device-resident batch, timed like ``value``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20   # > 126 MB L2
E2E_MIN_SECONDS = 0.25       # the end-to-end loop's least duration
E2E_MAX_STEPS = 4000
# Phase boundaries recorded by ffa_profile_phase_events (include/ffa_b200.h).
PHASES = ("first_pass", "finish", "fill")
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--config", type=int, default=1)
    p.add_argument("--mode", default="optimized", choices=["optimized", "conventional"])
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-cuda"])
    p.add_argument("--scale", type=float, default=1.0,
                   help="shrink the config's record count (and cfg2's frames) for small profiling runs")
    p.add_argument("--split", action="store_true",
                   help="partition one batch over the ranks (strong scaling) instead of one batch per rank")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="CPU work in the cpu_baseline sample")
    p.add_argument("--route", default="auto", choices=["auto", "pieces", "window"],
                   help="optimized mode's route for the device-resident timing (align's route=)")
    p.add_argument("--input", default="log-probs", choices=["log-probs", "logits-f32", "logits-bf16"],
                   help="what the batch holds: fp32 log-probabilities (the reference's input), or a "
                        "model's logits aligned as their log_softmax inside the kernels (from_logits)")
    args = p.parse_args()
    if args.warmup < 3:
        p.error("--warmup must be >= 3")
    return args


# ---------------------------------------------------------------- utilities

def rank_info():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(wl, element_bytes=4):
    """The path's algorithmic bytes: 32 B for every sector of a row holding a label column
    of the record (sectors counted from a 32 B-aligned record base), plus 12 B
    of output per frame and the 8 B int64 targets.  Returns (emission+target
    bytes read by the DP, full B_alg)."""
    read = 0
    out = 0
    per_sector = 32 // element_bytes
    for i in range(wl.batch):
        e, t = wl.record(i)
        T, V = e.shape
        cols = np.unique(np.r_[t, wl.blank])
        per_residue = np.array([np.unique((r + cols) // per_sector).size for r in range(per_sector)])
        residues = (np.arange(T, dtype=np.int64) * V) % per_sector
        read += 32 * int(per_residue[residues].sum()) + 8 * t.size
        out += 12 * T
    return read, read + out


def from_profile(config_name, key):
    """A per-launch figure of the first pass (`key: value`) from the committed
    ncu summary of that workload, if any: traffic_bytes_per_launch (dram
    bytes read + written) or warp_instructions_per_launch."""
    path = ROOT / "profiles" / f"ffa_viterbi_forward_{config_name}.md"
    if not path.exists():
        return None
    m = re.search(key + r":\s*([0-9.eE+]+)", path.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ["clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device_index):
        self.proc = None
        self.device = device_index

    def __enter__(self):
        import torch
        try:
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            target = str(self.device)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", target, f"--query-gpu={','.join(self.FIELDS)}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.samples = []
        if self.proc is None:
            return False
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(self.FIELDS):
                self.samples.append(parts)
        return False

    def summary(self):
        if not getattr(self, "samples", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for s in self.samples for k in range(4) if s[3 + k] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ------------------------------------------------------------ CPU baselines

def validity_scan_roofline(ffa, e_dev, frame_list, vocab, warmup, min_bytes=512 << 20):
    """The path's HBM-bound kernel: emission_validity (a NaN/+inf scan) over
    the batch's emissions repeated past min_bytes (larger than L2), timed
    with CUDA events.  A sleep kernel queued ahead keeps the device busy
    while the host prepares the call, so the events bracket device work only.
    Returns the scanned bytes, the device time and the GB/s."""
    import torch
    reps = max(1, -(-min_bytes // (e_dev.numel() * 4)))
    big = e_dev.repeat(reps, 1)
    views = list(big.split(frame_list * reps))
    for _ in range(warmup):
        ffa.emission_validity(views)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(5):
        torch.cuda.synchronize()
        torch.cuda._sleep(20_000_000)  # ~10 ms of device time ahead of the call
        a.record()
        valid = ffa.emission_validity(views)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    nbytes = big.numel() * 4
    ok = bool(valid.all().item())
    del big, views
    return {"kernel": "ffa_validity_scan", "bytes": nbytes, "records": len(frame_list) * reps,
            "ms": ms, "achieved": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s", "all_valid": ok}


def unfused_logits_ms(ffa, e_dev, t_dev, wl, args, flush):
    """Device time per step of what a caller without fused logits runs:
    torch.log_softmax in fp32, then the align on the materialised
    log-probabilities; queued and flushed as the value loop is."""
    import torch

    def step():
        emissions = torch.log_softmax(e_dev.float(), dim=-1)
        return ffa.align_packed(emissions, wl.lengths, t_dev, wl.target_lengths, blank_id=wl.blank, mode=args.mode)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(20_000_000)
    for a, b in evs:
        flush.zero_()
        a.record()
        step()
        b.record()
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / args.steps


def queued_device_ms(call, steps, warmup, flush):
    """Device time of `call` per step, timed as the value loop: `warmup`
    untimed calls, then `steps` calls queued back to back (no host sync),
    the L2 flushed on the device before each, CUDA events around each call.
    Returns the list of per-step milliseconds."""
    import torch
    for _ in range(warmup):
        flush.zero_()
        call()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        a.record(); b.record()
    torch.cuda.synchronize()
    torch.cuda._sleep(20_000_000)
    for a, b in evs:
        flush.zero_()
        a.record()
        call()
        b.record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def reference_cuda_lane(wl, e_dev, t_dev, steps, warmup, flush):
    """The reference's own CUDA extension (compiled in place from its
    alignment.cu into oracle/_ref) on the same device-resident batch, both
    modes, timed exactly like `value`; None if it is not built."""
    from oracle import oracle
    if not oracle.load_reference_cuda():
        return None
    if (2 * wl.target_lengths + 1 > 4096).any():
        return {"unavailable": "the reference's align rejects transcripts above 2047 tokens "
                               "(alignment.cu:684, max_states <= 4096)"}
    es = list(e_dev.split(wl.lengths.tolist()))
    ts = list(t_dev.split(wl.target_lengths.tolist()))
    blanks = [wl.blank] * wl.batch
    frames = int(wl.lengths.sum())
    out = {}
    for mode in ("optimized", "conventional"):
        ms = queued_device_ms(lambda: oracle.reference_cuda_align(es, ts, blanks, mode=mode, check_inputs=True),
                              steps, warmup, flush)
        out[mode] = {"value": frames * steps / (sum(ms) / 1e3), "ms_per_step": sum(ms) / steps}
    return out


def window_records(wl, sms, route="auto"):
    """Which records the library's route policy gives the window route
    (window_policy, ffa_host.cpp): row-staged (V <= 64, 16-byte rows), at most
    4096 states and 2048 frames, when more than 4 per SM of them are in the
    call; route="window" raises the frame limit to 8192."""
    row = wl.vocab <= 64 and (wl.vocab * 4) % 16 == 0
    limit = 8192 if route == "window" else 2048
    ok = (wl.lengths <= limit) & (2 * wl.target_lengths + 1 <= 4096) & row
    if route == "auto" and ok.sum() <= 4 * sms:
        ok[:] = False
    return ok


def strong_cfg4_lane(ffa, lib, rank, world, device, steps, warmup, flush, max_over_ranks, barrier, peak):
    """Strong scaling on the multi-GPU configuration (cfg4): every rank draws
    the same 8,256-record batch and aligns its LPT share (shard_of_rank),
    device-resident, timed as `value`; the whole box's frames/s over the
    slowest rank's time."""
    import torch
    from fast_forced_aligner_b200 import workloads
    from fast_forced_aligner_b200.sharding import shard_of_rank
    pool = workloads.config(4)
    shard = pool.subset(shard_of_rank(pool.lengths, pool.target_lengths, rank, world))
    e = torch.from_numpy(shard.emissions).to(device)
    t = torch.from_numpy(shard.targets).to(device)

    def call():
        return ffa.align_packed(e, shard.lengths, t, shard.target_lengths, blank_id=0, mode="optimized")
    barrier()
    ms = queued_device_ms(call, steps, warmup, flush)
    total = max_over_ranks(sum(ms))
    barrier()
    # The greedy pass of the window route (the launch that streams every row
    # of the window records once): its device time from the forward
    # profiling events, against the rows it reads and the bounds it writes.
    import ctypes
    greedy = None
    window = window_records(shard, torch.cuda.get_device_properties(device).multi_processor_count)
    if window.any():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for x in ev:
            x.record()
        times = []
        for _ in range(5):
            flush.zero_()
            lib.ffa_profile_forward_events(ctypes.c_void_p(ev[0].cuda_event), ctypes.c_void_p(ev[1].cuda_event))
            call()
            lib.ffa_profile_forward_events(None, None)
            torch.cuda.synchronize()
            times.append(ev[0].elapsed_time(ev[1]))
        g_ms = statistics.median(times)
        wf = int(shard.lengths[window].sum())
        nbytes = wf * shard.vocab * 4 + wf * 4  # every row of a window record (its alphabet fills V = 32), and m[t]
        greedy = {"kernel": "ffa_greedy_pass (window route: each frame's bound over the alphabet and the "
                            "reference's greedy chunk verdicts)", "bound": "hbm", "bytes": nbytes, "ms": g_ms,
                  "achieved": nbytes / (g_ms / 1e3) / 1e9, "unit": "GB/s", "peak": peak,
                  "frac": nbytes / (g_ms / 1e3) / 1e9 / peak, "frames": wf}
    frames = int(pool.lengths.sum())
    out = {"value": frames * steps / (total / 1e3), "unit": "frames/s", "ms_per_step": total / steps,
            "n_gpus": world, "scaling": "strong", "records_total": pool.batch, "frames_total": frames,
            "records_this_rank": shard.batch,
            "how": "cfg4 (8,256 records) LPT-partitioned over the ranks by record cost (shard_of_rank), "
                   "optimized mode, device-resident, L2 flushed before every step; max over ranks"}
    if greedy is not None:
        out["greedy_pass_rank0" if world > 1 else "greedy_pass"] = greedy
    return out


def cpu_reference_runner(wl):
    """The reference's corrected C++ comparator (oracle/_ref) over all host
    threads, one record per task with the GIL released, as in its benchmark
    adapter; falls back to our C oracle ("port") if the build is absent."""
    from oracle import oracle
    threads = oracle.default_threads()
    module = oracle.corrected_module()
    es, ts = wl.records()
    if module is not None:
        pool = ThreadPoolExecutor(max_workers=threads)
        inputs = [(e[None], t[None]) for e, t in zip(es, ts)]

        def run():
            return list(pool.map(lambda a: module.forced_align(a[0], a[1], wl.blank), inputs))
        return run, "reference", threads, pool

    def run_port():
        return oracle.align(es, ts, wl.blank, threads=threads)
    return run_port, "port", threads, None


def time_cpu(run, frames, seconds):
    run()  # warm the pool / caches
    done, start = 0, time.perf_counter()
    while True:
        run()
        done += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            return frames * done / elapsed, done, elapsed


# ------------------------------------------------------------------ our arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    import fast_forced_aligner_b200 as ffa
    from fast_forced_aligner_b200 import workloads
    from fast_forced_aligner_b200.build import LIB
    from fast_forced_aligner_b200.pipeline import AlignStream
    from fast_forced_aligner_b200.sharding import reduce_over_ranks, shard_of_rank

    rank, world, local = rank_info()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    # One process per GPU: its host batches and submitting thread on the
    # GPU's NUMA node (before any pinned buffer is touched).
    from fast_forced_aligner_b200.pipeline import bind_host_to_device
    host_cpus = bind_host_to_device(device) if world > 1 else None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        return reduce_over_ranks(x, "max", device)

    def sum_over_ranks(x):
        return reduce_over_ranks(x, "sum", device)

    ffa.load_extension()
    if args.split:
        pool = workloads.config(args.config, scale=args.scale)
        wl = pool.subset(shard_of_rank(pool.lengths, pool.target_lengths, rank, world))
        parallelism = f"one batch LPT-partitioned over {world} GPU(s) by record cost, no collective"
    else:
        wl = workloads.config(args.config, scale=args.scale, shard=rank)
        parallelism = f"records sharded, {world} independent GPU(s), no collective"
    records_total = int(sum_over_ranks(wl.batch))
    frames = int(wl.lengths.sum())
    frame_list, token_list = wl.lengths.tolist(), wl.target_lengths.tolist()
    from_logits = args.input != "log-probs"
    if from_logits:
        # Logits whose log_softmax is the workload's log-probabilities up to
        # rounding: each row shifted by a seeded offset, as a model's rows are.
        offsets = np.random.default_rng(1234).uniform(-8.0, 8.0, (wl.emissions.shape[0], 1)).astype(np.float32)
        e_host = torch.from_numpy(wl.emissions + offsets)
        if args.input == "logits-bf16":
            e_host = e_host.to(torch.bfloat16)
        e_host = e_host.pin_memory()
    else:
        e_host = torch.from_numpy(wl.emissions).pin_memory()
    t_host = torch.from_numpy(wl.targets).pin_memory()
    e_dev = e_host.to(device)
    t_dev = t_host.to(device)
    ffa.validate_inputs(list(e_dev.split(frame_list)), list(t_dev.split(token_list)), blank_id=wl.blank)

    def step(e, t):
        return ffa.align_packed(e, wl.lengths, t, wl.target_lengths, blank_id=wl.blank, mode=args.mode,
                                from_logits=from_logits, route=args.route)

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    import ctypes
    lib = ctypes.CDLL(str(LIB))
    lib.ffa_launch_count.restype = ctypes.c_int64
    torch.cuda.synchronize()

    # Warm-up as the timed loop runs: each step's result is still held while
    # the next step allocates its outputs, so the allocator's blocks for both
    # exist before timing starts.
    result = None
    for _ in range(args.warmup):
        flush.zero_()
        result = step(e_dev, t_dev)
    torch.cuda.synchronize()

    def events(n):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for ev in evs:
            ev.record()  # creates the CUDA event (torch creates it lazily)
        return evs

    # ---- device-resident timing: inputs in HBM.  Steps are queued back to
    # back with no host synchronisation between them, as batches stream in
    # production, so a call's host work overlaps the device work of the call
    # before it; the 256 MiB L2 flush runs on the device between consecutive
    # steps, and each step's events bracket that align call's device work.
    ev0, ev1 = events(args.steps), events(args.steps)
    f0, f1 = events(args.steps), events(args.steps)
    torch.cuda.synchronize()
    barrier()
    with ClockSampler(local) as clocks:
        # The device starts the timed loop busy (~10 ms of sleep, outside
        # every step's events), so the first step's host work is hidden as
        # every later step's is.
        torch.cuda._sleep(20_000_000)
        for k in range(args.steps):
            flush.zero_()
            lib.ffa_profile_forward_events(ctypes.c_void_p(f0[k].cuda_event), ctypes.c_void_p(f1[k].cuda_event))
            ev0[k].record()
            result = step(e_dev, t_dev)
            ev1[k].record()
            lib.ffa_profile_forward_events(None, None)
        torch.cuda.synchronize()
        barrier()
        step_ms = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]
        fwd_ms = [a.elapsed_time(b) for a, b in zip(f0, f1)]
        total_ms = max_over_ranks(sum(step_ms))

        # ---- one call at a time: its host and device latency together.
        lat0, lat1 = events(1)[0], events(1)[0]
        lat = []
        for _ in range(min(args.steps, 10)):
            flush.zero_()
            torch.cuda.synchronize()
            lat0.record()
            step(e_dev, t_dev)
            lat1.record()
            torch.cuda.synchronize()
            lat.append(lat0.elapsed_time(lat1))
        latency_ms = max_over_ranks(statistics.median(lat))

        # ---- end to end: pinned host inputs -> device -> align -> pinned host
        # results, every step, through AlignStream (each step's copies overlap
        # its neighbours' alignment).  The loop runs at least E2E_MIN_SECONDS
        # (as many batches as the device-timed step suggests, the same count
        # on every rank), so that one stall of the host or of the clock
        # sampler's queries does not decide the rate.
        astream = AlignStream(device)
        e2e_steps = max(args.steps, min(E2E_MAX_STEPS, int(math.ceil(
            E2E_MIN_SECONDS * 1e3 / max_over_ranks(statistics.median(step_ms))))))

        def e2e_step():
            return astream.submit(e_host, wl.lengths, t_host, wl.target_lengths, blank_id=wl.blank,
                                  mode=args.mode, from_logits=from_logits)
        # Warm-up with as many batches in flight as the timed loop has, so
        # that the pinned result blocks the timed loop cycles through are
        # allocated (page-locked) before it starts.
        for _ in range(max(args.warmup, args.steps)):
            pending = e2e_step()
        pending.result()
        torch.cuda.synchronize()
        barrier()
        e2e0, e2e1 = events(1)[0], events(1)[0]
        e2e0.record(astream.copy_in)
        for _ in range(e2e_steps):
            pending = e2e_step()
        e2e1.record(astream.copy_out)
        host_result = pending.result()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e2e0.elapsed_time(e2e1))
        barrier()

    # ---- per-phase device time of one call (outside the timed loops): events
    # at every phase boundary of ffa_align, L2 flushed first as above.
    n_points = len(PHASES) + 1
    points = [torch.cuda.Event(enable_timing=True) for _ in range(n_points)]
    for ev in points:
        ev.record()  # creates the CUDA event (torch creates it lazily)
    torch.cuda.synchronize()
    handles = (ctypes.c_void_p * n_points)(*[ctypes.c_void_p(ev.cuda_event) for ev in points])
    phase_us = {name: [] for name in PHASES}
    per_call = []
    for _ in range(max(3, args.warmup)):
        torch.cuda.synchronize()
        # Two flush passes queued ahead (no sync): the host submits the whole
        # call while they run, so each phase is timed on the device alone.
        flush.zero_(); flush.zero_()
        before = lib.ffa_launch_count()
        lib.ffa_profile_phase_events(handles, n_points)
        step(e_dev, t_dev)
        lib.ffa_profile_phase_events(None, 0)
        per_call.append(lib.ffa_launch_count() - before)
        torch.cuda.synchronize()
        for k, name in enumerate(PHASES):
            phase_us[name].append(1e3 * points[k].elapsed_time(points[k + 1]))
    phases = {name: round(statistics.median(v), 2) for name, v in phase_us.items()}
    launches = per_call[-1] * 2 * args.steps  # device-resident + end-to-end timed loops
    status_ok = bool((result.status == 0).all().item()) and bool((host_result.status == 0).all().item())
    # The validity scan reads fp32 records.
    scan = validity_scan_roofline(ffa, e_dev, frame_list, wl.vocab, args.warmup) \
        if e_dev.dtype == torch.float32 else None
    unfused = unfused_logits_ms(ffa, e_dev, t_dev, wl, args, flush) if from_logits else None

    ref_cuda = reference_cuda_lane(wl, e_dev, t_dev, args.steps, args.warmup, flush) \
        if world == 1 and not from_logits and args.scale == 1.0 else None
    strong = strong_cfg4_lane(ffa, lib, rank, world, device, args.steps, args.warmup, flush, max_over_ranks, barrier,
                              peaks()[0]) \
        if args.config == 1 and not args.split and not from_logits and args.scale == 1.0 else None

    all_frames = sum_over_ranks(frames)
    value = all_frames * args.steps / (total_ms / 1e3)
    e2e_value = all_frames * e2e_steps / (e2e_ms / 1e3)
    fwd_avg_ms = max_over_ranks(statistics.fmean(fwd_ms))
    read_bytes, alg_bytes = algorithmic_bytes(wl, e_dev.element_size())
    peak, peak_kind = peaks()
    # With records on the window route, the profiled launch is the greedy pass
    # (every row of those records once, and each frame's bound written).
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    win = window_records(wl, sms, args.route) if args.mode == "optimized" and args.route != "pieces" else None
    if win is not None and win.any():
        wf = int(wl.lengths[win].sum())
        read_bytes = wf * wl.vocab * e_dev.element_size() + wf * 4
        roofline_kernel = ("ffa_greedy_pass (window route: each frame's bound over the alphabet and the "
                           "reference's greedy chunk verdicts; its span overlaps the chunked route's kernels)")
    else:
        roofline_kernel = "ffa_viterbi_forward (first pass: streams every emission row)"
    achieved = read_bytes / (fwd_avg_ms / 1e3) / 1e9
    traffic = from_profile(wl.name, "traffic_bytes_per_launch")
    instructions = from_profile(wl.name, "warp_instructions_per_launch")
    cells = wl.cells()
    line = {
        "metric": "aligned frames/sec", "value": value, "unit": "frames/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "latency_ms_per_call": latency_ms,
        "step_ms": {"min": min(step_ms), "median": statistics.median(step_ms), "max": max(step_ms),
                    "slowest": int(np.argmax(step_ms))},
        "higher_is_better": True,
        "scaling": "strong" if args.split else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name if args.scale == 1.0 else f"{wl.name} at scale {args.scale}",
                   "records_per_gpu": wl.batch, "frames_per_gpu": frames,
                   "records_total": records_total, "frames_total": int(all_frames),
                   "vocab": wl.vocab, "mode": args.mode, "route": args.route, "check_inputs": True,
                   "inputs": ("packed device-resident fp32 [sum T, V] log-probabilities" if not from_logits
                              else f"packed device-resident {args.input[7:]} [sum T, V] logits, aligned as their "
                                   "log_softmax inside the kernels (from_logits)") + " + int64 targets",
                   "l2": "flushed (256 MiB write) before every timed step",
                   "timing": "steps queued back to back (no host sync between them); per-step device time "
                             "from events around each align call; latency_ms_per_call = one synced call, "
                             "host and device",
                   "parallelism": parallelism},
        "e2e": {"value": e2e_value, "unit": "frames/s", "steps": e2e_steps, "ms_per_step": e2e_ms / e2e_steps,
                "h2d_bytes_per_step": int(e_host.numel() * e_host.element_size() + t_host.numel() * 8),
                "d2h_bytes_per_step": int(frames * 12 + wl.batch * 8),
                "api": "fast_forced_aligner_b200.AlignStream.submit (align_packed, the torch op over the "
                       "C ABI, with host copies overlapped on separate streams)",
                "host_cpus": len(host_cpus) if host_cpus else None},
        "roofline": {"kernel": roofline_kernel,
                     "bound": "hbm", "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": traffic,
                     "algorithmic_bytes_per_launch": read_bytes,
                     "kernel_ms": fwd_avg_ms,
                     "note": "max-plus DP: bound by the per-frame dependency chain of each piece "
                             "or record and by instruction issue, not by HBM; see dp and phases_us"},
        "dp": {"longest_record_frames": int(wl.lengths.max()),
               "first_pass_cells_per_s": cells / (fwd_avg_ms / 1e3), "cells": cells},
        "phases_us": phases,
        "validity_scan": dict(scan, peak=peak, frac=scan["achieved"] / peak,
                              peak_source=f"{peak_kind} hbm_gbs") if scan else None,
        "b_alg_bytes": alg_bytes,
        "gpu_launches": launches,
        "gpu_launches_note": f"{per_call[-1]} kernels of libffa_b200 per align call (counted by "
                             "ffa_launch_count), in the device-resident and the end-to-end timed loops",
        "status_ok": status_ok,
    }
    if ref_cuda is not None and "unavailable" in ref_cuda:
        line["reference_cuda"] = ref_cuda
    elif ref_cuda is not None:
        line["reference_cuda"] = dict(
            ref_cuda, ratio_value=value / ref_cuda[args.mode]["value"],
            ratio_value_vs_optimized=value / ref_cuda["optimized"]["value"],
            how="the reference's CUDA extension (its alignment.cu compiled in place for sm_100a with the flags "
                "its loader passes) on the same device-resident batch, called with its public-API arguments "
                "(alignment.py:496-501), timed exactly as value")
    if strong is not None:
        line["strong_cfg4"] = strong
    if unfused is not None:
        line["unfused"] = {"ms_per_step": unfused, "value": frames * world / (unfused / 1e3),
                           "pipeline": "torch.log_softmax(logits.float(), -1) then align_packed on the "
                                       "fp32 log-probabilities (the reference's example pipeline), device-"
                                       "resident, timed as value"}
    clock = clocks.summary()
    line["clocks"] = clock
    if instructions is not None and args.route == "auto" and not (win is not None and win.any()):
        # The first pass's issue roofline: its warp instructions per launch (the
        # committed ncu summary) over its live duration, against every SMSP
        # issuing one warp instruction per cycle at the sampled clock.
        issue_peak = sms * 4 * clock["sm_mhz"] * 1e6 / 1e9 if clock.get("sm_mhz") else None
        issue = instructions / (fwd_avg_ms / 1e3) / 1e9
        line["roofline"]["issue"] = {
            "bound": "issue", "achieved": issue, "peak": issue_peak, "unit": "G warp-instructions/s",
            "frac": issue / issue_peak if issue_peak else None, "instructions_per_launch": instructions,
            "peak_source": f"{sms} SMs x 4 SMSPs x 1 warp-instruction per cycle at the sampled SM clock",
            "source": f"profiles/ffa_viterbi_forward_{wl.name}.md"}
    if rank == 0 and world == 1:
        run, kind, threads, pool = cpu_reference_runner(wl)
        cpu_value, passes, seconds = time_cpu(run, frames, args.cpu_seconds)
        if pool is not None:
            pool.shutdown()
        line["cpu_baseline"] = {"value": cpu_value, "unit": "frames/s", "cores": threads, "kind": kind,
                                "sample": f"{passes} passes over the {wl.name} batch "
                                          f"({wl.batch} records, {frames} frames) in {seconds:.1f} s"
                                          + (" (as fp32 log-probabilities: the reference takes no logits)"
                                             if from_logits else "")}
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------ reference arms

def run_reference_cpu(args):
    rank, world, _ = rank_info()
    if rank != 0:
        return
    from fast_forced_aligner_b200 import workloads
    wl = workloads.config(args.config)
    frames = int(wl.lengths.sum())
    run, kind, threads, pool = cpu_reference_runner(wl)
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    if pool is not None:
        pool.shutdown()
    value = frames * args.steps / sum(times)
    line = {
        "impl": "reference", "metric": "aligned frames/sec", "value": value, "unit": "frames/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name, "records_per_gpu": wl.batch, "frames_per_gpu": frames,
                   "vocab": wl.vocab, "mode": "conventional (CPU)"},
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": threads, "kind": kind,
                         "sample": f"{args.steps} timed passes over the {wl.name} batch "
                                   f"({wl.batch} records, {frames} frames)"},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_cuda(args):
    rank, world, local = rank_info()
    if rank != 0:
        return
    import torch
    from fast_forced_aligner_b200 import workloads
    from oracle import oracle
    if not oracle.load_reference_cuda():
        print(json.dumps({"impl": "reference-cuda", "unavailable": "oracle/_ref/fast_forced_aligner_cuda.so not built"}))
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = workloads.config(args.config)
    frames = int(wl.lengths.sum())
    e_dev = torch.from_numpy(wl.emissions).to(device)
    t_dev = torch.from_numpy(wl.targets).to(device)
    es = list(e_dev.split(wl.lengths.tolist()))
    ts = list(t_dev.split(wl.target_lengths.tolist()))
    blanks = [wl.blank] * wl.batch
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    results = {}
    for mode in ("optimized", "conventional"):
        for _ in range(args.warmup):
            oracle.reference_cuda_align(es, ts, blanks, mode=mode, check_inputs=True)
        torch.cuda.synchronize()
        # Timed as our arm: steps queued back to back, the L2 flush between
        # them, events around each call; then one synced call at a time.
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for k in range(args.steps):
            flush.zero_()
            ev[k][0].record()
            oracle.reference_cuda_align(es, ts, blanks, mode=mode, check_inputs=True)
            ev[k][1].record()
        torch.cuda.synchronize()
        total = sum(a.elapsed_time(b) for a, b in ev)
        lat = []
        for a, b in ev[:10]:
            flush.zero_()
            torch.cuda.synchronize()
            a.record()
            oracle.reference_cuda_align(es, ts, blanks, mode=mode, check_inputs=True)
            b.record()
            torch.cuda.synchronize()
            lat.append(a.elapsed_time(b))
        results[mode] = {"value": frames * args.steps / (total / 1e3), "ms_per_step": total / args.steps,
                         "latency_ms_per_call": statistics.median(lat)}
    line = {"impl": "reference-cuda", "metric": "aligned frames/sec",
            "value": results[args.mode]["value"], "unit": "frames/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": results[args.mode]["ms_per_step"],
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl.name, "records": wl.batch, "frames": frames, "mode": args.mode,
                       "l2": "flushed before every timed step",
                       "api": "reference align op with its public-API arguments (alignment.py:496-501)"},
            "modes": results}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference_cpu(args)
    elif args.impl == "reference-cuda":
        run_reference_cuda(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
