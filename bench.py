#!/usr/bin/env python
"""Throughput of the RF-DETR matcher step (fused cost kernel + exact batched LSAP) on B200.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rfm|reference]``

A step is one full ``HungarianMatcher`` pass (cost matrix + every assignment
problem + device unpack) over one batch of the ``sweep`` workload: 1024 images x
13 query groups x 300 queries, 2 classes, T ~ Poisson(8) clipped to [1, 60]
targets per image -> 13,312 [300 x T] problems per GPU.  Under torchrun each rank
matches its own 1024-image shard (weak scaling, no collective on the data path)
and ``value`` is all ranks' problems divided by the slowest rank's device time.

Keys beyond the base contract:
  e2e           the same metric through ``match_packed`` with pinned HOST inputs:
                the step's input copies and the D2H of its packed index pairs are
                inside the timed region;
  roofline      the cost kernel, HBM-bound: algorithmic bytes per launch over its
                CUDA-event duration, against the measured copy bandwidth;
  lsap          the solver kernel's device time and problems/s;
  cpu_baseline  the reference's CPU path (torch CPU op chain + SciPy on a thread
                pool of every host thread this process may use) on a bounded
                sample of the same workload, rank 0, N = 1;
  configs       (N = 1) every benchmark configuration -- step, crowd, ties and
                sweep -- with its device time through ``match_packed`` and the
                reference CPU path on the same inputs, serial (one thread, as the
                unpatched matcher solves) and on the reference's 8-thread pool;
  per_rank_step_ms  min / median / max / mean device ms of the timed steps on
                every rank.

Timed regions start behind about a millisecond of device-side work outside the
events (writes of the L2-flush buffer, which keep the GPU busy rather than idle),
so the host has enqueued the first steps before the GPU reaches them and a late
host launch cannot leave the GPU idle inside a step.

``--impl reference`` times that CPU path alone, with the same thread setting as
``cpu_baseline``.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "matched problems/s (cost+LSAP) at 1/2/4/8 B200; cost-kernel HBM GB/s vs peak"
UNIT = "problems/s"
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20
PEER_COPY_GBS = 770.0  # measured peer copy over NVLink on these B200s, per direction per GPU
LEAD_FILLS = 25  # writes of a 256 MiB buffer (~1 ms of device-side work) before each timed region
_LEAD_BUF: dict = {}


def device_lead(device) -> None:
    """About a millisecond of memory-bound device work, enqueued before a timed region: the host gets
    ahead of the GPU, and the GPU stays busy (an idle spin before the region left its next step slow)."""
    key = str(device)
    if key not in _LEAD_BUF:
        _LEAD_BUF[key] = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)
    for _ in range(LEAD_FILLS):
        _LEAD_BUF[key].zero_()
CONFIG_NAMES = ("step", "crowd", "ties", "sweep")
REFERENCE_POOL_THREADS = 8  # LAP_THREADS default of the parallel_lap patch (patches.py:210)


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["rfm", "reference"], default="rfm")
    ap.add_argument("--workload", default="sweep")
    ap.add_argument("--images", type=int, default=None, help="images per rank (default: the workload's)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample budget")
    ap.add_argument("--cpu-images", type=int, default=64, help="images in one CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-production-step", action="store_true",
                    help="skip the 5-layer x 8-image production-step timing (eager vs CUDA graph)")
    ap.add_argument("--sharded", action="store_true",
                    help="also time the strong-scaled sharded sweep (runs by default when N > 1)")
    ap.add_argument("--sharded-images", type=int, nargs="*", default=[1024, 8192],
                    help="batch sizes (images) of the strong-scaled sharded sweep")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-configuration table (N = 1)")
    ap.add_argument("--config-cpu-seconds", type=float, default=2.0,
                    help="CPU time budget of each CPU leg of the per-configuration table")
    ap.add_argument("--kernel", choices=["cost", "cost_qm", "lsap", "lsap_push", "label", "box", "msda"],
                    default=None,
                    help="profiling mode: run only this kernel's workload a few times (for an ncu capture) and exit")
    return ap.parse_args()


def workload_config(wl) -> dict:
    return {
        "workload": (f"{wl.name}: {wl.images} images x {wl.group_detr} groups x {wl.queries // wl.group_detr} "
                     f"queries x {wl.layers} layer(s), {wl.classes} classes, per-image T as documented "
                     f"in workloads.py; {wl.num_problems} [300 x T] problems per GPU per step"),
        "images_per_gpu": wl.images,
        "group_detr": wl.group_detr,
        "queries": wl.queries,
        "layers": wl.layers,
        "classes": wl.classes,
        "targets_per_gpu": int(sum(wl.sizes)),
        "problems_per_gpu_step": wl.num_problems,
        "l2": "flushed between timed steps (256 MiB write outside the events)",
    }


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.path = os.path.join("/tmp", f"rfm_clocks_{os.getpid()}.csv")
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        gpu_id = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        self.cmd = [exe, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50", "-i", gpu_id]

    def start(self) -> None:
        if not hasattr(self, "cmd"):
            return
        self.fh = open(self.path, "w")
        self.proc = subprocess.Popen(self.cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        time.sleep(0.3)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        max_mhz = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": len(rows)}


# --------------------------------------------------------------------------- helpers


def peak_hbm() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def cost_bytes(wl) -> int:
    """Algorithmic bytes of one rfm_cost launch: every cost element written once (L x Q x sum T
    float32), each prediction (box + logits row) and each target (box + int64 label) read once."""
    L, B, Q, C = wl.layers, wl.images, wl.queries, wl.classes
    return 4 * L * Q * sum(wl.sizes) + 16 * L * B * Q + 4 * L * B * Q * C + 24 * sum(wl.sizes) + 4 * (B + 1)


def lsap_bytes(plan) -> int:
    """Algorithmic bytes of one rfm_lsap launch: every problem's cost block read once, its
    descriptor read, its int64 (query, target) pairs written."""
    pr = plan.problems
    return int((4 * pr["num_queries"].astype(np.int64) * pr["num_targets"]).sum()) + 40 * pr.shape[0] \
        + 16 * plan.total_pairs


def dist_init(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def traffic_per_launch() -> float | None:
    """DRAM bytes of one cost-kernel launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "cost_kernel_sweep_traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


# --------------------------------------------------------------------------- CPU path


def gpu_local_cpus(device: torch.device) -> set[int] | None:
    """The host CPUs NVML names as nearest the GPU (its NUMA node), within this process's
    allowed set, or None when NVML cannot tell.  Only read: nothing about the GPU is changed."""
    try:
        import pynvml

        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 1) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:  # no NVML, no such call, or a foreign bus id format: leave the process as it is
        return None


def host_threads() -> int:
    """Host CPUs this process may run on (its affinity set)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_path_rate(wl, images: int, budget_s: float, lap_threads: int, torch_threads: int,
                  min_reps: int = 1) -> dict:
    """problems/s of the reference CPU path on the first ``images`` images, repeated for ~budget_s:
    the torch CPU op chain on ``torch_threads`` intra-op threads, then SciPy per block, serially when
    ``lap_threads`` is 1, else on a pool of that many threads."""
    from oracle.cpu_path import CpuMatcher

    images = min(images, wl.images)
    logits = wl.pred_logits[:, :images].contiguous()
    boxes = wl.pred_boxes[:, :images].contiguous()
    targets = wl.targets[:images]
    problems = wl.layers * wl.group_detr * sum(1 for t in targets if t["labels"].shape[0])
    saved = torch.get_num_threads()
    torch.set_num_threads(torch_threads)
    m = CpuMatcher(threads=lap_threads)
    try:
        m.match(logits, boxes, targets, wl.group_detr, wl.weights)  # warm
        reps, t0 = 0, time.perf_counter()
        while reps < min_reps or time.perf_counter() - t0 < budget_s:
            m.match(logits, boxes, targets, wl.group_detr, wl.weights)
            reps += 1
        elapsed = time.perf_counter() - t0
    finally:
        m.close()
        torch.set_num_threads(saved)
    return {"value": problems * reps / elapsed, "unit": UNIT, "seconds": elapsed, "reps": reps,
            "problems_per_rep": problems, "images": images, "scipy_threads": lap_threads,
            "torch_threads": torch_threads}


def cpu_baseline_setting() -> tuple[int, int]:
    """(SciPy pool threads, torch threads) of the headline CPU baseline and of ``--impl reference``:
    every host thread this process may use, for both."""
    n = host_threads()
    return n, n


def run_reference(args) -> None:
    world, rank, _ = dist_init(args)
    if rank != 0:
        return
    from rfdetr_training_throughput_b200 import workloads

    lap_threads, torch_threads = cpu_baseline_setting()
    wl = workloads.make(args.workload, images=args.images)
    images = min(args.cpu_images, wl.images)
    from oracle.cpu_path import CpuMatcher

    logits = wl.pred_logits[:, :images].contiguous()
    boxes = wl.pred_boxes[:, :images].contiguous()
    targets = wl.targets[:images]
    problems = wl.layers * wl.group_detr * sum(1 for t in targets if t["labels"].shape[0])
    torch.set_num_threads(torch_threads)
    m = CpuMatcher(threads=lap_threads)
    try:
        for _ in range(args.warmup):
            m.match(logits, boxes, targets, wl.group_detr, wl.weights)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            m.match(logits, boxes, targets, wl.group_detr, wl.weights)
        elapsed = time.perf_counter() - t0
    finally:
        m.close()
    value = problems * args.steps / elapsed
    sample_desc = (f"first {images} images of the {wl.name} workload per step ({problems} problems): torch CPU "
                   f"op chain ({torch_threads} threads) + scipy.optimize.linear_sum_assignment on a "
                   f"{lap_threads}-thread pool; host has {os.cpu_count()} CPUs, {host_threads()} usable")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 cost, fp64 LSAP",
        "data": "synthetic", "config": workload_config(wl),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": lap_threads, "kind": "port", "sample": sample_desc,
                         "host_cpu_count": os.cpu_count(), "torch_threads": torch_threads},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    line["config"]["cpu_sample"] = {"images": images}
    line["reference_gpu_lsap"] = reference_gpu_lsap()
    line["reference_gpu_cost"] = {"unavailable": (
        "the reference's cost kernel is Triton source JIT-compiled from the reference tree at run time "
        "(kernels_matcher.py:179-234); that tree is not on the GPU box and its sources are not copied here")}
    emit(line)


def reference_gpu_lsap() -> dict:
    """The reference's own GPU solver (lsap_kernel / batch_lap_cuda, kernels_lap.py:69-305, built from
    its source by oracle/build_ref.py) on the batches ``lsap_batches_rfm`` gives the repository's
    solver: the same B200, the same inputs."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    from oracle import build_ref

    mod = build_ref.load()
    if mod is None:
        return {"unavailable": "oracle/_ref holds no build of the reference solver (python -m oracle.build_ref)"}
    device = torch.device("cuda", 0)
    return {f"T{t}": time_solver(mod.batch_lap_cuda, lsap_batch(t, device), device) for t in LSAP_BATCH_TASKS} | {
        "unit": "ms per 520-problem batch", "batches": "520 x [300 x T] uniform costs, seed 5000 + T",
        "solver": "reference lsap_kernel (fp32 --use_fast_math, one 256-thread block per problem)"}


# --------------------------------------------------------------------------- GPU path


def time_device_steps(fn, steps: int, warmup: int, flush: torch.Tensor, device, barrier=None) -> list[float]:
    """Device ms of each of ``steps`` calls of ``fn`` (CUDA events on the launching stream), the L2
    flushed between calls outside the events.  The region starts behind a device-side delay so the
    host is ahead of the GPU from the first step on."""
    for _ in range(max(warmup, 1)):
        fn()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if barrier is not None:
        barrier()
    torch.cuda.synchronize(device)
    device_lead(device)
    for k in range(steps):
        starts[k].record()
        fn()
        ends[k].record()
        flush.zero_()
    torch.cuda.synchronize(device)
    if barrier is not None:
        barrier()
    return [a.elapsed_time(b) for a, b in zip(starts, ends)]


def step_stats(ms: list[float]) -> dict:
    return {"min": min(ms), "median": statistics.median(ms), "max": max(ms), "mean": statistics.mean(ms)}


def config_table(device, args, flush, sweep_wl) -> dict:
    """Every benchmark configuration on this GPU through ``match_packed`` (device time per step, L2
    flushed between steps) with the reference CPU path on the same inputs beside it: serial (one
    thread for the op chain and the solves) and on the reference's pool (8 SciPy threads, every host
    thread for the op chain).  The sweep's CPU legs run on its first ``--cpu-images`` images."""
    from rfdetr_training_throughput_b200 import matcher, workloads

    out = {"host_cpu_count": os.cpu_count(), "host_threads_usable": host_threads()}
    for name in CONFIG_NAMES:
        wl = sweep_wl if name == "sweep" else workloads.make(name)
        logits, boxes = wl.pred_logits.to(device), wl.pred_boxes.to(device)
        packed = matcher.PackedTargets.from_list(wl.targets_on(device), device)

        def fn():
            matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights)

        steps = max(3, min(args.steps, 50))
        ms = time_device_steps(fn, steps, max(args.warmup, 3), flush, device)
        mean = statistics.mean(ms)
        entry = {"problems": wl.num_problems, "images": wl.images, "layers": wl.layers, "classes": wl.classes,
                 "targets": int(sum(wl.sizes)), "max_targets": max(wl.sizes), "gpu_steps": steps,
                 "gpu_ms_per_step": step_stats(ms), "gpu_problems_per_s": wl.num_problems / (mean / 1e3)}
        if not args.no_cpu_baseline:
            images = args.cpu_images if name == "sweep" else wl.images
            serial = cpu_path_rate(wl, images, args.config_cpu_seconds, 1, 1)
            pool = cpu_path_rate(wl, images, args.config_cpu_seconds, REFERENCE_POOL_THREADS, host_threads())
            entry["cpu_serial"] = serial
            entry["cpu_pool"] = pool
            entry["gpu_over_cpu_pool"] = entry["gpu_problems_per_s"] / pool["value"]
        out[name] = entry
        del logits, boxes, packed
    return out


def run_rfm(args) -> None:
    world, rank, local = dist_init(args)
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)

    from rfdetr_training_throughput_b200 import MatchGraph, _lib, matcher, workloads

    wl = workloads.make(args.workload, shard=rank, images=args.images)
    logits = wl.pred_logits.to(device)
    boxes = wl.pred_boxes.to(device)
    packed = matcher.PackedTargets.from_list(wl.targets_on(device), device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def step(events=None, extras=None):
        return matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights, events=events,
                                    extras=extras)

    sampler = ClockSampler(device)
    sampler.start()
    extras: dict = {}
    step(extras=extras)
    plan = extras["plan"]
    # the production call: rfm_match, cost kernel and solver overlapped at their boundary
    step_ms = time_device_steps(step, args.steps, args.warmup, flush, device, barrier)
    clocks = sampler.stop()
    total_ms = float(sum(step_ms))

    # per-kernel durations (the roofline figures): the same steps issued as two calls with events
    # recorded around each kernel, outside the timed loop above
    kernel_events: dict = {}
    for k in range(args.steps):
        step(events=kernel_events)
        flush.zero_()
    torch.cuda.synchronize(device)

    def kernel_ms(name):
        ev = kernel_events.get(name, [])
        return [ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev), 2)]

    cost_ms = kernel_ms("cost")
    lsap_ms = kernel_ms("lsap")
    launches = len(cost_ms) + len(lsap_ms)

    # the same step replayed as a captured CUDA graph (one host call per step)
    graph = MatchGraph(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights, device=device)
    graph.logits.copy_(logits)
    graph.boxes.copy_(boxes)
    graph.labels.copy_(packed.labels)
    graph.tgt_boxes.copy_(packed.boxes)
    graph_ms = time_device_steps(graph.replay, args.steps, args.warmup, flush, device, barrier)
    del graph

    mine = torch.tensor([*step_stats(step_ms).values(), total_ms, float(sum(graph_ms))], dtype=torch.float64,
                        device=device)
    if world > 1:
        gathered = [torch.zeros_like(mine) for _ in range(world)]
        torch.distributed.all_gather(gathered, mine)
    else:
        gathered = [mine]
    per_rank = [dict(zip(("min", "median", "max", "mean", "total", "graph_total"), g.tolist())) for g in gathered]
    max_ms = max(r["total"] for r in per_rank)
    graph_max_ms = max(r["graph_total"] for r in per_rank)
    problems = wl.num_problems
    value = world * problems * args.steps / (max_ms / 1e3)

    # ---- end to end: pinned host inputs -> device -> match -> packed pairs back to host
    e2e = None
    if not args.no_e2e:
        e2e = e2e_timing(args, wl, plan, device, barrier, world, problems)

    # ---- production step (5 layers x 8 images x 13 groups, 520 problems): eager calls vs the CUDA graph
    production = None
    box_loss = None
    configs = None
    label_loss = None
    msda = None
    if world == 1 and not args.no_production_step:
        production = production_step_timing(device, max(args.warmup, 3))
        box_loss = box_loss_timing(device, max(args.warmup, 3))
        label_loss = label_loss_timing(device, max(args.warmup, 3), wl, logits, boxes, packed)
        msda = msda_timing(device, max(args.warmup, 3))
    cost_qmajor = None
    if world == 1:
        cost_qmajor = cost_query_major_timing(device, wl, logits, boxes, packed)
    lsap_batches = None
    if world == 1 and not args.no_configs:
        configs = config_table(device, args, flush, wl)
        lsap_batches = lsap_batches_rfm(device)

    # ---- sharded sweep: ONE batch split across the ranks + NCCL all-gather of the pairs
    sharded_info = None
    if world > 1 or args.sharded:
        # one process: a one-rank group of its own, so the same code path runs
        own_group = world == 1 and not torch.distributed.is_initialized()
        if own_group:
            import socket

            with socket.socket() as sock:
                sock.bind(("127.0.0.1", 0))
                port = sock.getsockname()[1]
            os.environ["MASTER_ADDR"] = "127.0.0.1"
            os.environ["MASTER_PORT"] = str(port)
            torch.distributed.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=120),
                                                 device_id=device)
        try:
            sharded_info = [run_sharded_sweep(args, world, rank, device, barrier, images)
                            for images in args.sharded_images]
        finally:
            if own_group:
                torch.distributed.destroy_process_group()

    # ---- roofline of the cost kernel (HBM-bound) and the solver figures
    peak, peak_kind = peak_hbm()
    cb = cost_bytes(wl)
    cost_avg_s = statistics.mean(cost_ms) / 1e3 if cost_ms else float("nan")
    achieved = cb / cost_avg_s / 1e9
    traffic = traffic_per_launch()
    roofline = {"kernel": "rfm cost_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_kind == "measured" else "fallback 6.65 TB/s", "traffic": traffic,
                "algorithmic_bytes_per_launch": cb, "avg_launch_us": cost_avg_s * 1e6}
    lb = lsap_bytes(plan)
    lsap_avg_s = statistics.mean(lsap_ms) / 1e3 if lsap_ms else float("nan")
    lsap = {"kernel": "rfm lsap_kernel", "avg_launch_us": lsap_avg_s * 1e6,
            "problems_per_s": problems / lsap_avg_s, "algorithmic_bytes_per_launch": lb,
            "achieved_gbs": lb / lsap_avg_s / 1e9, "share_of_step": (sum(lsap_ms) / total_ms) if total_ms else None,
            "cols_per_lane": plan.plan.cols_per_lane,
            "launch": "persistent warps (layout chosen at launch by batch size)"
            if plan.plan.flags & _lib.PLAN_PERSISTENT else f"{plan.plan.num_ctas} planned CTAs",
            "workspace_bytes": int(plan.plan.workspace_bytes)}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        lap_threads, torch_threads = cpu_baseline_setting()
        r = cpu_path_rate(wl, args.cpu_images, args.cpu_seconds, lap_threads, torch_threads)
        cpu = {"value": r["value"], "unit": UNIT, "cores": lap_threads, "kind": "port",
               "host_cpu_count": os.cpu_count(), "torch_threads": torch_threads,
               "sample": (f"first {r['images']} images of this workload ({r['problems_per_rep']} problems) x "
                          f"{r['reps']} reps in {r['seconds']:.1f} s: torch CPU op chain ({torch_threads} threads) "
                          f"+ SciPy on a {lap_threads}-thread pool (every host thread this process may use; the "
                          f"same setting as --impl reference)")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32 cost, fp64 LSAP duals", "data": "synthetic",
            "config": workload_config(wl), "roofline": roofline, "lsap": lsap, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clocks, "impl": "rfm", "sharded_sweep": sharded_info,
            "graph_replay": {"ms_per_step": graph_max_ms / args.steps,
                             "problems_per_s": world * problems * args.steps / (graph_max_ms / 1e3),
                             "what": "the same step through a captured MatchGraph (one host call per step)"},
            "production_step": production, "box_loss": box_loss, "label_loss": label_loss, "msda": msda,
            "configs": configs,
            "lsap_batches": lsap_batches,
            "library": _lib.version(), "step_ms": step_stats(step_ms), "per_rank_step_ms": per_rank,
            "step_ms_all": [round(x, 5) for x in step_ms], "cost_query_major": cost_qmajor,
        }
        emit(line)
    if world > 1:
        torch.distributed.destroy_process_group()


def e2e_timing(args, wl, plan, device, barrier, world: int, problems: int) -> dict:
    """The headline metric end to end: every step copies its inputs from pinned host memory, matches
    them and reads its packed pairs back, through ``PrefetchingMatcher`` (the upload of step k+1 on its
    own stream while step k is matched)."""
    # pinned buffers on the GPU's own NUMA node (the thread that pins them runs on that node's CPUs),
    # so the uploads do not cross the inter-socket link; the affinity is restored after
    saved_cpus = os.sched_getaffinity(0)
    local_cpus = gpu_local_cpus(device)
    if local_cpus:
        os.sched_setaffinity(0, local_cpus)
    h_logits = wl.pred_logits.pin_memory()
    h_boxes = wl.pred_boxes.pin_memory()
    h_labels = torch.cat([t["labels"] for t in wl.targets]).pin_memory()
    h_tboxes = torch.cat([t["boxes"] for t in wl.targets]).pin_memory()
    h_pairs = torch.empty((2, plan.total_pairs), dtype=torch.int64).pin_memory()
    h2d = sum(int(t.numel() * t.element_size()) for t in (h_logits, h_boxes, h_labels, h_tboxes))
    d2h = int(h_pairs.numel() * h_pairs.element_size())
    from rfdetr_training_throughput_b200.pipeline import PrefetchingMatcher

    pm = PrefetchingMatcher(wl.group_detr, weights=wl.weights, device=device)
    host_batch = (h_logits, h_boxes, h_labels, h_tboxes, tuple(wl.sizes))

    def e2e_run(steps: int) -> None:
        pm.copy_stream.wait_stream(torch.cuda.current_stream(device))
        nxt = pm.prefetch(*host_batch)
        for k in range(steps):
            cur = nxt
            if k + 1 < steps:
                nxt = pm.prefetch(*host_batch)
            res = pm.match(cur)
            h_pairs.copy_(res.pairs, non_blocking=True)

    e2e_run(max(args.warmup, 1))
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    e0.record()
    e2e_run(args.steps)
    e1.record()
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    e2e_t = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(e2e_t, op=torch.distributed.ReduceOp.MAX)
    os.sched_setaffinity(0, saved_cpus)
    ms_step = float(e2e_t.item()) / args.steps
    return {"value": world * problems * args.steps / (float(e2e_t.item()) / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms_step,
            "h2d_gbs_per_gpu": h2d / (ms_step / 1e3) / 1e9,
            "bound": ("host-to-device copy of the step's inputs (PCIe and host memory), not the kernels: the "
                      "device-resident step takes a small fraction of this time"),
            "path": "PrefetchingMatcher: pinned H2D of step k+1 on a copy stream overlapping match + D2H of step k",
            "host_buffers": (f"pinned by a thread on the {len(local_cpus)} GPU-local CPUs NVML reports"
                             if local_cpus else "pinned without NUMA placement (NVML gave no CPU set)")}


def cost_query_major_timing(device, wl, logits, boxes, packed, reps: int = 20) -> dict:
    """The drop-in cost call (``compute_compact_detection_cost_matrix``, the ``triton_matcher`` patch's
    contract: the compact ``[Q, sum T]`` query-major matrix) on the sweep, the kernel alone (C-ABI
    calls back to back between events, behind a device-side delay), and its HBM figure."""
    import ctypes

    from rfdetr_training_throughput_b200 import _lib

    L, B, Q, C = logits.shape
    S = packed.total
    out = torch.empty((L, Q, S), dtype=torch.float32, device=device)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(packed.sizes)]).astype(np.int32), device=device)
    P = ctypes.c_void_p
    stream = P(torch.cuda.current_stream(device).cuda_stream)
    lib = _lib.load()
    w = wl.weights
    args = [P(logits.data_ptr()), P(boxes.data_ptr()), P(packed.labels.data_ptr()), P(packed.boxes.data_ptr()),
            P(offs.data_ptr()), L, B, Q, C, S, S, _lib.LAYOUT_QUERY_MAJOR, float(w["cost_class"]),
            float(w["cost_bbox"]), float(w["cost_giou"]), float(w["focal_alpha"]), P(out.data_ptr()), stream]
    samples = []
    for _ in range(5):
        _lib.check("rfm_cost", lib.rfm_cost(*args))
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        device_lead(device)
        e0.record()
        for _ in range(reps):
            lib.rfm_cost(*args)
        e1.record()
        torch.cuda.synchronize(device)
        samples.append(e0.elapsed_time(e1) * 1e3 / reps)
    us = statistics.median(samples)
    peak, _kind = peak_hbm()
    cb = cost_bytes(wl)
    return {"what": "rfm_cost query-major (the compact [Q, sum T] matrix of the triton_matcher patch), sweep",
            "us_per_launch": us, "achieved_gbs": cb / us / 1e3, "frac_of_hbm": cb / us / 1e3 / peak,
            "timing": f"{reps} launches back to back per sample, median of 5 (no L2 flush between launches)"}


def production_step_timing(device, warmup: int, steps: int = 200) -> dict:
    """The production step (5 decoder layers x 8 images x 13 groups of 300 queries, 520 problems),
    inputs resident, steps issued back to back: wall-clock device time per step through
    ``match_packed`` (host work on every call) and through a captured ``MatchGraph`` replay."""
    from rfdetr_training_throughput_b200 import MatchGraph, matcher, workloads

    wl = workloads.make("step")
    logits, boxes = wl.pred_logits.to(device), wl.pred_boxes.to(device)
    packed = matcher.PackedTargets.from_list(wl.targets_on(device), device)
    graph = MatchGraph(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights, device=device)
    graph.logits.copy_(logits)
    graph.boxes.copy_(boxes)
    graph.labels.copy_(packed.labels)
    graph.tgt_boxes.copy_(packed.boxes)

    def eager():
        matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights)

    out = {"workload": "step: 5 layers x 8 images x 13 groups x 300 queries, 2 classes", "problems": wl.num_problems,
           "steps": steps}
    for name, fn in (("eager", eager), ("graph", graph.replay)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / steps
        out[f"{name}_ms_per_step"] = ms
        out[f"{name}_problems_per_s"] = wl.num_problems / (ms / 1e3)
    return out


def box_loss_timing(device, warmup: int, steps: int = 100) -> dict:
    """The criterion's matched-box losses (L1 + GIoU, forward and backward) on the production step's
    matched pairs: ``matched_box_losses`` (two kernels, no gathers) against the same loss written
    with torch ops the way the DETR-family criterion writes it (index gathers, then the diagonal of
    an N x N GIoU matrix per layer), both on the GPU."""
    from rfdetr_training_throughput_b200 import matcher, workloads
    from rfdetr_training_throughput_b200.loss import matched_box_losses

    wl = workloads.make("step")
    packed = matcher.PackedTargets.from_list(wl.targets_on(device), device)
    pred0 = wl.pred_boxes.to(device)
    res = matcher.match_packed(wl.pred_logits.to(device), pred0, packed, wl.group_detr, weights=wl.weights)
    tgts = [t["boxes"] for t in wl.targets_on(device)]
    per_layer = [res.layer(l) for l in range(wl.layers)]
    batch_idx = [torch.cat([torch.full_like(q, b) for b, (q, _t) in enumerate(p)]) for p in per_layer]
    src_idx = [torch.cat([q for q, _t in p]) for p in per_layer]
    tgt_cat = [torch.cat([tgts[b][t] for b, (_q, t) in enumerate(p)]) for p in per_layer]

    def xyxy(b):
        cx, cy, w, h = b.unbind(-1)
        return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)

    def giou_matrix(b1, b2):
        a1 = (b1[:, 2] - b1[:, 0]) * (b1[:, 3] - b1[:, 1])
        a2 = (b2[:, 2] - b2[:, 0]) * (b2[:, 3] - b2[:, 1])
        wh = (torch.min(b1[:, None, 2:], b2[:, 2:]) - torch.max(b1[:, None, :2], b2[:, :2])).clamp(min=0)
        inter = wh[..., 0] * wh[..., 1]
        union = a1[:, None] + a2 - inter
        wh = (torch.max(b1[:, None, 2:], b2[:, 2:]) - torch.min(b1[:, None, :2], b2[:, :2])).clamp(min=0)
        area = wh[..., 0] * wh[..., 1]
        return inter / union - (area - union) / area

    def torch_ops():
        x = pred0.detach().requires_grad_(True)
        total = 0.0
        for l in range(wl.layers):
            src = x[l][batch_idx[l], src_idx[l]]
            total = total + torch.nn.functional.l1_loss(src, tgt_cat[l], reduction="none").sum()
            total = total + (1 - torch.diag(giou_matrix(xyxy(src), xyxy(tgt_cat[l])))).sum()
        total.backward()

    def fused():
        x = pred0.detach().requires_grad_(True)
        l1, giou = matched_box_losses(x, packed, res)
        (l1.sum() + giou.sum()).backward()

    out = {"workload": "step matched pairs: 5 layers x 8 images x 13 groups", "pairs": int(res.pairs.shape[1]),
           "steps": steps}
    for name, fn in (("rfm", fused), ("torch_ops", torch_ops)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        out[f"{name}_fwd_bwd_us"] = e0.elapsed_time(e1) * 1e3 / steps
    return out


def label_loss_timing(device, warmup: int, sweep_wl, sweep_logits, sweep_boxes, sweep_packed,
                      steps: int = 50) -> dict:
    """The criterion's classification loss (IoU-aware BCE, RF-DETR's default) over the matched pairs,
    forward + backward: ``matched_label_losses`` (two kernels over the logits, positives read from
    the packed pairs) against the torch-op formulation of the same loss (index gathers, a dense
    weight tensor, index_put of the positives), both on the GPU, on the production step; and the
    kernels alone on the sweep's logits with their HBM figure (forward reads the logits, backward
    reads them and writes the gradient)."""
    import torch.nn.functional as F

    from rfdetr_training_throughput_b200 import matcher, workloads
    from rfdetr_training_throughput_b200.loss import matched_label_losses

    wl = workloads.make("step")
    packed = matcher.PackedTargets.from_list(wl.targets_on(device), device)
    logits0, boxes0 = wl.pred_logits.to(device), wl.pred_boxes.to(device)
    res = matcher.match_packed(logits0, boxes0, packed, wl.group_detr, weights=wl.weights)
    tl = [t["labels"] for t in wl.targets_on(device)]
    tb = [t["boxes"] for t in wl.targets_on(device)]
    per_layer = [res.layer(l) for l in range(wl.layers)]
    bidx = [torch.cat([torch.full_like(q, b) for b, (q, _t) in enumerate(p)]) for p in per_layer]
    qidx = [torch.cat([q for q, _t in p]) for p in per_layer]
    cls = [torch.cat([tl[b][t] for b, (_q, t) in enumerate(p)]) for p in per_layer]
    tgt = [torch.cat([tb[b][t] for b, (_q, t) in enumerate(p)]) for p in per_layer]

    def xyxy(b):
        cx, cy, w, h = b.unbind(-1)
        return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)

    def torch_ops():
        x = logits0.detach().requires_grad_(True)
        total = 0.0
        for l in range(wl.layers):
            src = x[l]
            a, b = xyxy(boxes0[l][bidx[l], qidx[l]]), xyxy(tgt[l])
            wh = (torch.min(a[:, 2:], b[:, 2:]) - torch.max(a[:, :2], b[:, :2])).clamp(min=0)
            inter = wh[:, 0] * wh[:, 1]
            area = lambda z: (z[:, 2] - z[:, 0]) * (z[:, 3] - z[:, 1])  # noqa: E731
            iou = inter / (area(a) + area(b) - inter)
            prob = src.sigmoid()
            pos_w = torch.zeros_like(src)
            neg_w = prob ** 2
            t = (prob[bidx[l], qidx[l], cls[l]].pow(0.25) * iou.pow(0.75)).clamp(min=0.01).detach()
            pos_w[bidx[l], qidx[l], cls[l]] = t
            neg_w[bidx[l], qidx[l], cls[l]] = 1 - t
            total = total + (neg_w * src - F.logsigmoid(src) * (pos_w + neg_w)).sum()
        total.backward()

    def fused():
        x = logits0.detach().requires_grad_(True)
        loss, _correct = matched_label_losses(x, boxes0, packed, res, mode="ia_bce")
        loss.sum().backward()

    out = {"workload": "step matched pairs: 5 layers x 8 images x 13 groups, 2 classes", "mode": "ia_bce",
           "pairs": int(res.pairs.shape[1]), "steps": steps}
    for name, fn in (("rfm", fused), ("torch_ops", torch_ops)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        out[f"{name}_fwd_bwd_us"] = e0.elapsed_time(e1) * 1e3 / steps

    # the two kernels alone on the sweep's logits (C-ABI calls back to back between events on the
    # launching stream, behind a device-side delay): forward reads the logits, backward reads them
    # and writes the gradient
    import ctypes

    from rfdetr_training_throughput_b200 import _lib
    from rfdetr_training_throughput_b200.loss import LABEL_LOSS_MODES, _offsets_on

    sres = matcher.match_packed(sweep_logits, sweep_boxes, sweep_packed, sweep_wl.group_detr, weights=sweep_wl.weights)
    L, B, Q, C = sweep_logits.shape
    lib = _lib.load()
    nparts = int(lib.rfm_label_loss_parts(L, B, Q, C))
    parts = torch.empty(nparts, dtype=torch.float32, device=device)
    correct = torch.empty(nparts, dtype=torch.int32, device=device)
    grad = torch.empty_like(sweep_logits)
    gl = torch.ones(L, dtype=torch.float32, device=device)
    P = ctypes.c_void_p
    toff = _offsets_on(sweep_packed.sizes, str(device))
    poff = _offsets_on(sres.per_image_key, str(device))
    common = [P(sweep_logits.data_ptr()), P(sweep_boxes.data_ptr()), P(sweep_packed.labels.data_ptr()),
              P(sweep_packed.boxes.data_ptr()), P(toff.data_ptr()), P(sres.pairs[0].data_ptr()),
              P(sres.pairs[1].data_ptr()), P(poff.data_ptr()), L, B, Q, C, sweep_packed.total,
              LABEL_LOSS_MODES["ia_bce"], 0.25]
    stream = P(torch.cuda.current_stream(device).cuda_stream)

    def fwd():
        _lib.check("rfm_label_loss_forward", lib.rfm_label_loss_forward(*common, P(parts.data_ptr()),
                                                                        P(correct.data_ptr()), stream))

    def bwd():
        _lib.check("rfm_label_loss_backward", lib.rfm_label_loss_backward(*common, P(gl.data_ptr()),
                                                                          P(grad.data_ptr()), stream))

    def per_launch_us(fn, rep: int = 20) -> float:
        samples = []
        for _ in range(7):
            fn()
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            device_lead(device)
            e0.record()
            for _ in range(rep):
                fn()
            e1.record()
            torch.cuda.synchronize(device)
            samples.append(e0.elapsed_time(e1) * 1e3 / rep)
        return statistics.median(samples)

    f_us, b_us = per_launch_us(fwd), per_launch_us(bwd)
    nbytes = sweep_logits.numel() * 4
    peak, _kind = peak_hbm()
    out["sweep"] = {"workload": "sweep logits [1, 1024, 3900, 2] and its 106k matched pairs", "logits_mb": nbytes / 1e6,
                    "forward_us": f_us, "backward_us": b_us, "forward_gbs": nbytes / f_us / 1e3,
                    "backward_gbs": 2 * nbytes / b_us / 1e3, "forward_frac_of_hbm": nbytes / f_us / 1e3 / peak,
                    "backward_frac_of_hbm": 2 * nbytes / b_us / 1e3 / peak,
                    "bytes": "forward reads the logits once; backward reads them and writes the gradient"}
    return out


def msda_timing(device, warmup: int, steps: int = 20) -> dict:
    """Deformable attention (the MSDeformAttn core), forward + backward, fp32, at the reference's
    production geometry (kernels_msda_cuda.py CASES / bench_msda.py: batch 8, 8 heads x 32 channels,
    4 points, levels 36x36 / 18x18 / 9x9; decoder 300 queries, encoder 1701): ``ms_deform_attn``
    (value in the kernel's [B, S, M, D] layout) against the grid_sample formulation rf-detr runs
    when no fused kernel is installed, both on the GPU."""
    import torch.nn.functional as F

    from rfdetr_training_throughput_b200.msda import ms_deform_attn

    shapes_l = [(36, 36), (18, 18), (9, 9)]
    shapes = torch.tensor(shapes_l, device=device, dtype=torch.int64)
    seq = sum(h * w for h, w in shapes_l)

    def grid_sample_core(value_bsmd, loc, w):
        b, _s, m, d = value_bsmd.shape
        q, levels, points = loc.shape[1], loc.shape[3], loc.shape[4]
        v = value_bsmd.permute(0, 2, 3, 1)  # [B, M, D, S], the fallback's layout
        per_level = v.split([h * ww for h, ww in shapes_l], dim=3)
        grids = 2 * loc - 1
        sampled = [F.grid_sample(per_level[i].reshape(b * m, d, h, ww), grids[:, :, :, i].transpose(1, 2).flatten(0, 1),
                                 mode="bilinear", padding_mode="zeros", align_corners=False)
                   for i, (h, ww) in enumerate(shapes_l)]
        wts = w.transpose(1, 2).reshape(b * m, 1, q, levels * points)
        return (torch.stack(sampled, dim=-2).flatten(-2) * wts).sum(-1).view(b, m * d, q).transpose(1, 2)

    out = {"geometry": "batch 8, 8 heads x 32 channels, 4 points, levels 36x36 / 18x18 / 9x9 (sequence 1701)",
           "steps": steps}
    for name, queries in (("decoder", 300), ("encoder", 1701)):
        g = torch.Generator(device=device).manual_seed(7)
        value = torch.randn((8, seq, 8, 32), device=device, generator=g)
        loc = torch.rand((8, queries, 8, 3, 4, 2), device=device, generator=g)
        w = torch.rand((8, queries, 8, 3, 4), device=device, generator=g)
        w = w / w.sum(-1, keepdim=True)
        seed = torch.randn((8, queries, 256), device=device, generator=g)
        entry = {"queries": queries}
        for impl, fn in (("rfm", lambda v, l, ww: ms_deform_attn(v, shapes, None, l, ww)),
                         ("grid_sample", grid_sample_core)):
            vv, ll, wwt = (t.clone().requires_grad_(True) for t in (value, loc, w))

            def run():
                vv.grad = ll.grad = wwt.grad = None
                fn(vv, ll, wwt).backward(seed)

            for _ in range(warmup):
                run()
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                run()
            e1.record()
            torch.cuda.synchronize(device)
            entry[f"{impl}_fwd_bwd_ms"] = e0.elapsed_time(e1) / steps
        entry["speedup"] = entry["grid_sample_fwd_bwd_ms"] / entry["rfm_fwd_bwd_ms"]
        out[name] = entry
    return out


#: The reference's own solver benchmark batches: 520 problems of [300 workers x T tasks] uniform
#: costs (the production step's problem count, kernels_lap.py:50-51,440-473), T across the range
#: it reports, up to its 256-task bound.
LSAP_BATCH_TASKS = (12, 37, 60, 108, 219, 256)


def lsap_batch(tasks: int, device) -> torch.Tensor:
    g = torch.Generator().manual_seed(5000 + tasks)
    return torch.rand((520, 300, tasks), generator=g, dtype=torch.float32).to(device)


def time_solver(fn, cost: torch.Tensor, device, rep: int = 5) -> float:
    """Median ms of one call (2 warm-up calls, then rep calls each between events, behind a delay)."""
    for _ in range(2):
        fn(cost)
    torch.cuda.synchronize(device)
    ms = []
    for _ in range(rep):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        device_lead(device)
        e0.record()
        fn(cost)
        e1.record()
        torch.cuda.synchronize(device)
        ms.append(e0.elapsed_time(e1))
    return statistics.median(ms)


def lsap_batches_rfm(device) -> dict:
    """``batch_linear_assignment`` (the torch_linear_assignment contract behind the cuda_lap patch,
    rfm_lsap_dense) on the reference's solver benchmark batches; the reference arm times the
    reference's own solver on the same batches."""
    from rfdetr_training_throughput_b200 import matcher

    return {f"T{t}": time_solver(matcher.batch_linear_assignment, lsap_batch(t, device), device)
            for t in LSAP_BATCH_TASKS} | {"unit": "ms per 520-problem batch",
                                          "batches": "520 x [300 x T] uniform costs, seed 5000 + T"}


def run_sharded_sweep(args, world: int, rank: int, device, barrier, images: int) -> dict:
    """Strong scaling: one ``images``-image batch split by image over the ranks, every rank matching
    its range, then one all-gather of the packed int64 pairs (NCCL over NVLink).  The headline figure
    is a ``ShardedMatcher`` step: this rank's match replayed as a CUDA graph into the gather's send
    buffer, then the all-gather, the result left in the gathered buffer (``GatheredPairs``: per-image
    views at host-known offsets, no copy).  Beside it, each part timed alone (replay, all-gather,
    the optional flat concatenation) and the eager ``sharded_match`` call.  Every figure is the max
    over ranks of the mean device ms per step, L2 flushed between steps."""
    from rfdetr_training_throughput_b200 import sharded, workloads

    wl = workloads.make(args.workload, images=images)  # the same batch on every rank
    lo, hi = sharded.shard_bounds(wl.images, world)[rank]
    offs = np.concatenate([[0], np.cumsum(wl.sizes)])
    logits = wl.pred_logits[:, lo:hi].to(device)
    boxes = wl.pred_boxes[:, lo:hi].to(device)
    labels = torch.cat([t["labels"] for t in wl.targets])[offs[lo]:offs[hi]].to(device)
    tboxes = torch.cat([t["boxes"] for t in wl.targets])[offs[lo]:offs[hi]].to(device)
    sizes = tuple(wl.sizes)
    steps = max(3, min(args.steps, 50))
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)

    sm = sharded.ShardedMatcher(sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights,
                                device=device)
    sm.graph.logits.copy_(logits)
    sm.graph.boxes.copy_(boxes)
    sm.graph.labels.copy_(labels)
    sm.graph.tgt_boxes.copy_(tboxes)

    def step():
        sm.graph.replay()
        return sm.gather(padded=True)

    def eager():
        return sharded.sharded_match(logits, boxes, labels, tboxes, sizes, wl.group_detr, weights=wl.weights,
                                     padded=True)[0]

    def mean_ms(fn) -> float:
        return statistics.mean(time_device_steps(fn, steps, max(args.warmup, 2), flush, device, barrier))

    parts = {"step": mean_ms(step), "replay": mean_ms(sm.graph.replay), "all_gather": mean_ms(lambda: sm.gather(True)),
             "flat_concat": mean_ms(lambda: sm.gather(True).flat()), "eager_step": mean_ms(eager)}
    same = bool(torch.equal(step().flat(), eager().flat()))

    # the same step with the pushed exchange: the solver stores every pair into every rank's
    # gathered buffer, a one-warp barrier ends the step; one graph replay, no collective
    push_unavailable = None
    try:  # every rank raises together if any rank cannot map the others' buffers
        sp = sharded.ShardedMatcher(sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights,
                                    device=device, exchange="push")
    except RuntimeError as e:
        sp, push_unavailable = None, str(e)
    same_push, push_error = True, 0
    if sp is not None:
        sp.graph.logits.copy_(logits)
        sp.graph.boxes.copy_(boxes)
        sp.graph.labels.copy_(labels)
        sp.graph.tgt_boxes.copy_(tboxes)

        def push_step():
            sp.replay()
            return sp.gather(padded=True)

        parts["push_step"] = mean_ms(push_step)
        same_push = bool(torch.equal(push_step().flat(), step().flat()))
        push_error = sp.exchange.error()
        sp.close()
    t = torch.tensor(list(parts.values()) + [0.0 if same_push else 1.0, float(push_error)], dtype=torch.float64,
                     device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    vals = t.tolist()
    ms = dict(zip(parts.keys(), vals))
    push_mismatch, push_error = vals[-2] > 0, int(vals[-1])
    gathered_pairs = int(sum(sm.shard.counts))
    # bytes one rank's pushes send over NVLink (16 per pair to each other rank), the largest rank's
    nvlink_bytes = max(16 * int(c) * (world - 1) for c in sm.shard.counts)
    del sm  # its graph holds no collective, but release it before the process group goes
    if push_unavailable is not None:
        push_info = {"unavailable": push_unavailable}
    else:
        push_info = {"ms_per_step": ms["push_step"], "problems_per_s": wl.num_problems / (ms["push_step"] / 1e3),
                     "equals_all_gather_on_every_rank": not push_mismatch, "barrier_gave_up": bool(push_error),
                     "nvlink_bytes_per_rank": nvlink_bytes,
                     "nvlink_floor_ms": nvlink_bytes / (PEER_COPY_GBS * 1e9) * 1e3,
                     "over_replay_ms": ms["push_step"] - ms["replay"],
                     "exchange": "the solver stores every pair into every rank's gathered buffer (CUDA IPC peer "
                                 "mappings, plain stores over NVLink), then a one-warp flag barrier; one graph "
                                 "replay per step, no collective"}
    return {"images": wl.images, "problems_per_step": wl.num_problems, "steps": steps,
            "ms_per_step": ms["step"], "problems_per_s": wl.num_problems / (ms["step"] / 1e3),
            "breakdown_ms": {"replay": ms["replay"], "all_gather": ms["all_gather"],
                             "all_gather_plus_flat_concat": ms["flat_concat"]},
            "best_exchange": "push" if ms.get("push_step", float("inf")) < ms["step"] else "nccl",
            "best_problems_per_s": wl.num_problems / (min(ms.get("push_step", float("inf")), ms["step"]) / 1e3),
            "eager_ms_per_step": ms["eager_step"], "eager_problems_per_s": wl.num_problems / (ms["eager_step"] / 1e3),
            "graph_equals_eager": same, "gathered_pairs": gathered_pairs, "scaling": "strong",
            "push": push_info,
            "result": "GatheredPairs (the all-gather's buffer, per-image views at host-known offsets)",
            "collective": "all_gather_into_tensor of int64 [2, width] per rank" if world > 1 else "none (1 rank)"}


_RESULT_FD: list = [None]


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's original stdout."""
    fd = _RESULT_FD[0]
    text = json.dumps(line) + "\n"
    if fd is None:
        sys.stdout.write(text)
        sys.stdout.flush()
    else:
        os.write(fd, text.encode())


def run_kernel(name: str, workload: str = "sweep", images: int | None = None) -> None:
    """A few launches of one kernel on its benchmark workload, for an ncu capture of that kernel:
    cost / lsap (the workload's step, issued as two calls), cost_qm (the drop-in query-major cost
    matrix, ``compute_compact_detection_cost_matrix``), label / box (the classification or the
    matched-box loss, forward and backward, on the workload's pairs), msda (deformable attention
    forward and backward, decoder geometry), lsap_push (the sharded step with the pushed exchange on
    a one-rank group: the solver with its push epilogue, replayed as a graph)."""
    from rfdetr_training_throughput_b200 import matcher, workloads

    dev = torch.device("cuda", 0)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    if name == "lsap_push":
        import socket

        from rfdetr_training_throughput_b200 import sharded

        with socket.socket() as sock:
            sock.bind(("127.0.0.1", 0))
            port = sock.getsockname()[1]
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.distributed.init_process_group("nccl", rank=0, world_size=1, device_id=dev)
        try:
            wl = workloads.make(workload, images=images)
            sm = sharded.ShardedMatcher(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr,
                                        weights=wl.weights, device=dev, exchange="push")
            sm.graph.logits.copy_(wl.pred_logits.to(dev))
            sm.graph.boxes.copy_(wl.pred_boxes.to(dev))
            pk = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
            sm.graph.labels.copy_(pk.labels)
            sm.graph.tgt_boxes.copy_(pk.boxes)
            for _ in range(4):
                sm.replay()
                flush.zero_()
            torch.cuda.synchronize()
            sm.check()
            sm.close()
        finally:
            torch.distributed.destroy_process_group()
        print("kernel lsap_push: ok")
        return
    if name == "cost_qm":
        wl = workloads.make(workload, images=images)
        lg, bx = wl.pred_logits.to(dev), wl.pred_boxes.to(dev)
        tg = wl.targets_on(dev)
        for _ in range(4):
            matcher.compute_compact_detection_cost_matrix({"pred_logits": lg, "pred_boxes": bx}, tg,
                                                         weights=wl.weights)
            flush.zero_()
    elif name in ("cost", "lsap", "label", "box"):
        wl = workloads.make(workload, images=images)
        lg, bx = wl.pred_logits.to(dev), wl.pred_boxes.to(dev)
        pk = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
        for _ in range(4):
            res = matcher.match_packed(lg, bx, pk, wl.group_detr, weights=wl.weights, events={})
            flush.zero_()
        if name == "box":
            from rfdetr_training_throughput_b200.loss import matched_box_losses

            b = bx.clone().requires_grad_(True)
            for _ in range(3):
                b.grad = None
                l1, giou = matched_box_losses(b, pk, res)
                (l1.sum() + giou.sum()).backward()
                flush.zero_()
        if name == "label":
            from rfdetr_training_throughput_b200.loss import matched_label_losses

            x = lg.clone().requires_grad_(True)
            for _ in range(3):
                x.grad = None
                loss, _c = matched_label_losses(x, bx, pk, res, mode="ia_bce")
                loss.sum().backward()
                flush.zero_()
    else:
        from rfdetr_training_throughput_b200.msda import ms_deform_attn

        g = torch.Generator(device="cuda").manual_seed(7)
        shapes = torch.tensor([(36, 36), (18, 18), (9, 9)], device=dev)
        v = torch.randn((8, 1701, 8, 32), device=dev, generator=g).requires_grad_(True)
        loc = torch.rand((8, 300, 8, 3, 4, 2), device=dev, generator=g).requires_grad_(True)
        w = torch.rand((8, 300, 8, 3, 4), device=dev, generator=g).requires_grad_(True)
        for _ in range(3):
            ms_deform_attn(v, shapes, None, loc, w).sum().backward()
    torch.cuda.synchronize(dev)
    print(f"kernel {name}: ok", file=sys.stderr)


def main() -> None:
    args = parse()
    if args.kernel is not None:
        run_kernel(args.kernel, args.workload, args.images)
        return
    # Everything else anything in the process writes to stdout (library banners such as NCCL's
    # version line under torchrun) goes to stderr, so stdout carries the JSON line alone.
    sys.stdout.flush()
    _RESULT_FD[0] = os.dup(1)
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_rfm(args)


if __name__ == "__main__":
    main()
