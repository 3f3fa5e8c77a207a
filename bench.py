#!/usr/bin/env python3
"""MetalBench-B200 headline benchmark (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A "step" is one pass of the hot path over one batch of synthetic input. The
timed region is exactly K steps bracketed by a barrier and a device
synchronise on both sides; the time is measured with CUDA events on the launch
stream and the maximum over ranks is reported. Inputs are larger than the
126 MB L2 for every workload whose config says so; the others flush L2 between
steps (said in ``config.l2``).

``--impl reference`` times the reference algorithm's CPU implementation on
this host's cores (the numpy oracle port, threaded over blocks: MLX and its
Metal path do not exist on Linux) for the same metric and config, on a
bounded sample of the workload.
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

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_PATH = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    try:
        p = json.loads(PEAKS_PATH.read_text())
        return p, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(key: str):
    """dram bytes per launch recorded by an ncu capture summary under profiles/
    (a line ``traffic_bytes_per_launch[<key>]: <int>``), or None."""
    for f in sorted((REPO / "profiles").glob("*.md")) + sorted((REPO / "profiles").glob("*.txt")):
        for line in f.read_text().splitlines():
            tag = f"traffic_bytes_per_launch[{key}]:"
            if line.strip().startswith(tag):
                try:
                    return int(float(line.split(":", 1)[1].strip()))
                except ValueError:
                    return None
    return None


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
class Workload:
    name = ""
    metric = ""
    unit = ""
    dtype = ""
    bound = "hbm"
    config: dict = {}

    def setup(self, torch, rank, world): ...
    def step(self): ...                  # one step on the current stream
    def work_per_step(self) -> float: ...  # metric numerator per rank per step
    def roofline_work(self) -> float: ...  # algorithmic bytes or FLOPs per dominant launch
    def launch_dominant(self): ...       # one launch of the dominant kernel
    def kernels_per_step(self) -> int: return 1
    def e2e_step(self): ...              # H2D inputs, step, D2H result
    def e2e_bytes(self): ...             # (h2d, d2h) per step
    def cpu_sample(self, threads): ...   # -> (value in unit, sample description)


class TransposeF32(Workload):
    """transpose fp32 8192x8192: HBM GB/s = read+write bytes / s."""
    name = "transpose_2d_f32_8192"
    metric = "transpose_2d fp32 8192x8192 HBM throughput"
    unit = "GB/s"
    dtype = "f32"
    bound = "hbm"
    R = C = 8192

    def __init__(self):
        self.config = {"workload": "transpose_2d", "shape": [self.R, self.C], "dtype": "fp32",
                       "l2": "inputs larger than L2 (256 MiB in, 256 MiB out)",
                       "parallelism": "replicas (one independent matrix per GPU)"}

    def setup(self, torch, rank, world):
        from metalbench_b200 import ops
        self.torch, self.ops = torch, ops
        g = torch.Generator(device="cuda").manual_seed(1 + rank)
        self.a = torch.rand((self.R, self.C), device="cuda", generator=g) * 2 - 1
        self.out = torch.empty((self.C, self.R), device="cuda")
        self.h_in = torch.empty((self.R, self.C), pin_memory=True)
        self.h_in.copy_(self.a.cpu())
        self.h_out = torch.empty((self.C, self.R), pin_memory=True)

    def step(self):
        self.ops.transpose_2d(self.a, self.out)

    launch_dominant = step

    def work_per_step(self):
        return 2.0 * self.R * self.C * 4 / 1e9  # GB

    def roofline_work(self):
        return 2.0 * self.R * self.C * 4  # bytes

    def e2e_step(self):
        self.a.copy_(self.h_in, non_blocking=True)
        self.ops.transpose_2d(self.a, self.out)
        self.h_out.copy_(self.out, non_blocking=True)

    def e2e_bytes(self):
        return self.R * self.C * 4, self.R * self.C * 4

    def cpu_sample(self, threads):
        import numpy as np
        import oracle.ops as O
        from concurrent.futures import ThreadPoolExecutor
        a = np.random.default_rng(1).uniform(-1, 1, (self.R, self.C)).astype(np.float32)
        out = np.empty((self.C, self.R), np.float32)
        blocks = [(i, min(i + 512, self.R)) for i in range(0, self.R, 512)]

        def blk(b):
            out[:, b[0]:b[1]] = O.transpose_2d(a[b[0]:b[1]])

        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(blk, blocks))  # warm
            t0, n = time.perf_counter(), 0
            while time.perf_counter() - t0 < 10.0:
                list(ex.map(blk, blocks))
                n += 1
            dt = time.perf_counter() - t0
        return n * self.work_per_step() / dt, f"{n} full 8192x8192 fp32 transposes (~10 s), " \
                                              f"512-row blocks over {threads} threads"


WORKLOADS = {"transpose": TransposeF32}
DEFAULT_WORKLOAD = "transpose"


# ---------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def run_reference(args, wl):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    vals, sample = [], ""
    for i in range(args.warmup + args.steps):  # each step is a bounded sample
        v, sample = wl.cpu_sample(threads)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {"metric": wl.metric, "value": value, "unit": wl.unit, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic", "config": wl.config,
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    wl = WORKLOADS[args.workload]()
    if args.impl == "reference":
        args.steps = args.steps or 1
        args.warmup = 0 if args.warmup is None else args.warmup
        return run_reference(args, wl)
    args.steps = args.steps or getattr(wl, "default_steps", 2000)
    args.warmup = max(3, args.warmup if args.warmup is not None else 20)

    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from metalbench_b200 import ops
    ops.init(local)
    wl.setup(torch, rank, world)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    # ---- timed region: exactly K steps -------------------------------------
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        wl.step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_total = max_over_ranks(e0.elapsed_time(e1))
    if sampler:
        sampler.stop()
    ms_step = ms_total / args.steps
    value = wl.work_per_step() * world / (ms_total / 1e3 / args.steps)

    # ---- dominant kernel: per-launch CUDA-event duration --------------------
    nl = min(200, max(20, args.steps))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(nl)]
    for a, b in ev:
        a.record(stream)
        wl.launch_dominant()
        b.record(stream)
    torch.cuda.synchronize()
    launch_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    peaks, peak_kind = load_peaks()
    if wl.bound == "hbm":
        achieved = wl.roofline_work() / (launch_ms / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
        r_unit = "GB/s"
    else:
        achieved = wl.roofline_work() / (launch_ms / 1e3) / 1e12
        peak = peaks["bf16_tflops"]
        r_unit = "TFLOP/s"

    # ---- end to end through the public API (pinned host in, host out) ------
    ne = max(3, min(20, args.steps))
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(stream)
    for _ in range(ne):
        wl.e2e_step()
    x1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(x0.elapsed_time(x1)) / ne
    e2e_value = wl.work_per_step() * world / (e2e_ms / 1e3)
    h2d, d2h = wl.e2e_bytes()

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample = wl.cpu_sample(threads)
        cpu = {"value": v, "unit": wl.unit, "cores": threads, "kind": "port", "sample": sample}
    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic", "config": wl.config,
        "roofline": {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": r_unit,
                     "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)"
                     if peak_kind == "measured" else "fallback",
                     "traffic": profile_traffic(wl.name), "launch_ms": launch_ms},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": wl.kernels_per_step() * args.steps,
        "clocks": sampler.summary() if sampler else None,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
