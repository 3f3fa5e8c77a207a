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


def traffic_key(workload: str, world: int) -> str:
    """Profiles record traffic per workload and GPU count: the dominant
    kernel's per-launch bytes change with the tensor-parallel degree."""
    return workload if world == 1 else f"{workload}@n{world}"


def blas_threads(threads: int):
    """Size numpy's BLAS pool explicitly (torchrun exports OMP_NUM_THREADS=1,
    which would otherwise leave the CPU baseline on one core at N>1) and
    return (context manager, threads actually in use)."""
    import numpy  # noqa: F401  (loads the BLAS library the limit applies to)
    from threadpoolctl import threadpool_info, threadpool_limits
    ctx = threadpool_limits(limits=threads, user_api="blas")
    got = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
    return ctx, (max(got) if got else threads)


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


from metalbench_b200.clocks import ClockSampler  # noqa: E402


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
class Workload:
    name = ""
    metric = ""
    unit = ""
    dtype = ""
    bound = "hbm"
    scaling = "weak"
    config: dict = {}

    def job_units(self, world: int) -> float:
        """Whole-job metric numerator per step: weak scaling adds every rank's
        work, strong scaling splits one job across the ranks."""
        return self.work_per_step() * (world if self.scaling == "weak" else 1)

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

    def setup(self, torch, rank, world, local):
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


class DecoderStackDecode(Workload):
    """8-layer LLaMA decoder stack: d_model 8192, 64 query /
    8 kv heads, head_dim 128, SwiGLU FFN 28672, RMSNorm eps 1e-5, RoPE theta 5e5,
    weights N(0, 0.02) seed 4; decode batch 64 at KV length 8192, tensor-parallel
    over the GPUs. One step = one new token for each of the 64 sequences through
    all 8 layers (a CUDA-graph replay). Every step writes its token at position
    8192 and attends over 8193 keys, so all steps cost the same."""
    name = "decoder_stack_decode"
    metric = "8-layer LLaMA decoder decode throughput (tokens/s)"
    unit = "tok/s"
    dtype = "bf16"
    bound = "hbm"
    scaling = "strong"
    default_steps = 100
    B, L, LAYERS = 64, 8192, 8
    D, H, HKV, FF = 8192, 64, 8, 28672

    def __init__(self):
        self.config = {"workload": "decoder_stack_decode", "model": "llama-8layer-d8192",
                       "d_model": self.D, "n_heads": self.H, "n_kv_heads": self.HKV,
                       "head_dim": 128, "ffn": self.FF, "layers": self.LAYERS,
                       "global_batch": self.B, "kv_len": self.L, "rope_theta": 500000.0,
                       "weights": "N(0,0.02) seed 4, random init", "kv_cache": "N(0,1) fill",
                       "l2": "inputs larger than L2 (17 GB KV + 13.7 GB weights per step at 1 GPU)"}

    def setup(self, torch, rank, world, local):
        from metalbench_b200.decoder import DecoderConfig
        from metalbench_b200.stack import DecoderStack, init_tensor_parallel
        self.torch = torch
        self.config["parallelism"] = f"tp{world}"
        init_tensor_parallel(rank, world, local)
        cfg = DecoderConfig(self.D, self.H, self.HKV, self.FF, rope_base=500000.0)
        self.stack = DecoderStack(cfg, self.LAYERS, self.B, self.L + 64, tp_rank=rank,
                                  tp_world=world)
        self.stack.fill_cache_random(self.L)
        g = torch.Generator(device="cuda").manual_seed(4)
        self.x = torch.randn((self.B, 1, self.D), generator=g, device="cuda").bfloat16()
        self.sp = torch.full((self.B,), self.L, dtype=torch.int32, device="cuda")
        self.stack.capture_decode(self.x, self.sp, self.L + 1)
        self.h_x = torch.empty((self.B, 1, self.D), dtype=torch.bfloat16, pin_memory=True)
        self.h_x.copy_(self.x.cpu())
        self.h_y = torch.empty((self.B, 1, self.D), dtype=torch.bfloat16, pin_memory=True)
        # dominant kernel: decode attention of one layer, driven directly
        from metalbench_b200 import _lib, ops
        self._lib, self._ops = _lib, ops
        c = self.stack.caches[0]
        self.hq, self.hkv = self.H // world, self.HKV // world
        self.q = torch.randn((self.B, self.hq * 128), device="cuda").bfloat16()
        self.ao = torch.empty_like(self.q)
        self.kvl = self.sp + 1
        self.aws_bytes = _lib.lib().mb_attention_decode_workspace_bytes(self.B, self.hq,
                                                                         self.hkv, self.L + 1)
        self.aws = torch.empty(self.aws_bytes, dtype=torch.uint8, device="cuda")
        self.cache0 = c

    def step(self):
        self.stack.replay()

    def launch_dominant(self):
        c = self.cache0
        self._lib.call("mb_attention_decode_bf16", self.q.data_ptr(), self.hq * 128,
                       c.k.data_ptr(), c.v.data_ptr(), c.block_table.data_ptr(), c.max_pages,
                       self.kvl.data_ptr(), self.L + 1, self.B, self.hq, self.hkv, 128,
                       self.ao.data_ptr(), self.hq * 128, self.aws.data_ptr(), self.aws_bytes,
                       self._ops._stream())

    dominant = "attn_decode_mma_kernel (one layer's KV read)"

    def work_per_step(self):
        return float(self.B)  # tokens

    def roofline_work(self):
        return 2.0 * self.B * (self.L + 1) * self.hkv * 128 * 2  # K and V bytes read

    def e2e_step(self):
        self.x.copy_(self.h_x, non_blocking=True)
        y = self.stack.replay()
        self.h_y.copy_(y, non_blocking=True)

    def e2e_bytes(self):
        return self.B * self.D * 2, self.B * self.D * 2

    def cpu_sample(self, threads):
        """One layer of the stack on the CPU oracle for 8 of the 64 sequences
        (KV 8192), extrapolated to 8 layers: tok/s = 8 / (8 * t_layer)."""
        import numpy as np
        import oracle.ops as O
        rng = np.random.default_rng(4)
        D, H, HKV, FF, Bs = self.D, self.H, self.HKV, self.FF, 8
        W = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)
             for s in [(D, D + 2 * HKV * 128), (D, D), (D, 2 * FF), (FF, D)]]
        kp = rng.standard_normal((Bs, HKV, self.L, 128), dtype=np.float32)
        vp = rng.standard_normal((Bs, HKV, self.L, 128), dtype=np.float32)
        x = rng.standard_normal((Bs, 1, D), dtype=np.float32)
        kw = dict(H=H, H_kv=HKV, base=500000.0, causal=True, k_past=kp, v_past=vp)
        O.decoder_layer(x, *W, **kw)  # warm
        t0, n = time.perf_counter(), 0
        while n < 1 or time.perf_counter() - t0 < 10.0:
            O.decoder_layer(x, *W, **kw)
            n += 1
        t_layer = (time.perf_counter() - t0) / n
        return Bs / (self.LAYERS * t_layer), (
            f"numpy oracle, 1 of 8 layers x {n} runs for {Bs} of 64 sequences at KV 8192 "
            f"(fp32, {threads} BLAS threads), extrapolated x8 layers")


class ShardedGemm(Workload):
    """bf16 GEMM C = A @ B at 16384^3 ("a sharded bf16 GEMM
    16384x16384x16384"), A, B ~ N(0,1) seed 4, column-sharded over the GPUs:
    rank r holds all of A and the column block B[:, r*N/P:(r+1)*N/P] and
    computes its block of C (no collective on the hot path). Strong scaling:
    the job is one 16384^3 product at every N."""
    name = "gemm_bf16_16384"
    metric = "sharded bf16 GEMM 16384^3 throughput"
    unit = "TFLOP/s"
    dtype = "bf16"
    bound = "tensor"
    scaling = "strong"
    default_steps = 20
    M = N = K = 16384

    def __init__(self):
        self.config = {"workload": "gemm_bf16_16384", "M": self.M, "N": self.N, "K": self.K,
                       "layout": "A [M,K] row-major, B [K,N] row-major (column block per rank)",
                       "l2": "inputs larger than L2 (512 MiB per operand)"}

    def setup(self, torch, rank, world, local):
        from metalbench_b200 import ops
        self.ops, self.torch = ops, torch
        self.config["parallelism"] = f"column-shard x{world}"
        self.nloc = self.N // world
        g = torch.Generator(device="cuda").manual_seed(4)
        self.a = torch.randn((self.M, self.K), generator=g, device="cuda").bfloat16()
        b = torch.randn((self.K, self.N), generator=g, device="cuda").bfloat16()
        self.b = b[:, rank * self.nloc:(rank + 1) * self.nloc].contiguous()
        del b
        self.c = torch.empty((self.M, self.nloc), device="cuda", dtype=torch.bfloat16)
        self.h_a = torch.empty_like(self.a, device="cpu").pin_memory()
        self.h_a.copy_(self.a)
        self.h_b = torch.empty_like(self.b, device="cpu").pin_memory()
        self.h_b.copy_(self.b)
        self.h_c = torch.empty_like(self.c, device="cpu").pin_memory()
        torch.cuda.empty_cache()

    def step(self):
        self.ops.gemm_bf16(self.a, self.b, self.c, b_layout="kn")

    launch_dominant = step
    dominant = "gemm_kernel<256,4,GemmProducer<bf16,256,MN-major B>> (this rank's column block)"

    def work_per_step(self):
        return 2.0 * self.M * self.N * self.K / 1e12  # TFLOP per step (whole job)

    def job_units(self, world):
        return self.work_per_step()

    def roofline_work(self):
        return 2.0 * self.M * self.nloc * self.K  # FLOP per launch on this rank

    def e2e_step(self):
        self.a.copy_(self.h_a, non_blocking=True)
        self.b.copy_(self.h_b, non_blocking=True)
        self.step()
        self.h_c.copy_(self.c, non_blocking=True)

    def e2e_bytes(self):
        return self.a.numel() * 2 + self.b.numel() * 2, self.c.numel() * 2

    def cpu_sample(self, threads):
        """numpy fp32 GEMM on 2048 rows of A (the full B), scaled to TFLOP/s."""
        import numpy as np
        import oracle.ops as O
        rng = np.random.default_rng(4)
        a = rng.standard_normal((2048, self.K), dtype=np.float32)
        b = rng.standard_normal((self.K, 2048), dtype=np.float32)
        O.sqr_mm(a, b, acc=np.float32)
        t0, n = time.perf_counter(), 0
        while n < 1 or time.perf_counter() - t0 < 10.0:
            O.sqr_mm(a, b, acc=np.float32)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return 2.0 * 2048 * 2048 * self.K / dt / 1e12, (
            f"numpy fp32 GEMM 2048x{self.K}x2048 (a 1/64 slice of the job), {n} runs, "
            f"{threads} BLAS threads")


WORKLOADS = {"transpose": TransposeF32, "decoder_stack": DecoderStackDecode,
             "gemm": ShardedGemm}
DEFAULT_WORKLOAD = "decoder_stack"


def count_our_launches(torch, fn) -> dict:
    """Kernels one step launches, from a CUDA-activity trace: ours (libmb200),
    NCCL's and torch's (index arithmetic around our calls)."""
    fn()
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as p:
        fn()
        torch.cuda.synchronize()
    out = {"ours": 0, "nccl": 0, "torch": 0}
    for e in p.events():
        if getattr(e, "device_type", None) is None or "cuda" not in str(e.device_type).lower():
            continue
        n = e.name
        if n.startswith("Memcpy") or n.startswith("Memset"):
            continue
        if "nccl" in n.lower():
            out["nccl"] += 1
        elif n.startswith("void at::") or n.startswith("at::") or "at::native" in n:
            out["torch"] += 1
        else:
            out["ours"] += 1
    return out


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
    ctx, threads = blas_threads(threads)
    vals, sample = [], ""
    with ctx:
        for i in range(args.warmup + args.steps):  # each step is a bounded sample
            v, sample = wl.cpu_sample(threads)
            if i >= args.warmup:
                vals.append(v)
    value = statistics.median(vals)
    line = {"metric": wl.metric, "value": value, "unit": wl.unit, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
            "dtype": wl.dtype, "data": "synthetic", "config": wl.config,
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
    wl.setup(torch, rank, world, local)
    n_launch = count_our_launches(torch, wl.step)

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
    value = wl.job_units(world) / (ms_total / 1e3 / args.steps)

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
        # a multi-millisecond GEMM runs under the power cap: sustained figure
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) \
            if launch_ms > 2.0 else peaks["bf16_tflops"]
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
    e2e_value = wl.job_units(world) / (e2e_ms / 1e3)
    h2d, d2h = wl.e2e_bytes()

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        ctx, threads = blas_threads(os.cpu_count() or 1)
        with ctx:
            v, sample = wl.cpu_sample(threads)
        cpu = {"value": v, "unit": wl.unit, "cores": threads, "kind": "port", "sample": sample}
    line = {
        "metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype,
        "data": "synthetic", "config": wl.config,
        "roofline": {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": r_unit,
                     "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)"
                     if peak_kind == "measured" else "fallback",
                     "traffic": profile_traffic(traffic_key(wl.name, world)), "launch_ms": launch_ms,
                     "kernel": getattr(wl, "dominant", wl.name)},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": n_launch["ours"] * args.steps,
        "gpu_launches_detail": {"per_step": n_launch, "timed_steps": args.steps},
        "clocks": sampler.summary() if sampler else None,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
